"""The fused local block (asrn_local_block: LN kernel + three persistent tcgen05 GEMMs with the causal conv, GELU, bias
and residual folded in) against the same BloqueLocal run as PyTorch ops under bf16 autocast, and the model forward
with fused blocks against the model with PyTorch blocks.

Bar: the block's increment h' - h within 2e-2 of max|h' - h| (bf16 autocast: the two differ only where a bf16
rounding of an intermediate falls the other way), logits within 2e-2."""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _block(d, k, ff, seed):
    from asrn_b200.model import BloqueLocal
    torch.manual_seed(seed)
    blq = BloqueLocal(d, k, ff)
    with torch.no_grad():                        # LayerNorm parameters off their (1, 0) start so every term counts
        for ln in (blq.ln1, blq.ln2):
            ln.weight.add_(torch.randn_like(ln.weight) * 0.2)
            ln.bias.add_(torch.randn_like(ln.bias) * 0.2)
    return blq


@pytest.mark.parametrize('B,L,d,k,ff', [(2, 300, 256, 4, 512), (1, 8192, 768, 4, 1536), (3, 129, 128, 3, 256),
                                        (2, 1, 128, 4, 128), (1, 77, 384, 5, 640)])
def test_fused_block_matches_pytorch_block(B, L, d, k, ff, cuda, monkeypatch):
    blq = _block(d, k, ff, 1).to(cuda).eval()
    g = torch.Generator().manual_seed(2)
    h = (torch.randn(B, L, d, generator=g) * 2).to(cuda)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
        assert blq._fused_ok(h)
        fused = blq(h)
        fused2 = blq(h)
        monkeypatch.setattr(type(blq), '_fused_ok', lambda self, x: False)
        ref = blq(h)
    assert fused.dtype == torch.float32 and fused.shape == h.shape
    assert torch.equal(fused, fused2)            # no atomics: the fused block is deterministic
    assert rel_err((fused - h).cpu().numpy(), (ref - h).cpu().numpy()) <= 2e-2


def test_fused_block_is_causal(cuda):
    """Changing position t changes no output before t (the conv's taps reach back only)."""
    blq = _block(256, 4, 512, 3).to(cuda).eval()
    g = torch.Generator().manual_seed(4)
    h = torch.randn(1, 500, 256, generator=g).to(cuda)
    h2 = h.clone()
    h2[0, 250] += 3.0
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
        a, b = blq(h), blq(h2)
    assert torch.equal(a[0, :250], b[0, :250]) and not torch.equal(a[0, 250:254], b[0, 250:254])


def test_model_with_fused_blocks_matches_pytorch_blocks(cuda, monkeypatch):
    import asrn_b200
    from asrn_b200.model import BloqueLocal
    m = asrn_b200.create_model(V=1000, d=256, n_capas=4, semilla=5).to(cuda).eval()
    x = torch.from_numpy(np.random.default_rng(1).integers(0, 1000, (2, 600))).to(cuda)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
        fused = m(x).float()
        monkeypatch.setattr(BloqueLocal, '_fused_ok', lambda self, h: False)
        ref = m(x).float()
    assert rel_err(fused.cpu().numpy(), ref.cpu().numpy()) <= 2e-2
