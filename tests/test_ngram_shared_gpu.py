"""The n-gram sort shared by the ASRN layers of a model (asrn_ngram_shared_sort / asrn_layer_forward_ngram): the layer
output with a shared sort equals its own-sort output (rows sorted in one block and tiled long rows), a model forward
that sorts once equals one that sorts in every layer, and a sort made for other tokens is refused.

The sort and scans give identical results either way; the layer's table sum (L2 reductions in an order that varies
from run to run) makes two forwards differ in their last bits, so outputs are compared within four times the spread of two
own-sort forwards, and within the parity bars (1e-5 fp32, 2e-2 bf16 of max|h' - h|)."""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _layer(d, seed=0):
    import asrn_b200
    torch.manual_seed(seed)
    layer = asrn_b200.ASRNLayer(d)
    with torch.no_grad():                        # move the neutral parameters off zero so every term counts
        layer.u_hawkes.normal_(0, 0.5)
        layer.w_vistos.normal_(0, 0.5)
        layer.d_racha.normal_(0, 0.3)
        layer.log_kappa.add_(torch.randn_like(layer.log_kappa) * 0.3)
    return layer


def _inputs(B, L, d, V, seed, cuda):
    from asrn_b200 import synthetic
    g = torch.Generator().manual_seed(seed)
    x = torch.from_numpy(synthetic.config_tokens('cfg3', B=B, L=L, seed=seed) % V).to(cuda)
    E = (torch.randn(B, L, d, generator=g) * 0.5).to(cuda)
    h = torch.randn(B, L, d, generator=g).to(cuda)
    return x, E, h


@pytest.mark.parametrize('B,L,half', [(2, 3000, False), (3, 8192, True), (1, 20000, True), (2, 1, False)])
def test_layer_with_shared_sort_equals_own_sort(B, L, half, cuda):
    d = 64
    layer = _layer(d).to(cuda).eval()
    x, E, h = _inputs(B, L, d, 300, 1, cuda)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
        own = layer(E, h, x)
        own2 = layer(E, h, x)
        ng = layer.ngram_sort(x)
        shared = layer(E, h, x, ngram=ng)
    y_own, y_own2, y_sh = ((t - h).float().cpu().numpy() for t in (own, own2, shared))
    spread = rel_err(y_own2, y_own)
    assert rel_err(y_sh, y_own) <= max(4 * spread, 1e-6)
    assert rel_err(y_sh, y_own) <= (2e-2 if half else 1e-5)


def test_shared_sort_for_other_tokens_is_refused(cuda):
    layer = _layer(64).to(cuda).eval()
    x, E, h = _inputs(1, 100, 64, 50, 2, cuda)
    ng = layer.ngram_sort(x)
    with torch.no_grad(), pytest.raises(ValueError):
        layer(E, h, (x + 1) % 50, ngram=ng)
    with torch.no_grad(), pytest.raises(ValueError):
        layer(E[:, :50], h[:, :50], x[:, :50], ngram=ng)


@pytest.mark.parametrize('half', [False, True])
def test_model_forward_sorts_once_and_equals_per_layer_sorts(half, cuda, monkeypatch):
    import asrn_b200
    m = asrn_b200.create_model(V=512, d=64, n_capas=6, semilla=3).to(cuda).eval()
    x = torch.from_numpy(np.random.default_rng(0).integers(0, 512, (2, 700))).to(cuda)
    calls = []
    orig = type(m.largos[0]).ngram_sort

    def counting(self, piezas):
        calls.append(1)
        return orig(self, piezas)

    monkeypatch.setattr(type(m.largos[0]), 'ngram_sort', counting)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
        shared = m(x)
        assert len(calls) == 1 and len(m.largos) == 3
        monkeypatch.setattr(type(m), '_ngram_shared', lambda self: False)
        own = m(x)
        own2 = m(x)
    assert len(calls) == 1
    spread = rel_err(own2.float().cpu().numpy(), own.float().cpu().numpy())
    err = rel_err(shared.float().cpu().numpy(), own.float().cpu().numpy())
    assert err <= max(4 * spread, 1e-6) and err <= (2e-2 if half else 1e-4)
