"""Training kernels against the reference's own autograd (fixtures tests/golden/grad_*.npz, written by
tests/golden/make_golden.py from asrn/estable.py:204-263 and asrn/nucleo.py:188-197, 518-537 on the CPU):
BucketAttention (asrn_bucket_attn_forward / _backward) and escaneo (asrn_scan_forward / _backward).

Bars: fp32 -- the attention output within 1e-5 of max|salida|, the signals' hay exact and max / peak within 1e-5
where a key is valid, every gradient within 1e-4 of its max (sums of up to 2C terms per slot, then over the tables,
in another order); bf16 operands -- output and gradients within 3e-2 (att and dS rounded to bf16 before their
products, as the reference's kernel does). The backward is deterministic (no atomics): two runs are bit-equal."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu


def _fixture(name):
    z = np.load(os.path.join(GOLDEN, name + '.npz'))
    return {k: z[k] for k in z.files if k != 'meta'}, json.loads(bytes(z['meta']).decode())


def _previous(sig, K):
    """(B, L, K): the signatures of t-1 .. t-K (NaN before the start) (asrn/nucleo.py:167-172)."""
    B, L = sig.shape
    pad = torch.cat([torch.full((B, K), float('nan'), dtype=sig.dtype, device=sig.device), sig], 1)
    return torch.stack([pad[:, K - k - 1:K - k - 1 + L] for k in range(K)], -1)


def _run(f, m, cuda, half):
    from asrn_b200.train import BucketAttention
    act = torch.bfloat16 if half else torch.float32
    leaves = {k: torch.from_numpy(f[k]).to(cuda) for k in ('phi', 'V', 'Qc', 'Kc', 'Bt', 'log_alfa')}
    for k in ('phi', 'V', 'Qc', 'Kc'):
        leaves[k] = leaves[k].to(act)
    for t in leaves.values():
        t.requires_grad_()
    w = torch.from_numpy(f['w_sufijo']).to(cuda).requires_grad_()
    gamma = torch.from_numpy(f['gamma']).to(cuda).requires_grad_()
    sig = torch.from_numpy(f['sig']).to(cuda).float()
    Pf = _previous(sig, m['K'])
    orden = torch.from_numpy(f['orden']).to(cuda)
    ids_o = torch.from_numpy(f['ids_o']).to(cuda)
    salida, sen = BucketAttention.apply(leaves['phi'], leaves['V'], leaves['Qc'], leaves['Kc'], leaves['Bt'],
                                        leaves['log_alfa'], w, gamma, Pf, orden, ids_o, m['T'], m['C'],
                                        1.0 / m['temperatura'], m['cf'] ** -0.5)
    G = torch.from_numpy(f['G']).to(cuda)
    (salida.float() * G).sum().backward()
    grads = {k: t.grad for k, t in leaves.items()}
    grads.update(w_sufijo=w.grad, gamma=gamma.grad)
    return salida, sen, grads


@pytest.mark.parametrize('name', ['grad_crowded', 'grad_default', 'grad_ragged'])
def test_bucket_attention_forward_and_gradients_match_reference(name, cuda):
    f, m = _fixture(name)
    salida, sen, grads = _run(f, m, cuda, False)
    assert rel_err(salida.detach().cpu().numpy(), f['salida']) <= 1e-5
    B, T, L = m['B'], m['T'], m['L']
    ref_sen = f['senal']                                            # (B, T, L, 3)
    got_sen = sen.view(B, T, L, 3).cpu().numpy()
    hay = ref_sen[..., 0] > 0
    assert np.array_equal(got_sen[..., 0] > 0, hay)
    for c in (1, 2):
        assert rel_err(got_sen[..., c][hay], ref_sen[..., c][hay]) <= 1e-5
    for k in ('phi', 'V', 'Qc', 'Kc', 'Bt', 'log_alfa', 'w_sufijo', 'gamma'):
        assert grads[k].dtype == torch.from_numpy(f['grad_' + k]).dtype, k
        assert rel_err(grads[k].cpu().numpy(), f['grad_' + k]) <= 1e-4, k


@pytest.mark.parametrize('name', ['grad_crowded', 'grad_ragged'])
def test_bucket_attention_bf16_operands(name, cuda):
    f, m = _fixture(name)
    salida, _, grads = _run(f, m, cuda, True)
    assert salida.dtype == torch.bfloat16
    assert rel_err(salida.detach().float().cpu().numpy(), f['salida']) <= 3e-2
    for k in ('phi', 'V', 'Qc', 'Kc', 'Bt', 'log_alfa', 'w_sufijo', 'gamma'):
        assert rel_err(grads[k].float().cpu().numpy(), f['grad_' + k]) <= 3e-2, k


def test_bucket_attention_backward_is_deterministic(cuda):
    f, m = _fixture('grad_crowded')
    a = _run(f, m, cuda, False)[2]
    b = _run(f, m, cuda, False)[2]
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_scan_forward_and_gradients_match_reference(cuda):
    from asrn_b200.train import escaneo
    f, _ = _fixture('grad_crowded')
    a = torch.from_numpy(f['scan_a']).to(cuda).requires_grad_()
    b = torch.from_numpy(f['scan_b']).to(cuda).requires_grad_()
    S = escaneo(a, b)
    assert rel_err(S.detach().cpu().numpy(), f['scan_S']) <= 1e-5
    (S * torch.from_numpy(f['scan_g']).to(cuda)).sum().backward()
    assert rel_err(a.grad.cpu().numpy(), f['scan_grad_a']) <= 1e-5
    assert rel_err(b.grad.cpu().numpy(), f['scan_grad_b']) <= 1e-5


@pytest.mark.parametrize('L', [1, 5, 1023, 1024, 1025, 70000])
def test_scan_lengths_against_sequential(L, cuda):
    """Ragged and long rows against a float64 sequential recurrence (forward and both gradients)."""
    from asrn_b200.train import escaneo
    g = torch.Generator().manual_seed(L)
    a = torch.rand(2, L, generator=g) * 0.999
    b = torch.randn(2, L, generator=g)
    up = torch.randn(2, L, generator=g)
    S_ref = torch.zeros(2, L, dtype=torch.float64)
    x = torch.zeros(2, dtype=torch.float64)
    for i in range(L):
        x = a[:, i].double() * x + b[:, i].double()
        S_ref[:, i] = x
    lam = torch.zeros(2, L, dtype=torch.float64)
    y = torch.zeros(2, dtype=torch.float64)
    for i in range(L - 1, -1, -1):
        y = up[:, i].double() + (a[:, i + 1].double() * y if i + 1 < L else 0)
        lam[:, i] = y
    ga_ref = lam * torch.cat([torch.zeros(2, 1, dtype=torch.float64), S_ref[:, :-1]], 1)
    ad, bd = a.to(cuda).requires_grad_(), b.to(cuda).requires_grad_()
    S = escaneo(ad, bd)
    (S * up.to(cuda)).sum().backward()
    assert rel_err(S.detach().cpu().numpy(), S_ref.numpy()) <= 1e-5
    assert rel_err(bd.grad.cpu().numpy(), lam.numpy()) <= 1e-5
    assert rel_err(ad.grad.cpu().numpy(), ga_ref.numpy()) <= 1e-5


def test_training_entry_points_refuse_cpu_tensors():
    from asrn_b200.train import escaneo
    with pytest.raises(RuntimeError):
        escaneo(torch.rand(2, 8), torch.rand(2, 8))
