"""The differentiable ASRNLayer (training path: asrn_b200.train.layer_forward_train, with the bucket attention and
scans on the training kernels) against the reference's own autograd through its whole layer forward (fixtures
tests/golden/layer_grad_*.npz, fp32 on the CPU, asrn/estable.py:407-421).

Bars (fp32): output within 1e-5 of max|y|; the gradients of E, h and of every parameter within 1e-4 of their max
(sums in another order: the attention's per-slot buffers, cuBLAS against the CPU's GEMMs). Under bf16 autocast the
training path runs and its gradients stay within 5e-2 of the fp32 reference's."""
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu


def _case(name, cuda):
    import asrn_b200
    z = np.load(os.path.join(GOLDEN, name + '.npz'))
    meta = json.loads(bytes(z['meta']).decode())
    layer = asrn_b200.ASRNLayer(meta['d'], **meta['opts'])
    layer.load_state_dict({k[6:]: torch.from_numpy(z[k]) for k in z.files if k.startswith('param.')})
    layer = layer.to(cuda).train()
    E = torch.from_numpy(z['E']).to(cuda).requires_grad_()
    h = torch.from_numpy(z['h']).to(cuda).requires_grad_()
    x = torch.from_numpy(z['tokens']).to(cuda)
    return z, layer, E, h, x


@pytest.mark.parametrize('name', ['layer_grad_crowded', 'layer_grad_default', 'layer_grad_ragged'])
def test_layer_gradients_match_reference(name, cuda):
    z, layer, E, h, x = _case(name, cuda)
    y = layer(E, h, x)
    assert y.grad_fn is not None
    assert rel_err(y.detach().cpu().numpy(), z['y']) <= 1e-5
    (y * torch.from_numpy(z['G']).to(cuda)).sum().backward()
    assert rel_err(E.grad.cpu().numpy(), z['grad_E']) <= 1e-4
    assert rel_err(h.grad.cpu().numpy(), z['grad_h']) <= 1e-4
    for k, p in layer.named_parameters():
        ref = z['grad.' + k]
        got = p.grad.cpu().numpy() if p.grad is not None else np.zeros_like(ref)
        assert rel_err(got, ref) <= 1e-4, k


def test_layer_gradients_under_bf16_autocast(cuda):
    z, layer, E, h, x = _case('layer_grad_crowded', cuda)
    with torch.autocast('cuda', dtype=torch.bfloat16):
        y = layer(E, h, x)
    (y.float() * torch.from_numpy(z['G']).to(cuda)).sum().backward()
    assert rel_err(y.detach().float().cpu().numpy(), z['y']) <= 5e-2
    assert rel_err(E.grad.cpu().numpy(), z['grad_E']) <= 5e-2
    assert rel_err(h.grad.cpu().numpy(), z['grad_h']) <= 5e-2
    for k in ('v.weight', 'o.weight', 'gamma', 'w_sufijo', 'log_kappa', 'd_racha'):
        assert rel_err(dict(layer.named_parameters())[k].grad.cpu().numpy(), z['grad.' + k]) <= 5e-2, k


def test_training_forward_equals_inference_forward(cuda):
    """The training path and the fused inference forward give the same h' (within the fp32 spread)."""
    z, layer, E, h, x = _case('layer_grad_default', cuda)
    y_train = layer(E, h, x).detach()
    with torch.no_grad():
        y_inf = layer(E, h, x)
    assert rel_err(y_train.cpu().numpy(), y_inf.cpu().numpy()) <= 1e-5


def test_a_training_step_lowers_the_loss(cuda):
    """Five SGD steps on a fixed batch through the training path lower a regression loss."""
    z, layer, E, h, x = _case('layer_grad_crowded', cuda)
    target = torch.from_numpy(z['G']).to(cuda) * 0.1
    opt = torch.optim.SGD(layer.parameters(), lr=1e-2)
    losses = []
    for _ in range(5):
        opt.zero_grad()
        loss = ((layer(E.detach(), h.detach(), x) - h.detach() - target) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]


def test_model_trains_end_to_end(cuda):
    """create_model's whole forward is differentiable (local blocks as torch modules, ASRN layers on the training
    path): three Adam steps of next-token cross-entropy on a fixed batch lower the loss, and every ASRN layer's
    parameters get a gradient."""
    import asrn_b200
    m = asrn_b200.create_model(V=64, d=64, n_capas=4, semilla=1).to(cuda).train()
    x = torch.from_numpy(np.random.default_rng(0).integers(0, 64, (2, 96))).to(cuda)
    opt = torch.optim.Adam(m.parameters(), lr=3e-3)
    losses = []
    for _ in range(3):
        opt.zero_grad()
        lg = m(x[:, :-1])
        loss = torch.nn.functional.cross_entropy(lg.float().reshape(-1, 64), x[:, 1:].reshape(-1))
        loss.backward()
        for layer in m.largos:
            assert layer.v.weight.grad is not None and torch.isfinite(layer.v.weight.grad).all()
            assert layer.gamma.grad is not None
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]
