"""Host-side checks that need no GPU: the C ABI library loads and exports every entry point of include/asrn_b200.h,
the Python layer/model mirror the reference's parameters and initialisation, and there is no CPU path."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, load_fixture


def header_symbols():
    text = open(os.path.join(ROOT, 'include', 'asrn_b200.h')).read()
    return sorted(set(re.findall(r'\b(asrn_[a-z0-9_]+)\s*\(', text)))


def test_library_exports_every_declared_symbol():
    from asrn_b200 import _lib
    lib = _lib.lib()
    declared = header_symbols()
    assert declared, 'no entry points found in the header'
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(declared) == _lib.exported_symbols()
    assert lib.asrn_abi_version() == _lib.ABI_VERSION
    assert lib.asrn_status_string(0) == b'ok'


def test_config_sizes_and_validation_without_gpu():
    import asrn_b200
    from asrn_b200 import _lib
    layer = asrn_b200.ASRNLayer(768)
    cfg = _lib.make_config(layer, 32, 8192, True)
    lib = _lib.lib()
    ws = lib.asrn_layer_workspace_bytes(ctypes.byref(cfg))
    # 262,144 tokens: bf16 accumulator 403 MB + bf16 copy of E 403 MB + small per-token intermediates
    assert 0.85e9 < ws < 1.1e9, ws
    assert lib.asrn_layer_prepared_bytes(ctypes.byref(cfg)) > 768 * 768 * 2
    bad = _lib.make_config(asrn_b200.ASRNLayer(64, chunk=64), 1, 8, False)
    assert lib.asrn_layer_workspace_bytes(ctypes.byref(bad)) == 0      # chunk > 32 rejected
    st = lib.asrn_layer_forward(ctypes.byref(bad), None, None, None, None, None, None, None, 0, None)
    assert st != 0


def test_layer_parameter_names_match_reference():
    import asrn_b200
    _, params, meta = load_fixture('layer_f32')
    layer = asrn_b200.ASRNLayer(meta['d'])
    sd = layer.state_dict()
    assert set(sd) == set(params)
    for k, v in params.items():
        assert tuple(sd[k].shape) == tuple(v.shape), k
    layer.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})


def test_create_model_same_seed_same_weights_as_reference():
    import asrn_b200
    z = np.load(os.path.join(ROOT, 'tests', 'golden', 'init_cfg1.npz'))
    m = asrn_b200.create_model(V=256, d=64, n_capas=4, semilla=0)
    sd = m.state_dict()
    names = sorted(k[4:] for k in z.files if k.startswith('sum.'))
    assert sorted(sd) == names
    for k in names:
        t = sd[k].double()
        assert abs(float(t.sum()) - float(z['sum.' + k])) <= 1e-9 * max(1.0, abs(float(z['sum.' + k]))), k
        assert np.allclose(t.reshape(-1)[:8].numpy(), z['first.' + k], atol=0, rtol=0), k


def test_model_state_dict_loads_reference_checkpoint():
    import asrn_b200
    _, params, meta = load_fixture('model_small')
    m = asrn_b200.create_model(V=meta['V'], d=meta['d'], n_capas=meta['n_capas'])
    m.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})


def test_no_cpu_fallback():
    import asrn_b200
    layer = asrn_b200.ASRNLayer(32, chunk=16, n_bits=4)
    E, h = torch.randn(1, 8, 32), torch.randn(1, 8, 32)
    with pytest.raises(RuntimeError, match='CUDA'):
        layer(E, h, torch.zeros(1, 8, dtype=torch.long))


def test_synthetic_streams_are_seeded():
    from asrn_b200 import synthetic
    a = synthetic.config_tokens('cfg3', B=2, L=4096, seed=0)
    b = synthetic.config_tokens('cfg3', B=2, L=4096, seed=0)
    assert np.array_equal(a, b) and a.max() < 50304 and a.min() >= 0
    x = synthetic.config_tokens('cfg2', B=1, L=4096)
    assert x.max() < 256


def test_grad_fixture_scan_matches_the_recurrence():
    """The reference's scan gradients in the gradient fixture follow l_i = g_i + a_{i+1} l_{i+1}, dL/da_i = l_i
    S_{i-1} (asrn/nucleo.py:518-537), restated here in float64."""
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'grad_crowded.npz'))
    a, b, g = (z[k].astype(np.float64) for k in ('scan_a', 'scan_b', 'scan_g'))
    S = np.zeros_like(a)
    x = np.zeros(a.shape[0])
    for i in range(a.shape[1]):
        x = a[:, i] * x + b[:, i]
        S[:, i] = x
    lam = np.zeros_like(a)
    y = np.zeros(a.shape[0])
    for i in range(a.shape[1] - 1, -1, -1):
        y = g[:, i] + (a[:, i + 1] * y if i + 1 < a.shape[1] else 0)
        lam[:, i] = y
    assert np.abs(S - z['scan_S']).max() <= 1e-4 * np.abs(S).max()
    assert np.abs(lam - z['scan_grad_b']).max() <= 1e-4 * np.abs(lam).max()
    ga = lam * np.concatenate([np.zeros((a.shape[0], 1)), S[:, :-1]], 1)
    assert np.abs(ga - z['scan_grad_a']).max() <= 1e-4 * np.abs(ga).max()
