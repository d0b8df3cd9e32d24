"""The CPU oracle (oracle/asrn_oracle.py) against the reference's own outputs (tests/golden/*.npz).

This pins the restatement: integer / index outputs bit-exact, fp32 outputs within 1e-5 of the reference (max-norm
relative, the form of the reference's own tests, tests/test_nucleo.py:459), bf16-autocast outputs within 2e-3.
"""
import numpy as np
import pytest

from conftest import LAYER_FIXTURES, layer_options, load_fixture, rel_err
from oracle import asrn_oracle as O


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_oracle_matches_reference_layer(name):
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    lay = O.Layer(params, meta['d'], **layer_options(meta))
    parts = O.layer_forward(lay, z['E'], z['h'], z['tokens'], half=half, return_parts=True)
    # integer and index outputs: bit-exact
    assert np.array_equal(parts['ids'], z['ids'])
    assert np.array_equal(parts['orden'], z['orden'])
    assert np.array_equal(parts['claves'], z['claves'], equal_nan=True)
    assert np.array_equal(parts['orden_ng'], z['orden_ng'])
    assert np.array_equal(parts['repetido'], z['repetido'])
    assert np.array_equal(parts['vistos'], z['vistos'])
    assert np.array_equal(parts['senal'][..., 0], z['senal'][..., 0])          # hay
    assert np.array_equal(parts['peso_total'], z['peso_total'])
    tol = 2e-3 if half else 1e-5
    for k in ('Qc', 'Kc', 'phi', 'salida', 'mejor', 'pico', 'out'):
        assert rel_err(parts[k], z[k]) <= tol, (k, rel_err(parts[k], z[k]))
    for k in ('beta', 'log_alfa', 'Bt', 'hawkes', 'racha'):
        assert rel_err(parts[k], z[k]) <= 1e-5, (k, rel_err(parts[k], z[k]))
    assert rel_err(parts['out'] - z['h'], z['out'] - z['h']) <= (2e-3 if half else 1e-5)


def test_bf16_rounding_matches_torch():
    import torch
    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 10.0 ** np.random.default_rng(1).integers(
        -30, 30, 100000)
    x = x.astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16(x), ref)


def test_scan_matches_recurrence():
    """escaneo == the sequential recurrence (tests/test_nucleo.py:382-391), with segment resets."""
    g = np.random.default_rng(0)
    for N in (1, 2, 3, 7, 64, 1000):
        a = g.random((3, 5, N))
        b = g.standard_normal((3, 5, N))
        a[..., ::7] = 0
        S = np.zeros_like(a)
        acc = np.zeros((3, 5))
        for i in range(N):
            acc = a[..., i] * acc + b[..., i]
            S[..., i] = acc
        assert np.allclose(O.escaneo(a, b), S, atol=1e-5)


def test_hawkes_matches_quadratic_definition():
    """hawkes = the O(N^2) sum of its definition; hawkes > 0 <=> vistos (tests/test_nucleo.py:287-313)."""
    z, params, meta = load_fixture('layer_f32')
    lay = O.Layer(params, meta['d'], **layer_options(meta))
    L = 150
    g = np.random.default_rng(0)
    x = g.integers(0, 6, (3, L))
    x[:, L // 2:L // 2 + L // 4] = x[:, :L // 4]
    sig = O.firmas_de_piezas(x)
    beta = (g.random((3, L)) * 0.5).astype(np.float64)
    Bt, log_alfa = np.cumsum(beta, 1), (g.standard_normal((3, L)) * 0.3).astype(np.float32)
    r = O.repeticion(lay, sig, beta, Bt, log_alfa)
    claves = O.claves_de(sig, lay['c_vistos'], lay.n)
    kappa, _ = lay.kappas()
    before = np.tril(np.ones((L, L), bool), -1)
    for k in range(lay.n):
        same = (claves[..., k][:, :, None] == claves[..., k][:, None, :]) & before
        kern = np.exp(log_alfa)[:, None, :] * np.exp(-kappa[k] * np.maximum(Bt[:, :, None] - Bt[:, None, :], 0))
        assert np.allclose(r['hawkes'][..., k], (same * kern).sum(-1), atol=1e-4)
    assert np.array_equal((r['hawkes'] > 0).astype(np.float32), r['vistos'])


@pytest.mark.parametrize('name', ['layer_f32', 'layer_bf16', 'layer_f32_opts', 'layer_f32_d96', 'layer_bf16_d256'])
def test_vectorised_oracle_matches_reference_layer(name):
    """The vectorised restatement (the reference's window formulation, used at benchmark sizes) against the
    reference's outputs, and conditioned on the reference's own bucket ids (ids_override) it gives the same h'."""
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    lay = O.Layer(params, meta['d'], **layer_options(meta))
    tol = 2e-3 if half else 1e-5
    parts = O.layer_forward_fast(lay, z['E'], z['h'], z['tokens'], half=half, return_parts=True)
    assert np.array_equal(parts['ids'], z['ids'])
    assert np.array_equal(parts['orden'], z['orden'])
    for k in ('salida', 'mejor', 'pico', 'out'):
        assert rel_err(parts[k], z[k]) <= tol, (k, rel_err(parts[k], z[k]))
    assert rel_err(parts['out'] - z['h'], z['out'] - z['h']) <= tol
    over = O.layer_forward_fast(lay, z['E'], z['h'], z['tokens'], half=half, ids_override=z['ids'])
    assert np.array_equal(over, parts['out'])


def test_vectorised_oracle_equals_per_query_definition_in_the_full_bucket_regime():
    """Small embeddings make the hash bias-dominated, so long bucket runs give every query C candidates (the regime of
    the benchmark): the vectorised windows and the per-query definition agree."""
    z, params, meta = load_fixture('layer_bf16')
    lay = O.Layer(params, meta['d'])
    g = np.random.default_rng(11)
    B, L, d = 1, 300, meta['d']
    x = g.integers(0, 40, (B, L))
    E = (g.standard_normal((40, d)) * 0.02).astype(np.float32)[x]
    h = g.standard_normal((B, L, d)).astype(np.float32)
    for half in (False, True):
        a = O.layer_forward(lay, E, h, x, half=half, return_parts=True)
        b = O.layer_forward_fast(lay, E, h, x, half=half)
        same = (a['ids_o'][:, 1:] == a['ids_o'][:, :-1]).mean()
        assert same > 0.5
        assert rel_err(b, a['out']) <= (2e-3 if half else 1e-5)


def test_flip_bound_rejects_a_flip_far_from_zero():
    """A planted bucket-bit flip on a phi far from zero fails the agreement check; one within rounding passes."""
    from conftest import check_ids_agree
    z, params, meta = load_fixture('layer_f32')
    ids, phi = z['ids'].copy(), z['phi']
    B, L, T = ids.shape
    nb = phi.shape[-1] // T
    ph = np.abs(phi.reshape(B, L, T, nb))
    big = np.unravel_index(np.argmax(ph), ph.shape)
    bad = ids.copy()
    bad[big[:3]] ^= 1 << big[3]
    with pytest.raises(AssertionError):
        check_ids_agree(bad, ids, phi, nb, half=False)
    phi_small = phi.copy().reshape(B, L, T, nb)
    phi_small[big] = 1e-9
    assert check_ids_agree(bad, ids, phi_small.reshape(phi.shape), nb, half=False) < 1.0
