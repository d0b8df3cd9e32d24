"""Device sampling (asrn_b200.sampling, asrn_sampler_fill / asrn_sample_argmax) against torch's own CPU draws, and
seeded generation against the reference's sampled sequences (tests/golden/gen_sampled.npz, written by the reference's
generate).

Bars: the device Exp(1) draws equal torch's CPU exponential_ (all but at most 1e-6 of them bit for bit, the rest
within one float ulp: CUDA's and the host's double log1p may round differently); the device draw equals
torch.multinomial(prob, 1) token for token; generated sequences equal the reference's."""
import numpy as np
import pytest
import torch

from conftest import load_fixture

pytestmark = pytest.mark.gpu


def _ulps(a, b):
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


@pytest.mark.parametrize('rows,V,steps,window', [(4, 50304, 5, 1 << 31), (3, 1000, 9, 3 * 1000 * 4 * 2),
                                                 (1, 7, 40, 1 << 31)])
def test_device_draws_equal_torch_cpu_exponential(rows, V, steps, window, cuda):
    from asrn_b200.sampling import DeviceSampler
    seed = 4321
    s = DeviceSampler(seed, rows, V, steps, cuda, window_bytes=window)
    g = torch.Generator().manual_seed(seed)
    prob = torch.full((rows, V), 1.0 / V, device=cuda)
    mism = 0
    for k in range(steps):
        want = torch.empty(rows, V).exponential_(1, generator=g).numpy()
        if k >= s._k0 + s._n:
            s._fill()
        got = s.q(k).cpu().numpy()
        u = _ulps(got, want)
        assert u.max() <= 1, f'step {k}: {u.max()} ulps'
        mism += int((u > 0).sum())
        s.sample(prob)                                         # advances the step (and the window when needed)
    assert mism <= max(1, int(1e-6 * rows * V * steps))


def _probs(rows, V, kind, seed):
    g = torch.Generator().manual_seed(seed)
    lg = torch.randn(rows, V, generator=g) * 4
    if kind == 'topk':
        cut = lg.topk(40, -1).values[:, -1:]
        lg = lg.masked_fill(lg < cut, -float('inf'))
    if kind == 'onehot':
        lg = torch.full((rows, V), -float('inf'))
        lg[:, 5] = 0
    return torch.softmax(lg, -1)


@pytest.mark.parametrize('kind', ['dense', 'topk', 'onehot'])
def test_device_draw_equals_torch_multinomial(kind, cuda):
    """Several successive draws with one seeded generator: the device draw is torch.multinomial(prob.cpu(), 1, g)."""
    from asrn_b200.sampling import DeviceSampler
    rows, V, steps, seed = 8, 50304, 4, 99
    s = DeviceSampler(seed, rows, V, steps, cuda)
    g = torch.Generator().manual_seed(seed)
    for k in range(steps):
        p = _probs(rows, V, kind, 10 + k)
        want = torch.multinomial(p, 1, generator=g)[:, 0].tolist()
        s.sample(p.to(cuda))
        assert s.tokens_and_check() == want


def test_device_draw_reports_a_bad_distribution(cuda):
    """A row with a negative, inf or nan element, or all zeros, raises as torch.multinomial does; the sampler stays
    usable."""
    from asrn_b200.sampling import DeviceSampler
    s = DeviceSampler(1, 3, 64, 4, cuda)
    for bad in ('neg', 'nan', 'zero'):
        p = torch.full((3, 64), 1 / 64, device=cuda)
        if bad == 'neg':
            p[1, 3] = -0.1
        elif bad == 'nan':
            p[2, 0] = float('nan')
        else:
            p[0] = 0
        with pytest.raises(RuntimeError):
            torch.multinomial(p.cpu(), 1)
        s.sample(p)
        with pytest.raises(RuntimeError):
            s.tokens_and_check()
    s.sample(torch.full((3, 64), 1 / 64, device=cuda))
    assert len(s.tokens_and_check()) == 3


@pytest.mark.parametrize('i', range(4))
def test_generate_sampling_matches_reference(i, cuda):
    """Seeded sampling (temperature, top-k, top-p, repetition penalty, no-repeat n-grams, quote conservation, a seed
    above 2^32) gives the reference's tokens."""
    import json
    import os
    import asrn_b200
    z, params, meta = load_fixture('model_small')
    ref = np.load(os.path.join(os.path.dirname(__file__), 'golden', 'gen_sampled.npz'))
    settings = json.loads(str(ref['settings']))
    m = asrn_b200.create_model(V=meta['V'], d=meta['d'], n_capas=meta['n_capas'])
    m.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})
    m = m.to(cuda).eval()
    x0 = torch.from_numpy(z['tokens'][:, :meta['L0']]).to(cuda)
    seqs, _ = asrn_b200.generate(m, x0, n_nuevos=meta['n_new'], devolver_logits=False, **settings[i])
    assert np.array_equal(seqs.numpy(), ref[f'seqs_{i}'])


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_argmax_rows_matches_torch(dtype, cuda):
    """asrn_argmax_rows against torch.argmax: random rows, rows of equal maxima (bf16 ties), a row with NaNs, a row of
    -inf, a length that is not a multiple of 8."""
    from asrn_b200.writer import argmax_rows
    g = torch.Generator().manual_seed(3)
    for V in (50304, 1001):
        x = torch.randn(64, V, generator=g)
        x[1] = torch.round(x[1])                     # many equal maxima
        x[2, [7, 900]] = float('nan')
        x[3] = -float('inf')
        x[4, :] = 0.0
        x[5, 500:] = x[5].max() + 1                  # the maximum first reached at 500
        xd = x.to(cuda, dtype)
        assert torch.equal(argmax_rows(xd).cpu(), xd.argmax(-1).cpu())
