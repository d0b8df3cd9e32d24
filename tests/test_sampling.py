"""Host side of the device sampler (asrn_b200.sampling; asrn_b200/csrc/sampler.cu) on the CPU: the seed state, the
jump-ahead polynomials against a directly iterated MT19937 stream, and the model of torch's CPU Exp(1) draw the device
kernel replays (pinned against torch itself)."""
import numpy as np
import pytest
import torch

from asrn_b200 import sampling

_MATRIX_A = np.uint32(0x9908b0df)


def _stream(state, n):
    """Untempered MT19937 words x_0 .. x_{623+n} from the 624-word window x_0..x_623 (227 words at a time)."""
    x = np.zeros(624 + n, np.uint32)
    x[:624] = state
    for b in range(624, 624 + n, 227):
        a = np.arange(b, min(b + 227, 624 + n))
        y = (x[a - 624] & np.uint32(0x80000000)) | (x[a - 623] & np.uint32(0x7fffffff))
        x[a] = x[a - 227] ^ (y >> np.uint32(1)) ^ np.where(x[a - 623] & np.uint32(1), _MATRIX_A, np.uint32(0))
    return x


def _temper(y):
    y = y ^ (y >> np.uint32(11))
    y = y ^ ((y << np.uint32(7)) & np.uint32(0x9d2c5680))
    y = y ^ ((y << np.uint32(15)) & np.uint32(0xefc60000))
    return y ^ (y >> np.uint32(18))


def _exp_draws(x, start, n):
    """torch's CPU exponential_(1) on n float elements whose first 32-bit output is x_{624 + start}: one 64-bit value
    per element (first output high), u = (value & (2^53 - 1)) 2^-53, q = float(-log1p(-u))."""
    out = _temper(x[624 + start:624 + start + 2 * n]).astype(np.uint64)
    v = ((out[0::2] << np.uint64(32)) | out[1::2]) & np.uint64((1 << 53) - 1)
    return (-np.log1p(-(v.astype(np.float64) * 2.0 ** -53))).astype(np.float32)


def test_seed_state_is_torchs_and_numpys_legacy_seeding():
    st = sampling.seed_state(1234)
    bg = np.random.MT19937(0)
    bg._legacy_seeding(1234)
    assert np.array_equal(st, bg.state['state']['key'])
    assert np.array_equal(sampling.seed_state(2 ** 40 + 9), sampling.seed_state(9))      # seed mod 2^32


@pytest.mark.parametrize('seed', [0, 1234])
def test_exp_draw_model_matches_torch(seed):
    """The draw the device kernel replays is torch's: successive exponential_ calls read successive outputs."""
    x = _stream(sampling.seed_state(seed), 2 * (3000 + 5000) + 64)
    g = torch.Generator().manual_seed(seed)
    a = torch.empty(3, 1000).exponential_(1, generator=g).numpy().ravel()
    b = torch.empty(5000).exponential_(1, generator=g).numpy()
    assert np.array_equal(a, _exp_draws(x, 0, 3000))
    assert np.array_equal(b, _exp_draws(x, 6000, 5000))


def test_multinomial_one_sample_is_argmax_of_p_over_q():
    """torch.multinomial(p, 1) = argmax(p / q), q the Exp(1) draws of p's shape: the rule the device argmax follows."""
    seed = 77
    p = torch.softmax(torch.randn(4, 300, generator=torch.Generator().manual_seed(1)) * 3, -1)
    p[1, 100:] = 0
    got = torch.multinomial(p, 1, generator=torch.Generator().manual_seed(seed))[:, 0].numpy()
    x = _stream(sampling.seed_state(seed), 2 * p.numel() + 64)
    q = _exp_draws(x, 0, p.numel()).reshape(p.shape)
    assert np.array_equal(got, np.argmax(p.numpy() / q, -1))


@pytest.mark.parametrize('J', [1, 623, 624, 19937, 100003, 2 * 4 * 5003])
def test_jump_polynomial_gives_the_stream_ahead(J):
    """S_{n+J} = XOR over the set coefficients i of x^J mod phi of S_{n+i}: the jumped window equals the stream's window
    at n + J (from n = 1 word for word; from the seed window the low 31 bits of the first word may differ, bits no
    later output reads) and the outputs after it agree."""
    P = sampling.jump_polys(J, 1)[0]
    bits = np.nonzero(np.unpackbits(P.view(np.uint8), bitorder='little'))[0]
    assert bits.max() < 19937
    x = _stream(sampling.seed_state(5), J + 20600 + 2000)
    for n in (0, 1, 700):
        S = np.bitwise_xor.reduce(x[n + bits[:, None] + np.arange(624)[None, :]], axis=0)
        want = x[n + J:n + J + 624]
        assert np.array_equal(S[1:], want[1:]) and (S[0] >> np.uint32(31)) == (want[0] >> np.uint32(31))
        if n:
            assert S[0] == want[0]
        assert np.array_equal(_stream(S, 1000)[624:], _stream(want, 1000)[624:])


def test_jump_polynomials_compose():
    """polys[l] = x^(2^l J): two jumps by J equal one jump by 2 J (checked on the stream)."""
    J = 3001
    P = sampling.jump_polys(J, 2)
    x = _stream(sampling.seed_state(9), 2 * J + 20600 + 100)
    b0 = np.nonzero(np.unpackbits(P[0].view(np.uint8), bitorder='little'))[0]
    b1 = np.nonzero(np.unpackbits(P[1].view(np.uint8), bitorder='little'))[0]
    S1 = np.bitwise_xor.reduce(x[1 + b1[:, None] + np.arange(624)[None, :]], axis=0)
    assert np.array_equal(S1, x[1 + 2 * J:1 + 2 * J + 624])
    Sj = np.bitwise_xor.reduce(x[1 + b0[:, None] + np.arange(624)[None, :]], axis=0)
    y = _stream(Sj, J + 20600)
    S2 = np.bitwise_xor.reduce(y[b0[:, None] + np.arange(624)[None, :]], axis=0)
    assert np.array_equal(S2, S1)
