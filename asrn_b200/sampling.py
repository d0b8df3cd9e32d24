"""Device sampling with the reference's random numbers (asrn/nucleo.py:1945-1962, :1996).

The reference draws each generated token on the host: torch.multinomial(prob.cpu(), 1, generator=g) with
g = torch.Generator('cpu').manual_seed(semilla). For one sample torch takes, per row, the argmax of prob / q with q one
Exp(1) draw per element of prob from g, so the k-th call on a (B, V) matrix uses a slice of g's stream that only
depends on the seed, k, B and V. DeviceSampler makes those q on the device ahead of time (libasrn_b200's MT19937
replay with jump-ahead: one block per step) and draws with a device argmax: the same tokens as the reference, no (B, V)
copy to the host and no host random numbers.
"""
import numpy as np
import torch

from . import _lib

_N = 624
_polys = {}                 # (words per step, levels) -> host uint32 array (levels, 624)


def seed_state(seed):
    """The 624-word MT19937 array torch.Generator('cpu').manual_seed(seed) starts from (uint32 numpy)."""
    st = np.zeros(_N, np.uint32)
    _lib.check(_lib.lib().asrn_sampler_seed_state(int(seed) % (1 << 64), st.ctypes.data), 'asrn_sampler_seed_state')
    return st


def jump_polys(words, levels):
    """polys[l] = x^(2^l * words) mod the MT19937 characteristic polynomial, l < levels (uint32 numpy (levels, 624))."""
    key = (int(words), int(levels))
    if key not in _polys:
        P = np.zeros((max(levels, 1), _N), np.uint32)
        for l in range(levels):
            _lib.check(_lib.lib().asrn_sampler_jump_poly(words << l, P[l].ctypes.data), 'asrn_sampler_jump_poly')
        _polys[key] = P
    return _polys[key]


class DeviceSampler:
    """torch.multinomial(prob, 1, generator=torch.Generator('cpu').manual_seed(seed)) for `steps` successive (rows, V)
    probability matrices, on the device.

    sample(prob) draws the next step's tokens ((rows, 1) int64 on prob's device). The Exp(1) draws are made a window of
    steps at a time (at most window_bytes of float32 on the device); the first window is made at construction, on the
    current stream. check() raises as torch.multinomial would if a drawn row was not a distribution (an element < 0,
    inf or nan, or all zero); reading the status costs a device sync, so generate() reads it together with the tokens.
    """

    def __init__(self, seed, rows, V, steps, device, window_bytes=1 << 31):
        self.rows, self.V, self.steps = int(rows), int(V), int(steps)
        self.device = torch.device(device)
        self.draws = self.rows * self.V
        self.window = max(1, min(self.steps, int(window_bytes) // (4 * max(self.draws, 1))))
        self.levels = max(1, (self.window - 1).bit_length())
        P = jump_polys(2 * self.draws, self.levels)
        self._polys = torch.from_numpy(P.view(np.int32)).to(self.device)
        self._state = torch.from_numpy(seed_state(seed).view(np.int32)).to(self.device)
        self._next = torch.empty_like(self._state)
        self._q = torch.empty(self.window, self.rows, self.V, dtype=torch.float32, device=self.device)
        # tokens and the status word in one buffer, so one copy brings both to the host
        self._out = torch.zeros(self.rows + 1, dtype=torch.int64, device=self.device)
        self.k = 0                  # steps drawn
        self._k0 = 0                # first step of the current window
        self._n = 0                 # steps in the current window
        if self.steps > 0 and self.draws > 0:
            self._fill()

    def _fill(self):
        self._k0 += self._n
        n = min(self.window, self.steps - self._k0)
        if n <= 0:
            raise RuntimeError('DeviceSampler: more draws than the steps it was made for')
        st = _lib.stream_ptr(self.device)
        _lib.check(_lib.lib().asrn_sampler_fill(self.draws, n, self.levels, _lib.ptr(self._state),
                                                _lib.ptr(self._polys), _lib.ptr(self._q), _lib.ptr(self._next), st),
                   'asrn_sampler_fill')
        self._state, self._next = self._next, self._state
        self._n = n

    def q(self, k):
        """The (rows, V) Exp(1) draws of step k of the current window (a view; tests compare it with torch)."""
        return self._q[k - self._k0]

    def sample(self, prob):
        """(rows, 1) int64: the next step's draw from prob ((rows, V) float32 on the device)."""
        if prob.shape != (self.rows, self.V) or prob.device != self.device:
            raise ValueError(f'prob: expected ({self.rows}, {self.V}) on {self.device}, got {tuple(prob.shape)} on '
                             f'{prob.device}')
        if self.k >= self._k0 + self._n:
            self._fill()
        p = prob.float().contiguous()
        st = _lib.stream_ptr(self.device)
        status = self._out[self.rows:]
        _lib.check(_lib.lib().asrn_sample_argmax(self.rows, self.V, _lib.ptr(p), _lib.ptr(self.q(self.k)),
                                                 _lib.ptr(self._out), _lib.ptr(status), st), 'asrn_sample_argmax')
        self.k += 1
        return self._out[:self.rows].unsqueeze(1)

    def tokens_and_check(self):
        """The last draw's tokens as a host list; raises RuntimeError as torch.multinomial does on a bad row."""
        host = self._out.cpu()
        if int(host[self.rows]) != 0:
            self._out[self.rows:].zero_()
            raise RuntimeError('probability tensor contains either `inf`, `nan` or element < 0, or a row sums to 0 '
                               '(invalid multinomial distribution)')
        return host[:self.rows].tolist()
