"""Seeded synthetic token streams for the benchmark configurations.

The reference ships no generator for its benchmark shapes, so this module defines one and every consumer
(parity tests, the CPU oracle timing, bench.py) draws from it with the same seed:

  zipf_tokens(B, L, V, s)      tokens from a finite Zipf(s) over V ranks (inverse CDF of p_k ~ k^-s, k = 1..V),
                               rank k mapped to token id k - 1
  plant_repeats(x, frac, lo, hi, max_dist)
                               overwrite spans of length U[lo, hi] with copies of earlier spans (the source starts
                               at most max_dist tokens before the destination) until `frac` of each row is covered
  uniform_bytes_with_repeats   configuration 1: uniform bytes, 30 % of positions copied from earlier spans of 16-64

Everything is numpy with an explicit Generator so the streams are identical on every machine.
"""
import numpy as np


def zipf_tokens(B, L, V, s=1.1, seed=0):
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, V + 1, dtype=np.float64)
    p = ranks ** (-s)
    cdf = np.cumsum(p)
    cdf /= cdf[-1]
    u = rng.random((B, L))
    return np.minimum(np.searchsorted(cdf, u, side='right'), V - 1).astype(np.int64)


def plant_repeats(x, frac, lo, hi, max_dist=None, seed=1):
    """In place on x (B, L): copies earlier spans forward until about `frac` of each row lies in planted copies."""
    rng = np.random.default_rng(seed)
    B, L = x.shape
    for b in range(B):
        covered = np.zeros(L, dtype=bool)
        target = int(frac * L)
        tries = 0
        while covered.sum() < target and tries < 100000:
            tries += 1
            n = int(rng.integers(lo, hi + 1))
            if 2 * n + 1 > L:
                n = max(1, (L - 1) // 2)
            dst = int(rng.integers(n, L - n + 1)) if L - n + 1 > n else n
            if dst + n > L:
                continue
            far = dst - n if max_dist is None else min(dst - n, max_dist)
            if far < 0:
                continue
            src = dst - n - int(rng.integers(0, far + 1))
            if src < 0:
                continue
            x[b, dst:dst + n] = x[b, src:src + n].copy()
            covered[dst:dst + n] = True
    return x


def uniform_bytes_with_repeats(B, L, seed=0, frac=0.30, lo=16, hi=64):
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 256, size=(B, L)).astype(np.int64)
    return plant_repeats(x, frac, lo, hi, seed=seed + 1)


def config_tokens(name, B=None, L=None, seed=0):
    """Token batches of the benchmark configurations (shapes may be reduced with B / L)."""
    if name == 'cfg1':
        return uniform_bytes_with_repeats(B or 8, L or 256, seed)
    if name == 'cfg2':
        x = zipf_tokens(B or 16, L or 4096, 256, 1.1, seed)
        return plant_repeats(x, 0.25, 8, 128, seed=seed + 1)
    if name == 'cfg3':
        x = zipf_tokens(B or 32, L or 8192, 50304, 1.1, seed)
        return plant_repeats(x, 0.20, 16, 256, seed=seed + 1)
    if name == 'cfg5':
        x = zipf_tokens(B or 64, L or 65536, 50304, 1.1, seed)
        return plant_repeats(x, 0.20, 16, 256, seed=seed + 1)
    if name == 'cfg4':
        x = zipf_tokens(B or 1, L or 262144, 50304, 1.1, seed)
        return plant_repeats(x, 0.20, 32, 512, max_dist=200000, seed=seed + 1)
    raise ValueError(f'unknown configuration {name!r}')
