"""asrn_bucket_sort_noalloc: the bucket sort for callers that cannot allocate device memory when they sort (a plug-in
running inside a host process whose allocator it does not own, or a serving loop that keeps a fixed memory footprint
after start-up). Its scratch for rows longer than one tile is a fixed array inside the library.

Checked through the C ABI against asrn_bucket_sort (the entry point with a caller-provided workspace) on two calls in a
row with different data, so the second call proves the shared scratch does not carry anything over from the first.
Sorting is integer work: the outputs must be identical. This file is collected last so that a run stopping at the first
failure has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _sort_with_workspace(lib, ids_rows, nb, dev):
    from asrn_b200 import _lib
    rows, L = ids_rows.shape
    orden = torch.empty(rows, L, dtype=torch.int32, device=dev)
    ids_o = torch.empty(rows, L, dtype=torch.int16, device=dev)
    nbytes = lib.asrn_bucket_sort_workspace_bytes(rows, L, nb)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    st = lib.asrn_bucket_sort(rows, L, nb, _lib.ptr(ids_rows), _lib.ptr(orden), _lib.ptr(ids_o), _lib.ptr(ws), nbytes,
                              _lib.stream_ptr(dev))
    assert st == 0
    return orden, ids_o


def _sort_noalloc(lib, ids_rows, nb, dev):
    from asrn_b200 import _lib
    rows, L = ids_rows.shape
    orden = torch.full((rows, L), -7, dtype=torch.int32, device=dev)
    ids_o = torch.full((rows, L), -7, dtype=torch.int16, device=dev)
    st = lib.asrn_bucket_sort_noalloc(rows, L, nb, _lib.ptr(ids_rows), _lib.ptr(orden), _lib.ptr(ids_o),
                                      _lib.stream_ptr(dev))
    return st, orden, ids_o


def test_noalloc_bucket_sort_matches_workspace_version_on_two_calls():
    from asrn_b200 import _lib
    assert torch.cuda.is_available(), 'GPU test selected but no CUDA device is visible'
    dev = torch.device('cuda:0')
    lib = _lib.lib()
    nb = 14
    cases = [(3, 20000, 1), (2, 30001, 2)]        # rows span 3 and 4 tiles of 8192 positions: the scratch is used
    for rows, L, seed in cases:
        g = np.random.default_rng(seed)
        ids = g.integers(0, 1 << nb, (rows, L)).astype(np.uint16)
        ids[:, L // 3:L // 2] = ids[:, :L // 2 - L // 3]
        t = torch.from_numpy(ids.view(np.int16)).to(dev)
        st, orden, ids_o = _sort_noalloc(lib, t, nb, dev)
        assert st == 0, lib.asrn_status_string(st)
        ref_orden, ref_ids = _sort_with_workspace(lib, t, nb, dev)
        torch.cuda.synchronize()
        assert torch.equal(orden, ref_orden)
        assert torch.equal(ids_o, ref_ids)
        assert np.array_equal(orden.cpu().numpy(), np.argsort(ids.astype(np.int64), axis=-1, kind='stable'))


def test_noalloc_bucket_sort_rejects_requests_beyond_its_scratch():
    from asrn_b200 import _lib
    dev = torch.device('cuda:0')
    lib = _lib.lib()
    rows, L, nb = 64, 200000, 14                  # 51 MB of keys + histograms: more than the 32 MiB array
    t = torch.zeros(rows, L, dtype=torch.int16, device=dev)
    st, _, _ = _sort_noalloc(lib, t, nb, dev)
    assert st == _lib.ASRN_ERR_WORKSPACE
    small = torch.randint(0, 1 << nb, (4, 5000), dtype=torch.int32).to(torch.int16).to(dev)   # one tile: no scratch
    st, orden, _ = _sort_noalloc(lib, small, nb, dev)
    assert st == 0
    assert np.array_equal(orden.cpu().numpy(), np.argsort(small.cpu().numpy().view(np.uint16).astype(np.int64),
                                                           axis=-1, kind='stable'))


def test_noalloc_bucket_sort_empty_input_matches_workspace_version():
    """Empty input returns ASRN_OK from both entry points, whatever the bit count (nothing is sorted or checked)."""
    from asrn_b200 import _lib
    dev = torch.device('cuda:0')
    lib = _lib.lib()
    for rows, L, nb in ((0, 100, 14), (3, 0, 14), (0, 0, 99)):
        assert lib.asrn_bucket_sort_noalloc(rows, L, nb, None, None, None, _lib.stream_ptr(dev)) == 0
        assert lib.asrn_bucket_sort(rows, L, nb, None, None, None, None, 0, _lib.stream_ptr(dev)) == 0
