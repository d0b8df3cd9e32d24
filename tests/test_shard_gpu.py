"""Sequence-chunk sharding on the GPU: the shard's sorted rows against the selection rule, the sharded forward
(every rank emulated in one process) against the unsharded layer, and -- with two GPUs -- two NCCL ranks."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _rows_rule(orden, ids, C, q_lo, q_hi):
    """numpy statement of the shard's rows: local slots, and earlier-shard slots within C before a local slot of the
    same bucket."""
    out = []
    for o, i in zip(orden, ids):
        keep = []
        for s in range(len(o)):
            p = o[s]
            if q_lo <= p < q_hi:
                keep.append(s)
            elif p < q_lo:
                for k in range(1, C + 1):
                    if s + k >= len(o) or i[s + k] != i[s]:
                        break
                    if o[s + k] >= q_lo:
                        if o[s + k] < q_hi:
                            keep.append(s)
                        break
        out.append(keep)
    return out


@pytest.mark.parametrize('q', [(0, 700), (700, 1400), (1400, 2100), (2100, 2800)])
def test_shard_rows_follow_the_rule(q, cuda):
    from asrn_b200 import _lib, stages
    rng = np.random.default_rng(1)
    rows, L, nb, C = 3, 2800, 4, 8
    ids = torch.from_numpy(rng.integers(0, 1 << nb, (rows, L)).astype(np.int16)).to(cuda)
    orden, ids_o = stages.bucket_sort(ids, nb)
    q_lo, q_hi = q
    lib, s = _lib.lib(), _lib.stream_ptr(cuda)
    counts = torch.empty(rows, dtype=torch.int64, device=cuda)
    assert lib.asrn_shard_rows(rows, L, C, q_lo, q_hi, _lib.ptr(orden), _lib.ptr(ids_o), 0, None, None,
                               _lib.ptr(counts), s) == 0
    Lv = int(counts.max())
    ov = torch.empty(rows, Lv, dtype=torch.int32, device=cuda)
    iv = torch.empty(rows, Lv, dtype=torch.int16, device=cuda)
    assert lib.asrn_shard_rows(rows, L, C, q_lo, q_hi, _lib.ptr(orden), _lib.ptr(ids_o), Lv, _lib.ptr(ov),
                               _lib.ptr(iv), None, s) == 0
    o_np, i_np = orden.cpu().numpy(), ids_o.cpu().numpy()
    keep = _rows_rule(o_np, i_np, C, q_lo, q_hi)
    pad = 0 if q_lo > 0 else q_hi
    for r in range(rows):
        n = len(keep[r])
        assert counts[r].item() == n
        assert np.array_equal(ov[r, :n].cpu().numpy(), o_np[r, keep[r]])
        assert np.array_equal(iv[r, :n].cpu().numpy(), i_np[r, keep[r]])
        assert (ov[r, n:].cpu().numpy() == pad).all() and (iv[r, n:].cpu().numpy().view(np.uint16) == 0xFFFF).all()


@pytest.mark.parametrize('world,nb,C', [(2, 4, 8), (4, 4, 8), (3, 6, 32), (4, 14, 32)])
def test_rows_from_tails_equal_rows_from_the_full_sort(world, nb, C, cuda):
    """asrn_shard_merge (each shard sorts only its chunk; earlier chunks reach it as bucket tails) gives exactly the rows
    of asrn_shard_rows over the full sorted rows, and the row lengths; integer work, so bit-exact. Rows span several
    sort tiles (Lc > 8192) in the last case."""
    from types import SimpleNamespace
    from asrn_b200 import _lib, shard, stages
    rng = np.random.default_rng(nb + world)
    rows = 3
    Lc = 12000 if nb == 14 else 700
    L = world * Lc
    ids = rng.integers(0, 1 << nb, (rows, L)).astype(np.int16)
    ids[:, L // 2:L // 2 + 300] = ids[:, 100:400]                 # repeated stretches: long runs in some buckets
    ids_t = torch.from_numpy(ids).to(cuda)
    orden, ids_o = stages.bucket_sort(ids_t, nb)
    layer = SimpleNamespace(n_bits=nb, chunk=C)
    lib, s = _lib.lib(), _lib.stream_ptr(cuda)
    tails = []
    for r in range(world):
        c0 = r * Lc
        o_loc, i_loc = stages.bucket_sort(ids_t[:, c0:c0 + Lc].contiguous(), nb)
        tails.append(shard._tails(layer, o_loc, i_loc, c0))
    tails = torch.stack(tails, 0)
    for r in range(world):
        c0, c1 = r * Lc, (r + 1) * Lc
        o_loc, i_loc = stages.bucket_sort(ids_t[:, c0:c1].contiguous(), nb)
        ov, iv, row_len = shard.shard_rows(layer, o_loc, i_loc, tails[:r] if r > 0 else None, c0, L)
        Lv = ov.shape[1]
        counts = torch.empty(rows, dtype=torch.int64, device=cuda)
        ov_ref = torch.empty(rows, Lv, dtype=torch.int32, device=cuda)
        iv_ref = torch.empty(rows, Lv, dtype=torch.int16, device=cuda)
        assert lib.asrn_shard_rows(rows, L, C, c0, c1, _lib.ptr(orden), _lib.ptr(ids_o), Lv, _lib.ptr(ov_ref),
                                   _lib.ptr(iv_ref), _lib.ptr(counts), s) == 0
        torch.cuda.synchronize()
        assert torch.equal(row_len, counts)
        assert torch.equal(ov, ov_ref) and torch.equal(iv, iv_ref)


@pytest.mark.parametrize('world,B,L', [(2, 2, 6000), (3, 1, 9000), (4, 2, 8192), (2, 1, 40000)])
def test_chunk_ngram_memory_equals_whole_rows(world, B, L, cuda):
    """The n-gram memory computed per chunk (local sort and scans, per-group summaries exchanged, carries folded in
    rank order; the streak carried as an affine map) equals the whole-row computation at every position: seen flags
    bit-exact, Hawkes intensity and streak within 1e-5. Repetitive text (12 symbols, a copied stretch) so that groups
    span chunks; the last case has chunks longer than one sort tile."""
    import asrn_b200
    from asrn_b200 import shard, stages
    torch.manual_seed(3)
    layer = asrn_b200.ASRNLayer(32)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for n_, p_ in layer.named_parameters():
            if n_ in ('log_kappa', 'log_kappa_racha'):
                p_.add_(torch.randn(p_.shape, generator=g) * 0.5)
    layer = layer.to(cuda)
    rng = np.random.default_rng(world * 7 + L)
    tok = rng.integers(0, 12, size=(B, L))
    tok[:, L // 2:L // 2 + L // 8] = tok[:, 100:100 + L // 8]
    sig = torch.from_numpy(tok.astype(np.float32)).to(cuda)
    beta = torch.from_numpy(rng.uniform(0.01, 2.0, size=(B, L))).to(cuda)
    Bt = torch.cumsum(beta, 1)
    la = torch.from_numpy(rng.uniform(-3.0, 0.5, size=(B, L)).astype(np.float32)).to(cuda)
    ref = stages.repetition(layer, sig, beta, Bt, la)
    full = dict(sig=sig, Bt=Bt, log_alfa=la)
    Lc = L // world
    ngs = [shard.ngram_sort(layer, full, r * Lc, Lc, False) for r in range(world)]
    keys = torch.stack([x['keys'] for x in ngs], 0)
    summ = torch.stack([x['summ'] for x in ngs], 0)
    vh = [shard.ngram_finish(layer, full, ngs[r], keys[:r] if r else None, summ[:r] if r else None, r * Lc, Lc,
                             False) for r in range(world)]
    betas = [beta[:, r * Lc:(r + 1) * Lc].contiguous() for r in range(world)]
    maps = torch.stack([shard.racha_chunk(layer, vh[r][0], betas[r], None, False, want_racha=False)[1]
                        for r in range(world)], 0)
    vis = torch.cat([v for v, _ in vh], 1)
    haw = torch.cat([h for _, h in vh], 1)
    racha = torch.cat([shard.racha_chunk(layer, vh[r][0], betas[r], shard.racha_before(maps, r), False)[0]
                       for r in range(world)], 1)
    torch.cuda.synchronize()
    assert torch.equal(vis, ref['vistos'])
    assert rel_err(haw.cpu().numpy(), ref['hawkes'].cpu().numpy()) <= 1e-5
    assert rel_err(racha.cpu().numpy(), ref['racha'].cpu().numpy()) <= 1e-5


def _layer_and_inputs(cuda, d, B, L, nb, seed=0):
    import asrn_b200
    torch.manual_seed(seed)
    layer = asrn_b200.ASRNLayer(d, n_bits=nb)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for n, p in layer.named_parameters():
            if n in ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha', 'cq.weight',
                     'w_sufijo', 'w_vistos', 'g_conf.weight', 'g_conf.bias'):
                p.add_(torch.randn(p.shape, generator=g) * 0.5)
    layer = layer.to(cuda).eval()
    from asrn_b200 import synthetic
    x = torch.from_numpy(synthetic.config_tokens('cfg4', B=B, L=L, seed=seed) % 512).to(cuda)
    table = torch.randn(512, d, generator=g).to(cuda)
    E = table[x]
    h = E + torch.randn(B, L, d, generator=g).to(cuda) * 0.5
    return layer, E, h, x


@pytest.mark.parametrize('world,half,B,L,nb', [(2, False, 2, 4096, 4), (4, False, 1, 8192, 6), (2, True, 2, 4096, 4),
                                               (4, True, 1, 8192, 14), (2, False, 1, 40960, 6)])
def test_emulated_sharded_forward_matches_unsharded(world, half, B, L, nb, cuda):
    """The sharded algorithm (clock offsets, halo, exclusive rings, queries restricted to the shard, n-gram memory
    over the full sequence) gives the unsharded layer's h' (fp32: 1e-4; bf16: 2e-2). Few buckets (nb = 4 / 6) so
    that rings cross chunk boundaries; the last case has rows longer than one sort / n-gram tile."""
    from asrn_b200 import shard
    layer, E, h, x = _layer_and_inputs(cuda, 64, B, L, nb)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
        ref = layer(E, h, x)
        got = shard.forward_emulated(layer, E, h, x, world)
    tol = 2e-2 if half else 1e-4
    assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) <= tol
    assert rel_err((got - h).cpu().numpy(), (ref - h).cpu().numpy()) <= tol


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason='needs 2 GPUs')
def test_two_nccl_ranks_match_unsharded():
    """Two processes, one GPU each, NCCL all-gathers: each rank's h' chunk equals the unsharded layer's."""
    env = dict(os.environ, NCCL_NVLS_ENABLE='0')
    cmd = ['timeout', '-k', '30', '240', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node=2', '--master-addr=127.0.0.1', f'--master-port={_free_port()}',
           os.path.join(HERE, '_shard_ranks.py')]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert 'shard ranks ok' in r.stdout
