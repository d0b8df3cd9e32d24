"""Host logic of the sequence-chunk sharding (asrn_b200/shard.py) on the CPU: chunk bounds, clock offsets and the
exchange steps as world-size-2 gloo ranks (the NCCL path runs the same calls on GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch


def test_chunk_bounds():
    from asrn_b200 import shard
    assert [shard.chunk_bounds(12, 3, r) for r in range(3)] == [(0, 4), (4, 8), (8, 12)]
    with pytest.raises(ValueError):
        shard.chunk_bounds(10, 3, 0)


def test_streak_before_each_chunk_composes_the_earlier_maps():
    """racha_before folds the earlier chunks' affine maps S_last = A S_before + B in rank order: equal to running the
    streak recursion S_t = a_t S_{t-1} + r_t over the whole row."""
    from asrn_b200 import shard
    rng = np.random.default_rng(1)
    world, Lc = 4, 6
    a = rng.uniform(0.0, 1.0, (world * Lc,))
    r = rng.integers(0, 2, (world * Lc,)).astype(np.float64)
    S, before = 0.0, []
    maps = []
    for q in range(world):
        before.append(S)
        A, B0 = 1.0, 0.0
        for t in range(q * Lc, (q + 1) * Lc):
            S = a[t] * S + r[t]
            A, B0 = a[t] * A, a[t] * B0 + r[t]
        maps.append([A, B0])
    m = torch.tensor(maps, dtype=torch.float32).view(world, 1, 2)
    for q in range(world):
        assert abs(shard.racha_before(m, q).item() - before[q]) <= 1e-5 * max(1.0, abs(before[q]))


def test_clock_offsets_give_the_global_cumulative_sum():
    from asrn_b200 import shard
    rng = np.random.default_rng(0)
    B, world, Lc = 2, 3, 5
    beta = torch.from_numpy(rng.uniform(0.01, 2.0, (B, world * Lc)))
    local = torch.cat([torch.cumsum(beta[:, r * Lc:(r + 1) * Lc], 1) for r in range(world)], 1)
    sums = torch.stack([local[:, (r + 1) * Lc - 1] for r in range(world)], 0)
    shard._apply_clock_offsets(local, sums, Lc)
    assert torch.allclose(local, torch.cumsum(beta, 1), rtol=1e-14, atol=0)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from asrn_b200 import shard
        res = {}
        last = torch.full((2, 3), float(rank + 1))
        res['halo'] = shard.exchange_halo(last, world, rank)
        res['sums'] = shard.exchange_chunk_sums(torch.tensor([rank + 0.5, 10.0 * rank], dtype=torch.float64), world)
        res['seq1'] = shard._gather_seq(torch.arange(4).view(1, 4, 1) + 100 * rank, world, None)
        res['seq2'] = shard._gather_seq(torch.arange(8).view(2, 4) + 100 * rank, world, None)
        tails = (torch.arange(2 * 4 * 3).view(2, 4, 3) + 1000 * rank).to(torch.int32)
        res['tails'] = shard.exchange_tails(tails, world, None)
        keys = (torch.arange(6).view(2, 3) + 10 * rank).to(torch.int64)
        summ = torch.full((2, 3, 32), rank + 1, dtype=torch.uint8)
        res['ng'] = shard.exchange_ngram(keys, summ, world, None)
        res['maps'] = shard.exchange_racha_maps(torch.tensor([[0.5, 1.0 + rank]]), world, None)
        n = 2 + rank                                          # ranks publish different numbers of rows
        payload = (torch.arange(n * 6).view(n, 6) + 100 * rank).to(torch.uint8)
        pay_all, idx_all, finish = shard.exchange_rows_async(payload, torch.arange(n) * 10 + rank, world, None)
        finish()
        res['rows'] = (pay_all, idx_all)
        res['firsts'] = shard.exchange_first_rows(torch.full((2, 4), float(rank + 1)).to(torch.bfloat16), world, None)
        torch.save(res, os.path.join(out, f'rank{rank}.pt'))
    finally:
        dist.destroy_process_group()


def test_exchange_steps_with_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method='spawn')
    r0 = torch.load(tmp_path / 'rank0.pt')
    r1 = torch.load(tmp_path / 'rank1.pt')
    assert torch.equal(r0['halo'], torch.zeros(2, 3)) and torch.equal(r1['halo'], torch.full((2, 3), 1.0))
    for r in (r0, r1):
        assert torch.equal(r['sums'], torch.tensor([[0.5, 0.0], [1.5, 10.0]], dtype=torch.float64))
        assert torch.equal(r['seq1'].view(-1), torch.tensor([0, 1, 2, 3, 100, 101, 102, 103]))
        expect2 = torch.cat([torch.arange(8).view(2, 4), torch.arange(8).view(2, 4) + 100], 1)
        assert torch.equal(r['seq2'], expect2)
        t0 = torch.arange(2 * 4 * 3).view(2, 4, 3).to(torch.int32)
        assert torch.equal(r['tails'], torch.stack([t0, t0 + 1000], 0))
        k0 = torch.arange(6).view(2, 3).to(torch.int64)
        assert torch.equal(r['ng'][0], torch.stack([k0, k0 + 10], 0))
        assert (r['ng'][1][0] == 1).all() and (r['ng'][1][1] == 2).all()
        assert torch.equal(r['maps'], torch.tensor([[[0.5, 1.0]], [[0.5, 2.0]]]))
        pay_all, idx_all = r['rows']
        assert pay_all.shape == (2, 3, 6) and idx_all.tolist() == [[0, 10, -1], [1, 11, 21]]
        assert torch.equal(pay_all[0, :2], torch.arange(12).view(2, 6).to(torch.uint8))
        assert torch.equal(pay_all[1], (torch.arange(18).view(3, 6) + 100).to(torch.uint8))
        assert torch.equal(r['firsts'].float(), torch.stack([torch.full((2, 4), 1.0), torch.full((2, 4), 2.0)]))


# ---- failure detection of the exchange (host-side faults on gloo ranks; no GPU involved) -----------------------------

def _carries(rank, world, Lc=4, C=3, rows=2, nbins=4, B=2):
    """A consistent set of one rank's carries: chunk sums of beta, bucket tails inside the rank's chunk, sorted n-gram
    keys and streak maps."""
    sums = torch.tensor([1.5 + rank, 0.25], dtype=torch.float64)
    tails = torch.zeros(rows, nbins, C + 1, dtype=torch.int32)
    for r in range(rows):
        for b in range(nbins):
            n = (r + b + rank) % (C + 1)
            tails[r, b, 0] = n
            tails[r, b, 1:1 + n] = torch.arange(n, dtype=torch.int32) + rank * Lc
    keys = torch.arange(B * 3 * Lc, dtype=torch.int64).view(B * 3, Lc) * 7 + 5     # unsigned images: ascending
    maps = torch.tensor([[0.5, 1.0 + rank]] * B, dtype=torch.float32)
    return sums, tails, keys, maps


def _exchange_and_validate(world, rank, corrupt=None, Lc=4, C=3):
    from asrn_b200 import shard
    sums, tails, keys, maps = _carries(rank, world, Lc, C)
    if corrupt == 'tail_count' and rank == 1:
        tails[0, 1, 0] = C + 2
    if corrupt == 'tail_position' and rank == 1:
        tails[1, 2, 0] = 2
        tails[1, 2, 1:3] = torch.tensor([0, 1], dtype=torch.int32)          # rank 0's chunk, not rank 1's
    if corrupt == 'sum' and rank == 1:
        sums[0] = float('nan')
    if corrupt == 'map' and rank == 1:
        maps[0, 0] = 3.0
    if corrupt == 'keys' and rank == 1:
        keys[0, 1] = keys[0, 2] + 1                                         # out of order
    s = shard.exchange_chunk_sums(sums, world)
    t = shard.exchange_tails(tails, world)
    k, _ = shard.exchange_ngram(keys, torch.zeros(keys.shape + (32,), dtype=torch.uint8), world)
    m = shard.exchange_racha_maps(maps, world)
    n = int(shard.carry_violations(sums=s, maps=m, keys=k, tails=t, Lc=Lc, C=C))
    if n:
        raise shard.ShardExchangeError(f'{n} violations')
    return 'ok'


def _fault_rank(rank, world, port, out, scenario, timeout_s):
    """One gloo rank of a fault scenario; records what it observed in out/rank<r>.txt and exits 0 (a rank that hit
    an error leaves without tearing the group down: its peers may be gone)."""
    import datetime
    import time
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    from asrn_b200 import shard
    t0 = time.time()
    try:
        if scenario.startswith('corrupt_'):
            res = _exchange_and_validate(world, rank, corrupt=scenario[len('corrupt_'):])
        elif scenario == 'clean':
            res = _exchange_and_validate(world, rank)
        elif scenario == 'late_within_timeout':
            if rank == 1:
                time.sleep(1.0)
            res = _exchange_and_validate(world, rank)
        elif scenario == 'late_past_timeout':
            if rank == 1:
                time.sleep(3 * timeout_s)
            res = _exchange_and_validate(world, rank)
        elif scenario == 'leaves_between_steps':
            _exchange_and_validate(world, rank)                            # step 1: every rank
            if rank == 1:
                with open(os.path.join(out, f'rank{rank}.txt'), 'w') as f:
                    f.write('left 0.0')
                os._exit(0)                                                  # gone before step 2
            res = _exchange_and_validate(world, rank)                        # step 2: the peer has left
        else:
            raise ValueError(scenario)
    except shard.ShardExchangeError:
        res = 'invalid'
    except Exception as exc:                                                # the backend's error for a lost peer
        res = 'error:' + type(exc).__name__
    with open(os.path.join(out, f'rank{rank}.txt'), 'w') as f:
        f.write(f'{res} {time.time() - t0:.2f}')
    if res == 'ok':
        dist.destroy_process_group()
    os._exit(0)


def _run_fault(tmp_path, scenario, timeout_s=3):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_fault_rank, args=(world, _free_port(), str(tmp_path), scenario, timeout_s), nprocs=world,
                       start_method='spawn')
    out = []
    for r in range(world):
        res, secs = (tmp_path / f'rank{r}.txt').read_text().split()
        out.append((res, float(secs)))
    return out


@pytest.mark.timeout(120)
@pytest.mark.parametrize('what', ['tail_count', 'tail_position', 'sum', 'map', 'keys'])
def test_exchange_detects_a_corrupted_carry(tmp_path, what):
    """A rank that sends inconsistent carry state: every rank's validation of the gathered state reports it."""
    res = _run_fault(tmp_path, 'corrupt_' + what)
    assert [r for r, _ in res] == ['invalid', 'invalid']


@pytest.mark.timeout(120)
@pytest.mark.parametrize('scenario', ['clean', 'late_within_timeout'])
def test_exchange_of_consistent_carries_passes(tmp_path, scenario):
    """Consistent carries pass validation, also when one rank reaches the exchange late but within the timeout."""
    assert [r for r, _ in _run_fault(tmp_path, scenario)] == ['ok', 'ok']


@pytest.mark.timeout(120)
def test_exchange_reports_a_rank_late_past_the_timeout(tmp_path):
    """Rank 1 reaches the exchange three timeouts late: rank 0's collective ends with the backend's error within a
    few timeouts instead of waiting for it."""
    res = _run_fault(tmp_path, 'late_past_timeout', timeout_s=2)
    assert res[0][0].startswith('error:')
    assert res[0][1] < 5 * 2


@pytest.mark.timeout(120)
def test_exchange_reports_a_rank_that_left_between_steps(tmp_path):
    """Rank 1 leaves after step 1: rank 0's step-2 exchange ends with an error instead of hanging."""
    res = _run_fault(tmp_path, 'leaves_between_steps', timeout_s=3)
    assert res[1][0] == 'left'
    assert res[0][0].startswith('error:')
    assert res[0][1] < 5 * 3


# ---- the compact row exchange (host logic of shard.tail_index / _row_payload / _scatter_rows) ------------------------

def test_tail_index_lists_each_tail_position_once():
    from asrn_b200 import shard
    B, T, nb, C, Lc, c0 = 2, 3, 3, 4, 10, 20
    tails = torch.zeros(B * T, 1 << nb, C + 1, dtype=torch.int32)
    tails[0, 1, 0] = 2
    tails[0, 1, 1:3] = torch.tensor([c0 + 3, c0 + 7])
    tails[2, 4, 0] = 3                                   # the same sequence (row 2 -> b = 0), one position repeated
    tails[2, 4, 1:4] = torch.tensor([c0 + 1, c0 + 3, c0 + 9])
    tails[4, 5, 0] = 1                                   # row 4 -> b = 1
    tails[4, 5, 1] = c0 + 9
    tails[5, 6, 1:] = c0 + 5                             # count 0: these entries are not part of the tail
    assert shard.tail_index(tails, c0, Lc, B, T).tolist() == [1, 3, 7, 9, 19]


def test_scattered_rows_land_at_the_key_and_the_value_after_it():
    """A published row of position p fills phi / Qc / Kc at p and the value row (E of p + 1) at p + 1, as the scoring
    kernel reads them; the value row of a sequence's last position is dropped."""
    from asrn_b200 import shard
    B, Lc, L, c0, d, P, cf = 1, 4, 8, 0, 4, 3, 2
    loc = {'phi': torch.arange(B * Lc * P, dtype=torch.float32).view(B, Lc, P).to(torch.bfloat16),
           'Qc': torch.ones(B, Lc, cf, dtype=torch.bfloat16), 'Kc': torch.full((B, Lc, cf), 2.0).to(torch.bfloat16),
           'Ea': (torch.arange(B * Lc * d, dtype=torch.float32).view(B, Lc, d) + 100).to(torch.bfloat16)}
    nxt = torch.full((B, 1, d), 7.0).to(torch.bfloat16)   # the next chunk's first row
    Ea_next = torch.cat([loc['Ea'][:, 1:], nxt], 1)
    sel = torch.tensor([1, 3])
    payload = shard._row_payload(loc, sel, Ea_next)
    widths = shard._row_widths(loc, Ea_next)
    full = {k: torch.zeros((B * L + 1,) + tuple(loc[k].shape[2:]), dtype=torch.bfloat16)   # + the spare row
            for k in ('phi', 'Qc', 'Kc', 'Ea')}
    padded = torch.cat([payload, torch.zeros_like(payload[:1])])          # a padding row, index -1
    shard._scatter_rows(full, padded, torch.tensor([1, 3, -1]), widths, L)
    f = {k: v[:B * L].view((B, L) + tuple(v.shape[1:])) for k, v in full.items()}
    assert torch.equal(f['phi'][0, 1], loc['phi'][0, 1]) and torch.equal(f['phi'][0, 3], loc['phi'][0, 3])
    assert torch.equal(f['Kc'][0, 3], loc['Kc'][0, 3]) and f['phi'][0, 2].abs().sum() == 0
    assert torch.equal(f['Ea'][0, 2], loc['Ea'][0, 2]) and torch.equal(f['Ea'][0, 4], nxt[0, 0])
    assert f['phi'][0, L - 1].abs().sum() == 0                          # the padding row went to the spare row
    before = full['Ea'].clone()
    shard._scatter_rows(full, payload[1:], torch.tensor([L - 1]), widths, L)   # last position: no value row
    assert torch.equal(full['Ea'][:B * L], before[:B * L])


def test_compact_tails_round_trip():
    """The exchanged form of the tails (non-empty buckets only) expands back to the dense array."""
    from asrn_b200 import shard
    g = torch.Generator().manual_seed(0)
    tails = torch.zeros(2, 3, 8, 5, dtype=torch.int32)
    for q in range(2):
        for _ in range(6):
            r, b = int(torch.randint(3, (1,), generator=g)), int(torch.randint(8, (1,), generator=g))
            n = int(torch.randint(1, 5, (1,), generator=g))
            tails[q, r, b, 0] = n
            tails[q, r, b, 1:1 + n] = torch.arange(n, dtype=torch.int32) + 10 * q
    packed = [shard.compact_tails(tails[q]) for q in range(2)]
    m = max(ix.numel() for _, ix in packed) + 1
    ent = torch.zeros(2, m, 20, dtype=torch.uint8)
    idx = torch.full((2, m), -1, dtype=torch.int64)
    for q, (e, ix) in enumerate(packed):
        ent[q, :ix.numel()] = e
        idx[q, :ix.numel()] = ix
    assert torch.equal(shard.expand_tails(ent, idx, tails.shape[1:]), tails)


def test_compact_equals_nonzero():
    """The synchronisation-free compactions of set flags give nonzero()'s indices (padded with -1 up to a capacity,
    or cut at it)."""
    from asrn_b200 import shard
    g = torch.Generator().manual_seed(3)
    for n in (1, 17, 1000):
        flags = torch.rand(n, generator=g) < 0.3
        want = flags.nonzero().squeeze(1)
        m = want.numel()
        assert torch.equal(shard.compact(flags, m), want)
        padded = shard.compact_cap(flags, m + 5)
        assert torch.equal(padded[:m], want) and (padded[m:] == -1).all()
        if m > 2:
            assert torch.equal(shard.compact_cap(flags, m - 2), want[:m - 2])


def test_pack_unpack_round_trip():
    """The packed exchange buffer: parts of mixed types and shapes (a size-1 column slice included, whose stride is
    not 1) come back unchanged from a (world, bytes) buffer."""
    from asrn_b200.shard import _pack, _unpack
    g = torch.Generator().manual_seed(0)
    Bt = torch.randn(1, 4096, dtype=torch.float64, generator=g)
    parts = [Bt[:, -1], Bt, torch.randint(0, 9, (3, 5), dtype=torch.int32, generator=g),
             torch.randn(2, 3, generator=g).to(torch.bfloat16), torch.randint(0, 2, (7,), dtype=torch.uint8,
                                                                               generator=g)]
    buf, meta = _pack(parts)
    assert buf.dtype == torch.uint8 and buf.numel() % 8 == 0
    world = torch.stack([buf, buf])
    for i, t in enumerate(parts):
        got = _unpack(world, meta, i)
        assert got.shape == (2,) + tuple(t.shape)
        assert torch.equal(got[1], t) and got.dtype == t.dtype
