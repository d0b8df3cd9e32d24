"""Sequence-chunk sharding of one ASRN layer forward over several GPUs (one long sequence, e.g. 262,144 tokens).

The reference runs a sequence on one device; here rank r of `world` owns the contiguous positions [c0, c1) of every
sequence (L = world * Lc, equal chunks) and computes h' for them:

  phase 1 (local)   the context stage and the sign-hash projection of the chunk (asrn/estable.py:153-194,
                    asrn/nucleo.py:644-664); the hash of the chunk's first position needs E of the previous position,
                    the one-row halo from rank r - 1 (zeros on rank 0, as the reference's E_{-1} = 0)
                    then the sort of the chunk's rows by bucket (asrn/estable.py:220-221) and per (row, bucket) the
                    bucket's tail, its last <= C positions (asrn_shard_tails)
  exchange (NCCL)   (1) the halo rows, (2) per sequence the chunk's sum of beta (fp64): rank r's clock is the
                    exclusive sum of the earlier chunks plus its own cumulative sum (asrn/estable.py:418),
                    (3) the bucket tails, (4) the per-position scalars (signature, clock, beta, log_alfa) of all L
                    positions, (5) the feature rows (phi, Qc, Kc) and value rows (bf16 E of the next position) of
                    only the positions in each rank's tails: a later rank's rows hold no other earlier-chunk position,
                    so the rows every rank receives shrink from all L positions to the union of the tails, plus the
                    first bf16 E row of every chunk (the value row of the chunk before's last position); all-gathers
                    over NVLink
  phase 2 (local)   the shard's own rows: for every bucket with local slots its exclusive ring -- the C most recent
                    earlier-chunk positions, from the earlier ranks' tails -- then its local run (asrn_shard_merge);
                    candidate scoring of the local queries (asrn_score_shard); the n-gram memory over the full
                    sequence (its Hawkes and streak scans carry state across chunks), kept for the chunk; the gate
                    of the chunk.

`forward` runs one rank under torch.distributed (NCCL); `forward_emulated` runs every rank's phases in one process
(the exchange becomes concatenation), so that the sharded algorithm can be checked against the unsharded layer on one
GPU. The exchange is NCCL collectives only (no peer-memory loads in the kernels). No step waits on the host: every
shard row's length stays on the device (the rows are sized by a bound, the scoring kernel stops at each row's end).

Failure detection. Every received carry is checked on the device: the chunk sums of beta (finite, >= 0), the streak
maps (A in [0, 1], B0 finite and >= 0), the sorted n-gram keys (ascending) and, inside asrn_shard_merge, each bucket
tail it uses (count in [0, C], positions ascending inside the sender's chunk; an inconsistent tail is treated as empty,
so it cannot index features out of range). The result lands in a device status word whose copy to the host is read
without stalling the stream: the next forward raises ShardExchangeError if the previous one saw a violation, and
check_exchange(device) waits for it. A rank that is late beyond the process group's timeout, or that left, makes the
other ranks' next collective fail with the backend's error (give the group a short timeout).
"""
import torch

from . import _lib, stages
from .layer import compute_half, ctypes_ref

_SEQ_KEYS = ('phi', 'Qc', 'Kc', 'sig', 'log_alfa', 'beta', 'Bt', 'Ea')
_SCALAR_KEYS = ('sig', 'log_alfa', 'beta', 'Bt')      # gathered for every position (24 B each)
last_exchange = {}    # this rank's last compact row exchange: rows sent, padded rows per rank, rows in the chunk
_ROW_KEYS = ('phi', 'Qc', 'Kc')                       # gathered only for the positions in the tails


def tail_flags(tails, c0, Lc, B, T):
    """(B * Lc,) bool: which positions p of this chunk (flat index b * Lc + p - c0) appear in its bucket tails (rows
    b * T + tau), the only positions of the chunk that a later shard's rows hold. No host synchronisation."""
    dev = tails.device
    rows, _, C1 = tails.shape
    C = C1 - 1
    cnt = tails[..., 0].long().clamp(0, C)
    valid = torch.arange(C, device=dev) < cnt.unsqueeze(-1)
    rel = torch.where(valid, tails[..., 1:].long() - c0, Lc).clamp(0, Lc)
    b = (torch.arange(rows, device=dev) // T).view(rows, 1, 1)
    flags = torch.zeros(B * (Lc + 1), dtype=torch.bool, device=dev)
    flags.index_fill_(0, (b * (Lc + 1) + rel).view(-1), True)
    return flags.view(B, Lc + 1)[:, :Lc].reshape(-1)


def compact(flags, n):
    """The ascending indices of the n set flags (n known to the host), without a host synchronisation."""
    dev = flags.device
    pos = torch.cumsum(flags.long(), 0) - 1
    out = torch.full((flags.numel() + 1,), -1, dtype=torch.int64, device=dev)
    out.index_put_((torch.where(flags, pos, flags.numel()),), torch.arange(flags.numel(), device=dev))
    return out[:n]


def compact_cap(flags, cap):
    """The ascending indices of the set flags in a (cap,) tensor padded with -1 (flags past cap are dropped: the
    caller checks the count against cap on the device)."""
    dev = flags.device
    pos = torch.cumsum(flags.long(), 0) - 1
    out = torch.full((max(flags.numel(), cap) + 1,), -1, dtype=torch.int64, device=dev)
    tgt = torch.where(flags & (pos < cap), pos, out.numel() - 1)
    out.index_put_((tgt,), torch.arange(flags.numel(), device=dev))
    out[-1:].fill_(-1)
    return out[:cap]


def tail_index(tails, c0, Lc, B, T):
    """Local flat indices b * Lc + (p - c0), ascending, of the positions p of this chunk in its bucket tails."""
    return tail_flags(tails, c0, Lc, B, T).nonzero().squeeze(1)


def compact_tails(tails, n=None):
    """The non-empty bucket tails of a chunk: flat indices row * 2^nb + bucket (int64) and their (count, positions)
    entries as raw bytes (n, (C + 1) * 4). In the heavy regime few buckets are used, so this is far smaller than the
    dense (rows, 2^nb, C + 1) array the merge kernel reads. n: their number if the host knows it (no synchronisation)."""
    flat = tails.reshape(-1, tails.shape[-1])
    ne = flat[:, 0] != 0
    nz = ne.nonzero().squeeze(1) if n is None else compact(ne, n)
    return flat[nz].contiguous().view(torch.uint8), nz


def expand_tails(ent_all, idx_all, shape):
    """(world, m, bytes) entries and (world, m) indices (-1 = padding) -> dense (world,) + shape int32 tails, zeros
    (empty tails) elsewhere."""
    world = ent_all.shape[0]
    R = 1
    for x in shape[:-1]:
        R *= x
    flat = torch.zeros(world * R + 1, shape[-1], dtype=torch.int32, device=ent_all.device)
    # every rank's entries in one copy (the same launches whatever the number of ranks)
    rows = ent_all.contiguous().view(torch.int32).view(-1, shape[-1])
    base = torch.arange(world, device=idx_all.device).unsqueeze(1) * R
    dst = torch.where(idx_all >= 0, base + idx_all, world * R).reshape(-1)   # padding into the spare row
    flat.index_copy_(0, dst, rows)
    return flat[:world * R].view((world,) + tuple(shape))


def _row_payload(loc, sel, Ea_next):
    """(n, row bytes) uint8: for each selected local position its phi, Qc and Kc rows and the bf16 E row of the
    next position (its value row), as raw bytes."""
    parts = []
    for k in _ROW_KEYS:
        x = loc[k]
        parts.append(x.reshape(-1, x.shape[-1])[sel].contiguous().view(torch.uint8))
    parts.append(Ea_next.reshape(-1, Ea_next.shape[-1])[sel].contiguous().view(torch.uint8))
    return torch.cat(parts, 1)


def _row_payload_next(loc, sel, Lc):
    """As _row_payload, with the value rows taken straight from the chunk's own E rows: the value row of local
    position p is E[p + 1]; a sequence's last local position gets a zero row (the receiver writes the next chunk's
    first row there). Only the selected rows are read (no shifted copy of the chunk)."""
    parts = []
    for k in _ROW_KEYS:
        x = loc[k]
        parts.append(x.reshape(-1, x.shape[-1])[sel].contiguous().view(torch.uint8))
    ea = loc['Ea'].reshape(-1, loc['Ea'].shape[-1])
    rows = ea[(sel + 1).clamp(max=ea.shape[0] - 1)]
    rows = rows.masked_fill(((sel % Lc) == Lc - 1).unsqueeze(1), 0)
    parts.append(rows.contiguous().view(torch.uint8))
    return torch.cat(parts, 1)


def _row_widths(loc, Ea_next):
    return [loc[k].shape[-1] * loc[k].element_size() for k in _ROW_KEYS] + \
        [Ea_next.shape[-1] * Ea_next.element_size()]


def _full_rows(loc, B, L, c0, c1, Ea_first_next):
    """Zero-filled feature tensors of B * L rows (flat index b * L + p) plus one spare row at the end, holding this
    chunk's own rows and, at c1, the next chunk's first value row; the earlier chunks' rows are scattered in by
    _scatter_rows (padding entries land in the spare row, so no step needs the host)."""
    full = {}
    for k in _ROW_KEYS + ('Ea',):
        x = loc[k]
        t = torch.zeros((B * L + 1,) + tuple(x.shape[2:]), dtype=x.dtype, device=x.device)
        t[:B * L].view((B, L) + tuple(x.shape[2:]))[:, c0:c1] = x
        full[k] = t
    if Ea_first_next is not None and c1 < L:
        full['Ea'][:B * L].view((B, L) + tuple(Ea_first_next.shape[1:]))[:, c1] = Ea_first_next
    return full


def _scatter_rows(full, payload, gidx, widths, L):
    """Rows of another chunk (payload (n, bytes), global flat indices b * L + p, -1 = padding) into full: phi, Qc, Kc
    at p, the value row at p + 1 (where the scoring kernel reads the value of key p)."""
    off = 0
    for k, w in zip(_ROW_KEYS + ('Ea',), widths):
        t = full[k].view(-1, full[k].shape[-1])
        spare = t.shape[0] - 1
        rows = payload[:, off:off + w].contiguous().view(t.dtype).view(-1, t.shape[-1])
        if k == 'Ea':                                   # the value row of the sequence's last position is unused
            dst = torch.where((gidx >= 0) & ((gidx + 1) % L != 0), gidx + 1, spare)
        else:
            dst = torch.where(gidx >= 0, gidx, spare)
        t.index_copy_(0, dst, rows)                     # padding rows all land in the spare row
        off += w


class ShardExchangeError(RuntimeError):
    """State received from another shard broke its invariants (corrupted in transit or sent by a faulty rank)."""


def carry_violations(sums=None, maps=None, keys=None, tails=None, Lc=None, C=None):
    """Number of invariant violations (int64 tensor on the carries' device; 0 = consistent) in exchanged carries:
      sums  (world, B) fp64 chunk sums of beta: finite and >= 0 (beta = min(softplus, beta_max) >= 0);
      maps  (world, B, 2) streak maps S_last = A S_before + B0: A in [0, 1], B0 finite and >= 0;
      keys  (world, B * n, Lc) sorted n-gram keys: ascending along the last dimension;
      tails (world, rows, 2^nb, C + 1) bucket tails: count in [0, C], positions strictly ascending inside the sender's
            chunk [r Lc, (r + 1) Lc). (On the GPU the merge kernel checks the tails it uses; this full scan is for the
            host-side path.)"""
    bad = []
    if sums is not None:
        bad.append((~torch.isfinite(sums) | (sums < 0)).sum())
    if maps is not None:
        A, B0 = maps[..., 0], maps[..., 1]
        bad.append((~torch.isfinite(maps).all(-1) | (A < 0) | (A > 1) | (B0 < 0)).sum())
    if keys is not None and keys.shape[-1] > 1:
        k = keys.view(torch.int64) if keys.dtype != torch.int64 else keys
        # order-preserving images of the fp64 keys are unsigned 64-bit: compare with the sign bit flipped
        flip = torch.bitwise_xor(k, -(1 << 63))
        bad.append((flip[..., 1:] < flip[..., :-1]).sum())
    if tails is not None:
        world = tails.shape[0]
        cnt = tails[..., 0].to(torch.int64)
        pos = tails[..., 1:].to(torch.int64)
        used = torch.arange(C, device=tails.device) < cnt.unsqueeze(-1)
        lo = (torch.arange(world, device=tails.device, dtype=torch.int64) * Lc).view(world, 1, 1, 1)
        out = used & ((pos < lo) | (pos >= lo + Lc))
        desc = used[..., 1:] & (pos[..., 1:] <= pos[..., :-1])
        bad += [((cnt < 0) | (cnt > C)).sum(), out.sum(), desc.sum()]
    if not bad:
        return torch.zeros((), dtype=torch.int64)
    return torch.stack([b.to(torch.int64) for b in bad]).sum()


_pending = {}


def _defer_status(status):
    """Copy a step's status word to pinned host memory behind the step's work; read it at the next forward."""
    dev = status.device
    host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    host.copy_(status.view(1), non_blocking=True)
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(dev))
    _pending[dev] = (host, ev)


def _raise_reported(dev, block):
    item = _pending.get(dev)
    if item is None:
        return
    host, ev = item
    if not block and not ev.query():
        return
    ev.synchronize()
    del _pending[dev]
    st = int(host.item())
    if st != 0:
        raise ShardExchangeError(f'a sharded forward received inconsistent state from another shard (status {st}: '
                                 f'{_lib.lib().asrn_status_string(st).decode() if st < 16 else "invalid carries"})')


def check_exchange(device):
    """Wait for the last sharded forward on `device` and raise ShardExchangeError if it received inconsistent state."""
    _raise_reported(torch.device(device), block=True)


def chunk_bounds(L, world, rank):
    """[c0, c1) of rank `rank` when L positions are split in `world` equal contiguous chunks."""
    if L % world:
        raise ValueError(f'sequence length {L} is not a multiple of the {world} ranks')
    Lc = L // world
    return rank * Lc, (rank + 1) * Lc


def _phase1(layer, E, h, tokens, E_halo, half, c0, E_ext=None):
    """Local stages of one chunk starting at position c0. E, h (B, Lc, d) fp32, tokens (B, Lc) or None, E_halo (B, d):
    E of the position before the chunk. E_ext: a (B, Lc + 1, d) buffer whose rows 1 .. Lc are E's own storage; the
    halo goes to its row 0 (else the extended rows are a copy)."""
    ctx = stages.context(layer, h, tokens, E=None if tokens is not None else E, half=half)
    Bt = stages.clock(ctx['beta'])
    if E_ext is not None and E_ext.shape[1] == E.shape[1] + 1 and E_ext[:, 1:].data_ptr() == E.data_ptr():
        E_ext[:, 0].copy_(E_halo)
    else:
        E_ext = torch.cat([E_halo.unsqueeze(1).to(E.dtype), E], 1)
    hs = stages.hash(layer, E_ext, half=half)
    B, Lc = E.shape[:2]
    T = layer.n_tablas
    loc = dict(phi=hs['phi'][:, 1:].contiguous(), Qc=ctx['Qc'], Kc=ctx['Kc'], sig=ctx['sig'],
               log_alfa=ctx['log_alfa'], beta=ctx['beta'], Bt=Bt, Ea=hs['Ea'][:, 1:].contiguous(),
               glogit=ctx['glogit'])
    ids = hs['ids_rows'].view(B * T, Lc + 1)[:, 1:].contiguous()
    loc['orden'], loc['ids'] = stages.bucket_sort(ids, layer.n_bits)
    loc['tails'] = _tails(layer, loc['orden'], loc['ids'], c0)
    return loc


def _workspace(layer, rows, dev):
    n = _lib.lib().asrn_shard_workspace_bytes(rows, layer.n_bits)
    if n == 0:
        raise ValueError(f'sequence sharding needs n_bits <= 15 (got {layer.n_bits})')
    return torch.empty(n, dtype=torch.uint8, device=dev)


def _tails(layer, orden_loc, ids_loc, c0):
    """(rows, 2^nb, C + 1) int32 bucket tails of a sorted chunk: [0] = count, then its last <= C global positions."""
    rows, Lc = orden_loc.shape
    dev = orden_loc.device
    C = layer.chunk
    tails = torch.empty(rows, 1 << layer.n_bits, C + 1, dtype=torch.int32, device=dev)
    ws = _workspace(layer, rows, dev)
    _lib.check(_lib.lib().asrn_shard_tails(rows, Lc, layer.n_bits, C, c0, _lib.ptr(orden_loc), _lib.ptr(ids_loc),
                                           _lib.ptr(tails), _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev)),
               'asrn_shard_tails')
    return tails


def shard_rows(layer, orden_loc, ids_loc, tails_prev, c0, L, status=None):
    """The shard's sorted rows from its sorted chunk and the earlier ranks' tails (n_prev, rows, 2^nb, C + 1):
    (orden_v, ids_v) (rows, Lv) and the used length of every row (rows,) int64, all on the device. status (1,) int32
    on the device (optional) receives ASRN_ERR_DATA if a received tail is inconsistent."""
    rows, Lc = orden_loc.shape
    dev = orden_loc.device
    C, nb = layer.chunk, layer.n_bits
    Lv = (Lc + min(c0, (1 << nb) * C) + 31) // 32 * 32
    orden_v = torch.empty(rows, Lv, dtype=torch.int32, device=dev)
    ids_v = torch.empty(rows, Lv, dtype=torch.int16, device=dev)
    row_len = torch.empty(rows, dtype=torch.int64, device=dev)
    ws = _workspace(layer, rows, dev)
    n_prev = 0 if tails_prev is None else tails_prev.shape[0]
    _lib.check(_lib.lib().asrn_shard_merge(rows, Lc, nb, C, c0, n_prev,
                                           None if n_prev == 0 else _lib.ptr(tails_prev), _lib.ptr(orden_loc),
                                           _lib.ptr(ids_loc), Lv, _lib.ptr(orden_v), _lib.ptr(ids_v),
                                           _lib.ptr(row_len), L, _lib.ptr(ws), ws.numel(), _lib.ptr(status),
                                           _lib.stream_ptr(dev)),
               'asrn_shard_merge')
    return orden_v, ids_v, row_len


def _apply_clock_offsets(Bt_full, chunk_sums, Lc):
    """Bt_full (B, L) of local cumulative sums per chunk; chunk_sums (world, B) fp64 -> global clock in place."""
    world = chunk_sums.shape[0]
    offs = torch.cumsum(chunk_sums, 0) - chunk_sums                # exclusive sum over the earlier chunks
    Bt_full.view(Bt_full.shape[0], world, Lc).add_(offs.transpose(0, 1).unsqueeze(-1))
    return Bt_full


def _phase2(layer, loc, full, tails_prev, rep, h, c0, c1, half, status=None):
    """Scoring and gate of the chunk [c0, c1) from the gathered full-sequence features, the earlier ranks' bucket
    tails and the chunk's n-gram memory rep = (vistos, hawkes, racha)."""
    B, L = full['sig'].shape
    T = layer.n_tablas
    dev = h.device
    lib = _lib.lib()
    s = _lib.stream_ptr(dev)
    orden_v, ids_v, row_len = shard_rows(layer, loc['orden'], loc['ids'], tails_prev, c0, L, status)
    Lv = orden_v.shape[1]
    Lc = c1 - c0
    d = layer.d
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _lib.make_config(layer, B, Lv, half)
    acc = torch.zeros(B, Lc, d, dtype=torch.bfloat16 if half else torch.float32, device=dev)
    hay = torch.empty(B, Lc, T, dtype=torch.uint8, device=dev)
    mx = torch.empty(B, Lc, T, dtype=torch.float32, device=dev)
    pk = torch.empty(B, Lc, T, dtype=torch.float32, device=dev)
    _lib.check(lib.asrn_score_shard(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), L, c0, c1, _lib.ptr(orden_v),
                                    _lib.ptr(ids_v), _lib.ptr(full['phi']), _lib.ptr(full['Qc']),
                                    _lib.ptr(full['Kc']), _lib.ptr(full['sig']), _lib.ptr(full['Bt']),
                                    _lib.ptr(full['log_alfa']), _lib.ptr(full['Ea']), _lib.ptr(row_len),
                                    _lib.ptr(acc), _lib.ptr(hay), _lib.ptr(mx), _lib.ptr(pk), s), 'asrn_score_shard')
    vistos, hawkes, racha = rep
    return stages.gate(layer, h, loc['glogit'], acc, hay, mx, pk, vistos, hawkes, racha, half=half)


# ---- n-gram memory of a chunk, carried across the shards ------------------------------------------------------------

def ngram_sort(layer, full, c0, Lc, half):
    """Sort and local scans of the chunk's n-gram keys (asrn_ngram_chunk_sort): the published part (sorted keys and
    per-group summaries, each (B * n, Lc)) and the workspace the finish step continues from."""
    B, L = full['sig'].shape
    n = layer.vistos
    dev = full['sig'].device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _lib.make_config(layer, B, Lc, half)
    lib = _lib.lib()
    ws = torch.empty(max(1, lib.asrn_ngram_chunk_workspace_bytes(ctypes_ref(cfg))), dtype=torch.uint8, device=dev)
    keys = torch.empty(B * n, Lc, dtype=torch.int64, device=dev)
    summ = torch.empty(B * n, Lc, 32, dtype=torch.uint8, device=dev)
    _lib.check(lib.asrn_ngram_chunk_sort(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), L, c0, _lib.ptr(full['sig']),
                                         _lib.ptr(full['Bt']), _lib.ptr(full['log_alfa']), _lib.ptr(keys),
                                         _lib.ptr(summ), _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev)),
               'asrn_ngram_chunk_sort')
    return dict(keys=keys, summ=summ, ws=ws)


def ngram_finish(layer, full, ng, keys_prev, summ_prev, c0, Lc, half):
    """vistos (B, Lc, n) and hawkes (B, Lc, n) of the chunk from its sort state and the earlier shards' published
    keys / summaries ((n_prev, B * n, Lc), rank order; None for the first shard)."""
    B, L = full['sig'].shape
    n = layer.vistos
    dev = full['sig'].device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _lib.make_config(layer, B, Lc, half)
    vistos = torch.empty(B, Lc, n, dtype=torch.uint8, device=dev)
    hawkes = torch.empty(B, Lc, n, dtype=torch.float32, device=dev)
    n_prev = 0 if keys_prev is None else keys_prev.shape[0]
    _lib.check(_lib.lib().asrn_ngram_chunk_finish(
        ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), L, c0, n_prev, None if n_prev == 0 else _lib.ptr(keys_prev),
        None if n_prev == 0 else _lib.ptr(summ_prev), _lib.ptr(ng['keys']), _lib.ptr(full['Bt']),
        _lib.ptr(full['log_alfa']), _lib.ptr(vistos), _lib.ptr(hawkes), _lib.ptr(ng['ws']), ng['ws'].numel(),
        _lib.stream_ptr(dev)), 'asrn_ngram_chunk_finish')
    return vistos, hawkes


def racha_chunk(layer, vistos, beta, racha_in, half, want_racha=True):
    """Streak of a chunk from the value before it (racha_in (B,), None = 0): (racha (B, Lc) or None, map (B, 2))."""
    B, Lc, _ = vistos.shape
    dev = vistos.device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _lib.make_config(layer, B, Lc, half)
    racha = torch.empty(B, Lc, dtype=torch.float32, device=dev) if want_racha else None
    rmap = torch.empty(B, 2, dtype=torch.float32, device=dev)
    lib = _lib.lib()
    ws = torch.empty(max(1, lib.asrn_racha_workspace_bytes(ctypes_ref(cfg))), dtype=torch.uint8, device=dev)
    _lib.check(lib.asrn_racha_chunk(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), _lib.ptr(vistos),
                                    _lib.ptr(beta), _lib.ptr(racha_in), _lib.ptr(racha), _lib.ptr(rmap),
                                    _lib.ptr(ws), ws.numel(), _lib.stream_ptr(dev)), 'asrn_racha_chunk')
    return racha, rmap


def racha_before(maps, rank):
    """maps (world, B, 2) of every chunk -> (B,) streak value before chunk `rank` (0 for the first)."""
    S = torch.zeros(maps.shape[1], dtype=torch.float32, device=maps.device)
    for q in range(rank):
        S = maps[q, :, 0] * S + maps[q, :, 1]
    return S


def _check(layer, E, h, tokens):
    if not (E.is_cuda and h.is_cuda):
        raise RuntimeError('asrn_b200 runs on CUDA tensors only')
    if E.shape != h.shape or E.dim() != 3 or E.shape[-1] != layer.d:
        raise ValueError(f'E and h must be (B, L, {layer.d}); got {tuple(E.shape)} and {tuple(h.shape)}')
    if tokens is not None and tokens.shape != E.shape[:2]:
        raise ValueError(f'piezas must be {tuple(E.shape[:2])}; got {tuple(tokens.shape)}')


@torch.no_grad()
def forward_emulated(layer, E, h, tokens, world):
    """Every rank's phases of the sharded forward in one process (the exchange becomes concatenation). E, h (B, L, d)
    and tokens (B, L) of the whole sequences; returns h' (B, L, d) fp32."""
    _check(layer, E, h, tokens)
    half = compute_half('cuda')
    B, L, d = E.shape
    E, h = E.float(), h.float()
    bounds = [chunk_bounds(L, world, r) for r in range(world)]
    locs = []
    for r, (c0, c1) in enumerate(bounds):
        halo = E[:, c0 - 1] if c0 > 0 else torch.zeros(B, d, device=E.device)
        locs.append(_phase1(layer, E[:, c0:c1].contiguous(), h[:, c0:c1].contiguous(),
                            None if tokens is None else tokens[:, c0:c1].contiguous(), halo, half, c0))
    full = {k: torch.cat([lc[k] for lc in locs], 1) for k in _SCALAR_KEYS}
    packed = [compact_tails(lc['tails']) for lc in locs]          # the exchanged form of the tails
    m = max(1, max(ix.numel() for _, ix in packed))
    ent_all = torch.zeros(world, m, packed[0][0].shape[1], dtype=torch.uint8, device=E.device)
    idx_all = torch.full((world, m), -1, dtype=torch.int64, device=E.device)
    for q, (ent, ix) in enumerate(packed):
        ent_all[q, :ix.numel()] = ent
        idx_all[q, :ix.numel()] = ix
    tails = expand_tails(ent_all, idx_all, locs[0]['tails'].shape)
    sums = torch.stack([lc['Bt'][:, -1] for lc in locs], 0)
    _apply_clock_offsets(full['Bt'], sums, L // world)
    Lc = L // world
    # the compact row exchange: each chunk publishes the rows of its tail positions; rank r sees the earlier ranks'
    T = layer.n_tablas
    pubs = []
    for r, (c0, c1) in enumerate(bounds):
        nxt = locs[r + 1]['Ea'][:, :1] if r + 1 < world else torch.zeros_like(locs[r]['Ea'][:, :1])
        Ea_next = torch.cat([locs[r]['Ea'][:, 1:], nxt], 1)
        sel = tail_index(locs[r]['tails'], c0, Lc, B, T)
        gidx = (sel // Lc) * L + c0 + sel % Lc
        pubs.append((_row_payload(locs[r], sel, Ea_next), gidx, _row_widths(locs[r], Ea_next)))
    ngs = [ngram_sort(layer, full, c0, Lc, half) for c0, _ in bounds]
    keys = torch.stack([g['keys'] for g in ngs], 0)
    summ = torch.stack([g['summ'] for g in ngs], 0)
    vh = [ngram_finish(layer, full, ngs[r], keys[:r] if r > 0 else None, summ[:r] if r > 0 else None, c0, Lc, half)
          for r, (c0, _) in enumerate(bounds)]
    maps = torch.stack([racha_chunk(layer, v, lc['beta'], None, half, want_racha=False)[1]
                        for (v, _), lc in zip(vh, locs)], 0)
    outs = []
    for r, (lc, (c0, c1)) in enumerate(zip(locs, bounds)):
        vistos, hawkes = vh[r]
        racha, _ = racha_chunk(layer, vistos, lc['beta'], racha_before(maps, r), half)
        fr = dict(full)
        fr.update(_full_rows(lc, B, L, c0, c1, locs[r + 1]['Ea'][:, 0] if r + 1 < world else None))
        for q in range(r):
            _scatter_rows(fr, pubs[q][0], pubs[q][1], pubs[q][2], L)
        outs.append(_phase2(layer, lc, fr, tails[:r] if r > 0 else None, (vistos, hawkes, racha),
                            h[:, c0:c1].contiguous(), c0, c1, half))
    return torch.cat(outs, 1)


def _gather_seq(x, world, group):
    """All-gather of a per-chunk tensor (B, Lc, ...) into (B, world * Lc, ...) (rank order = position order)."""
    import torch.distributed as dist
    x = x.contiguous()
    dt = x.dtype
    xb = x.view(-1).view(torch.uint8)       # as bytes: int16 bucket ids have no NCCL / gloo type
    if x.shape[0] == 1:                     # chunks are contiguous in position: one flat gather, no copy
        out = torch.empty(world * xb.numel(), dtype=torch.uint8, device=x.device)
        dist.all_gather_into_tensor(out, xb, group=group)
        return out.view(dt).view((1, world * x.shape[1]) + tuple(x.shape[2:]))
    parts = [torch.empty_like(xb) for _ in range(world)]
    dist.all_gather(parts, xb, group=group)
    return torch.cat([p.view(dt).view(x.shape) for p in parts], 1)


def exchange_first_rows(first, world, group=None):
    """(B, d) bf16 E of this chunk's first position -> (world, B, d): every chunk's, in rank order."""
    import torch.distributed as dist
    x = first.contiguous()
    flat = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(flat.view(-1).view(torch.uint8), x.view(-1).view(torch.uint8), group=group)
    return flat


def exchange_counts(local, world, group=None):
    """(k,) int64 device counts of this rank -> (world, k) list of lists on the host: the forward's one host
    synchronisation (the padded sizes of the variable-length exchange must be known to allocate)."""
    import torch.distributed as dist
    counts = torch.empty(world, local.numel(), dtype=torch.int64, device=local.device)
    dist.all_gather_into_tensor(counts.view(-1), local.contiguous(), group=group)
    return counts.tolist()


def exchange_varlen_async(items, world, group=None, counts=None, async_op=True):
    """Variable-length exchange of several items, each this rank's (n, bytes) uint8 payload and (n,) int64 indices:
    returns per item (payloads (world, m, bytes), indices (world, m)) padded to the largest n of any rank (index -1
    marks padding), and finish(), which makes the current stream wait for the collectives. The counts of all items go
    in one small all-gather that the host reads (the padded sizes must be known to allocate); the rest is issued
    without waiting."""
    import torch.distributed as dist
    dev = items[0][0].device
    if counts is None:
        counts = exchange_counts(torch.tensor([p.shape[0] for p, _ in items], dtype=torch.int64, device=dev), world,
                                 group)
    ms = [max(1, max(c[j] for c in counts)) for j in range(len(items))]
    out, works = [], []
    for (payload, gidx), m in zip(items, ms):
        pad = torch.zeros(m, payload.shape[1], dtype=torch.uint8, device=dev)
        pad[:payload.shape[0]] = payload
        idx = torch.full((m,), -1, dtype=torch.int64, device=dev)
        idx[:gidx.shape[0]] = gidx
        pay_all = torch.empty(world, m, payload.shape[1], dtype=torch.uint8, device=dev)
        idx_all = torch.empty(world, m, dtype=torch.int64, device=dev)
        works.append(dist.all_gather_into_tensor(pay_all.view(-1), pad.view(-1), group=group, async_op=async_op))
        works.append(dist.all_gather_into_tensor(idx_all.view(-1), idx, group=group, async_op=async_op))
        out.append((pay_all, idx_all))

    def finish():
        for w in works:
            if w is not None:
                w.wait()
    return out, finish


def exchange_rows_async(payload, gidx, world, group=None):
    """exchange_varlen_async of one item: (payloads (world, m, bytes), indices (world, m), finish)."""
    parts, finish = exchange_varlen_async([(payload, gidx)], world, group)
    pay_all, idx_all = parts[0]
    return pay_all, idx_all, finish


def exchange_halo(last, world, rank, group=None):
    """(B, d) E of this chunk's last position -> E of the position before this chunk (zeros on rank 0)."""
    import torch.distributed as dist
    x = last.contiguous()
    lasts = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(lasts.view(-1), x.view(-1), group=group)
    return lasts[rank - 1] if rank > 0 else torch.zeros_like(last)


def exchange_chunk_sums(chunk_sum, world, group=None):
    """(B,) fp64 sum of this chunk's beta -> (world, B): every chunk's sum, in rank order."""
    import torch.distributed as dist
    flat = torch.empty(world * chunk_sum.numel(), dtype=chunk_sum.dtype, device=chunk_sum.device)
    dist.all_gather_into_tensor(flat, chunk_sum.contiguous().view(-1), group=group)
    return flat.view((world,) + tuple(chunk_sum.shape))


def exchange_tails(tails, world, group=None):
    """(rows, 2^nb, C + 1) int32 bucket tails of this chunk -> (world, rows, 2^nb, C + 1), in rank order."""
    import torch.distributed as dist
    flat = torch.empty((world,) + tuple(tails.shape), dtype=tails.dtype, device=tails.device)
    dist.all_gather_into_tensor(flat.view(-1), tails.contiguous().view(-1), group=group)
    return flat


def exchange_ngram(keys, summ, world, group=None):
    """This chunk's sorted n-gram keys (B * n, Lc) int64 and summaries (B * n, Lc, 32) uint8 -> both with a leading
    rank dimension (world, ...), in rank order."""
    import torch.distributed as dist
    out = []
    for x in (keys, summ):
        flat = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(flat.view(-1), x.contiguous().view(-1), group=group)
        out.append(flat)
    return out[0], out[1]


def exchange_racha_maps(rmap, world, group=None):
    """(B, 2) streak map of this chunk -> (world, B, 2)."""
    import torch.distributed as dist
    flat = torch.empty((world,) + tuple(rmap.shape), dtype=rmap.dtype, device=rmap.device)
    dist.all_gather_into_tensor(flat.view(-1), rmap.contiguous().view(-1), group=group)
    return flat


@torch.no_grad()
def forward(layer, E, h, tokens=None, group=None):
    """One rank of the sharded forward under torch.distributed: E, h (B, Lc, d), tokens (B, Lc) are this rank's chunk
    of every sequence (chunks in rank order); returns h' (B, Lc, d) fp32 for the chunk. Every rank calls it with the
    same shapes; the collectives are the same on every rank, in the same order. Eager, with one host synchronisation
    (the sizes of the variable-length exchange); ShardedForward replays it as a CUDA graph instead."""
    import torch.distributed as dist
    _check(layer, E, h, tokens)
    _raise_reported(E.device, block=False)
    if dist.get_world_size(group) == 1:
        return layer(E.float().contiguous(), h.float().contiguous(), tokens)
    out, status, _ = _forward(layer, E, h, tokens, group, None)
    _defer_status(status)
    return out


def _forward(layer, E, h, tokens, group, caps, bufs=None):
    """The sharded forward. caps None: the exchange is sized from the counts read by the host (one synchronisation);
    caps = (tails, rows): fixed capacities, no host synchronisation (a count above its capacity is recorded in the
    status word). Returns (h' of the chunk, device status word, device (tails, rows) counts of this rank)."""
    import torch.distributed as dist
    if caps is not None:
        return _forward_packed(layer, E, h, tokens, group, caps, bufs)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    half = compute_half('cuda')
    B, Lc, d = E.shape
    L = world * Lc
    c0, c1 = rank * Lc, (rank + 1) * Lc
    E, h = E.float().contiguous(), h.float().contiguous()
    # (1) halo rows: E of every chunk's last position
    halo = exchange_halo(E[:, -1], world, rank, group)
    loc = _phase1(layer, E, h, tokens, halo, half, c0)
    # (2) chunk sums of beta (= the last local clock value) -> clock offsets
    sums = exchange_chunk_sums(loc['Bt'][:, -1], world, group)
    # (3) the per-position scalars of every position, the first value row of every chunk
    full = {k: _gather_seq(loc[k], world, group) for k in _SCALAR_KEYS}
    firsts = exchange_first_rows(loc['Ea'][:, 0], world, group)
    _apply_clock_offsets(full['Bt'], sums, Lc)
    # what this rank publishes: the positions in its tails and its non-empty tails (device-side counts)
    flags = tail_flags(loc['tails'], c0, Lc, B, layer.n_tablas)
    t_ne = loc['tails'][..., 0].reshape(-1) != 0
    local_counts = torch.stack([t_ne.sum(), flags.sum()])
    # (4) n-gram memory: the chunk's sort and per-group summaries (queued before the exchange of (5))
    ng = ngram_sort(layer, full, c0, Lc, half)
    nxt = firsts[rank + 1].unsqueeze(1) if rank + 1 < world else torch.zeros_like(loc['Ea'][:, :1])
    Ea_next = torch.cat([loc['Ea'][:, 1:], nxt], 1)
    widths = _row_widths(loc, Ea_next)
    # (5) the non-empty tails and the feature / value rows of the tail positions, padded to the largest rank's count
    if caps is None:
        counts = exchange_counts(local_counts, world, group)
        n_tails, n_rows = counts[rank]
        sel = compact(flags, n_rows)
        t_ent, t_idx = compact_tails(loc['tails'], n_tails)
        over = None
    else:
        n_tails, n_rows = caps
        counts = [list(caps)] * world
        sel = compact_cap(flags, n_rows)
        flat = loc['tails'].reshape(-1, loc['tails'].shape[-1])
        t_idx = compact_cap(t_ne, n_tails)
        t_ent = flat[t_idx.clamp(min=0)].contiguous().view(torch.uint8)
        over = (local_counts[0] > n_tails) | (local_counts[1] > n_rows)
    payload = _row_payload(loc, sel.clamp(min=0), Ea_next)
    gidx = torch.where(sel >= 0, (sel // Lc) * L + c0 + sel % Lc, -1)
    ((ent_all, tidx_all), (pay_all, gidx_all)), finish = exchange_varlen_async(
        [(t_ent, t_idx), (payload, gidx)], world, group, counts, async_op=caps is None)
    last_exchange.update(rows_padded=int(pay_all.shape[1]), rows_chunk=B * Lc, row_bytes=int(payload.shape[1]),
                         tails_padded=int(tidx_all.shape[1]), tails_dense=int(t_ne.numel()), counts=local_counts)
    full.update(_full_rows(loc, B, L, c0, c1, firsts[rank + 1] if rank + 1 < world else None))
    finish()
    for q in range(rank):
        _scatter_rows(full, pay_all[q], gidx_all[q], widths, L)
    tails = expand_tails(ent_all[:rank], tidx_all[:rank], loc['tails'].shape) if rank > 0 else None
    keys, summ = exchange_ngram(ng['keys'], ng['summ'], world, group)
    vistos, hawkes = ngram_finish(layer, full, ng, keys[:rank] if rank > 0 else None,
                                  summ[:rank] if rank > 0 else None, c0, Lc, half)
    _, rmap = racha_chunk(layer, vistos, loc['beta'], None, half, want_racha=False)
    maps = exchange_racha_maps(rmap, world, group)
    racha, _ = racha_chunk(layer, vistos, loc['beta'], racha_before(maps, rank), half)
    bad = carry_violations(sums=sums, maps=maps, keys=keys).clamp(max=1)
    if over is not None:
        bad = torch.maximum(bad, over.to(bad.dtype))
    status = bad.to(torch.int32).mul(_lib.ASRN_ERR_DATA).view(1)
    out = _phase2(layer, loc, full, tails, (vistos, hawkes, racha), h, c0, c1, half, status)
    return out, status, local_counts


def _pack(parts, cache=None):
    """Tensors -> one uint8 buffer (each part at an 8-byte aligned offset, the padding zero) and the (dtype, shape,
    offset) of each part: one copy per part into the buffer, which `cache` (a dict) keeps for the next call."""
    meta, off = [], 0
    for t in parts:
        meta.append((t.dtype, tuple(t.shape), off))
        off += (t.numel() * t.element_size() + 7) // 8 * 8
    dev = parts[0].device
    buf = None if cache is None else cache.get('_pack')
    if buf is None or buf.numel() != off or buf.device != dev:
        buf = torch.zeros(off, dtype=torch.uint8, device=dev)
        if cache is not None:
            cache['_pack'] = buf
    for t, (dt, shape, o) in zip(parts, meta):
        buf[o:o + t.numel() * t.element_size()].view(dt).view(shape).copy_(t)
    return buf, meta


def _unpack(buf, meta, i):
    """Part i of a packed buffer (world, bytes) -> (world,) + its shape, a strided view (no copy)."""
    dt, shape, off = meta[i]
    n = 1
    for x in shape:
        n *= x
    nb = n * torch.empty(0, dtype=dt).element_size()
    return buf[:, off:off + nb].view(dt).view((buf.shape[0],) + shape)


def _all_gather_bytes(buf, world, group, cache=None):
    import torch.distributed as dist
    out = None if cache is None else cache.get('_gathered')
    if out is None or tuple(out.shape) != (world, buf.numel()):
        out = torch.empty(world, buf.numel(), dtype=torch.uint8, device=buf.device)
        if cache is not None:
            cache['_gathered'] = out
    dist.all_gather_into_tensor(out.view(-1), buf, group=group)
    return out


def _forward_packed(layer, E, h, tokens, group, caps, bufs=None):
    """The sharded forward with fixed exchange capacities caps = (tails, rows) and no host synchronisation, its
    exchanges packed into four all-gathers: (1) the halo row; (2) in one buffer, the chunk sums of beta, the
    per-position signature, clock and log_alfa, the chunk's first bf16 E row, its non-empty bucket tails and the
    feature / value rows of its tail positions (the value row of a chunk's last position is taken from the next
    chunk's first row on arrival); (3) the n-gram keys and summaries; (4) the streak maps. The full-length feature buffers must hold numbers
    in every row (a masked key's value row still enters the value product with weight 0): they come from `bufs` (a
    dict kept by the caller, zero-filled on first use and reused, so a captured step does no memset; a reused row
    holds the finite values of an earlier step) or are zero-filled here. A count above its capacity is recorded in
    the status word."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    half = compute_half('cuda')
    B, Lc, d = E.shape
    L = world * Lc
    c0, c1 = rank * Lc, (rank + 1) * Lc
    T, nb = layer.n_tablas, layer.n_bits
    cap_t, cap_r = caps
    E, h = E.float().contiguous(), h.float().contiguous()
    halo = exchange_halo(E[:, -1], world, rank, group)
    loc = _phase1(layer, E, h, tokens, halo, half, c0, None if bufs is None else bufs.get('_E_ext'))
    # what this chunk publishes: its non-empty tails (compacted), the positions in them, their rows
    tails = loc['tails']
    C1 = tails.shape[-1]
    flat = tails.reshape(-1, C1)
    t_ne = flat[:, 0] != 0
    t_idx = compact_cap(t_ne, cap_t)
    t_rows = flat[t_idx.clamp(min=0)]
    cnt = t_rows[:, 0].long().clamp(0, C1 - 1)
    used = (torch.arange(C1 - 1, device=E.device) < cnt.unsqueeze(1)) & (t_idx >= 0).unsqueeze(1)
    b_of = (t_idx.clamp(min=0) // (1 << nb)) // T
    rel = torch.where(used, t_rows[:, 1:].long() - c0, Lc).clamp(0, Lc)
    flags = torch.zeros(B * (Lc + 1), dtype=torch.bool, device=E.device)
    flags.index_fill_(0, (b_of.unsqueeze(1) * (Lc + 1) + rel).view(-1), True)
    flags = flags.view(B, Lc + 1)[:, :Lc].reshape(-1)
    sel = compact_cap(flags, cap_r)
    widths = _row_widths(loc, loc['Ea'])
    payload = _row_payload_next(loc, sel.clamp(min=0), Lc)      # a sequence's last row: fixed on arrival
    gidx = torch.where(sel >= 0, (sel // Lc) * L + c0 + sel % Lc, -1)
    local_counts = torch.stack([t_ne.sum(), flags.sum()])
    over = (local_counts[0] > cap_t) | (local_counts[1] > cap_r)
    # (beta is not sent: the sequence-wide steps read sig, the clock and log_alfa only)
    buf, meta = _pack([loc['Bt'][:, -1], loc['Bt'], loc['sig'], loc['log_alfa'], loc['Ea'][:, 0],
                       t_rows, t_idx, payload, gidx], bufs)
    got = _all_gather_bytes(buf, world, group, bufs)
    sums = _unpack(got, meta, 0)                                          # (world, B)
    full = {}
    for i, k in ((1, 'Bt'), (2, 'sig'), (3, 'log_alfa')):
        full[k] = _unpack(got, meta, i).permute(1, 0, 2).reshape(B, L)    # (world, B, Lc) -> (B, L)
    _apply_clock_offsets(full['Bt'], sums, Lc)
    firsts = _unpack(got, meta, 4)                                        # (world, B, d)
    ng = ngram_sort(layer, full, c0, Lc, half)
    # the feature rows: this chunk's own, the earlier chunks' tail positions, every chunk start's value row
    for k in _ROW_KEYS + ('Ea',):
        x = loc[k]
        shape = (B * L + 1,) + tuple(x.shape[2:])
        t = None if bufs is None else bufs.get(k)
        if t is None or tuple(t.shape) != shape or t.dtype != x.dtype:
            t = torch.zeros(shape, dtype=x.dtype, device=x.device)
            if bufs is not None:
                bufs[k] = t
        t[:B * L].view((B, L) + tuple(x.shape[2:]))[:, c0:c1] = x
        full[k] = t
    pay_all, gidx_all = _unpack(got, meta, 7), _unpack(got, meta, 8)
    if rank > 0:                                   # the earlier ranks' rows in one scatter
        _scatter_rows(full, pay_all[:rank].reshape(-1, pay_all.shape[-1]), gidx_all[:rank].reshape(-1), widths, L)
    ea = full['Ea'][:B * L].view(B, L, -1)
    q_hi = min(rank + 2, world)                    # chunk starts 1 .. q_hi - 1 (up to c1), in one indexed write
    if q_hi > 1:
        starts = torch.arange(1, q_hi, device=ea.device) * Lc
        ea[:, starts] = firsts[1:q_hi].transpose(0, 1).to(ea.dtype)
    tails_prev = None
    if rank > 0:
        ent = _unpack(got, meta, 5)[:rank].contiguous().view(torch.uint8).view(rank, cap_t, -1)
        tails_prev = expand_tails(ent, _unpack(got, meta, 6)[:rank], tails.shape)
    keys, summ = exchange_ngram(ng['keys'], ng['summ'], world, group)
    vistos, hawkes = ngram_finish(layer, full, ng, keys[:rank] if rank > 0 else None,
                                  summ[:rank] if rank > 0 else None, c0, Lc, half)
    _, rmap = racha_chunk(layer, vistos, loc['beta'], None, half, want_racha=False)
    maps = exchange_racha_maps(rmap, world, group)
    racha, _ = racha_chunk(layer, vistos, loc['beta'], racha_before(maps, rank), half)
    bad = torch.maximum(carry_violations(sums=sums, maps=maps, keys=keys).clamp(max=1), over.to(torch.int64))
    status = bad.to(torch.int32).mul(_lib.ASRN_ERR_DATA).view(1)
    out = _phase2(layer, loc, full, tails_prev, (vistos, hawkes, racha), h, c0, c1, half, status)
    last_exchange.update(rows_padded=cap_r, rows_chunk=B * Lc, row_bytes=int(payload.shape[1]), tails_padded=cap_t,
                         tails_dense=int(t_ne.numel()), counts=local_counts, packed_bytes=int(buf.numel()))
    return out, status, local_counts


class ShardedForward:
    """The sharded forward of one rank for fixed shapes, replayed as one CUDA graph (NCCL collectives included): no
    host synchronisation and no per-op launch cost inside a step. The first (eager) pass measures how many tail rows
    and tails each rank publishes; the exchange is then sized to the largest count of any rank times `margin` (plus
    `extra`), and a later input whose counts exceed that is reported like inconsistent state (ShardExchangeError at
    the next call or check_exchange): build a new ShardedForward for it. Every rank builds and calls it in the same
    order; call close() (or drop it) before destroying the process group."""

    def __init__(self, layer, E, h, tokens=None, group=None, margin=1.5, extra=64):
        import torch.distributed as dist
        _check(layer, E, h, tokens)
        self.layer, self.group = layer, group
        self.device = E.device
        B, Lc, d = E.shape
        # the input buffers of the graph: E lives in rows 1 .. Lc of a (B, Lc + 1, d) buffer whose row 0 receives the
        # previous chunk's last row (so the hash reads the extended rows in place); for one sequence E is contiguous
        self.E_ext = torch.empty(B, Lc + 1, d, dtype=torch.float32, device=E.device)
        self.E = self.E_ext[:, 1:]
        self.E.copy_(E)
        self.h = h.float().contiguous().clone()
        self.tokens = None if tokens is None else tokens.contiguous().clone()
        world = dist.get_world_size(group)
        with torch.no_grad():
            _, _, cnt = _forward(layer, self.E, self.h, self.tokens, group, None)
            counts = exchange_counts(cnt, world, group)
        self.caps = tuple(int(max(c[j] for c in counts) * margin) + extra for j in range(2))
        self.bufs = {'_E_ext': self.E_ext}                      # full-length feature rows, zeroed once, reused
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side), torch.no_grad():           # warm the capacity path (allocations, kernels)
            _forward(layer, self.E, self.h, self.tokens, group, self.caps, self.bufs)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.out, self.status, _ = _forward(layer, self.E, self.h, self.tokens, group, self.caps, self.bufs)

    def __call__(self, E=None, h=None, tokens=None):
        """h' of this rank's chunk for new inputs of the captured shapes (the returned tensor is overwritten by the
        next call). The inputs are copied into the graph's input buffers (self.E, self.h, self.tokens); a caller that
        writes its inputs there itself passes nothing (or those buffers) and no copy is made."""
        _raise_reported(self.device, block=False)
        for dst, src in ((self.E, E), (self.h, h), (self.tokens, tokens)):
            if dst is not None and src is not None and src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        self.graph.replay()
        _defer_status(self.status)
        return self.out

    def close(self):
        self.graph = None
        self.out = self.status = None
        self.bufs = {}
