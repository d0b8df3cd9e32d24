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


def tail_index(tails, c0, Lc, B, T):
    """Local flat indices b * Lc + (p - c0), ascending, of the positions p of this chunk that appear in its bucket
    tails (rows b * T + tau): the only positions of the chunk that a later shard's rows hold."""
    dev = tails.device
    rows, _, C1 = tails.shape
    C = C1 - 1
    cnt = tails[..., 0].long().clamp(0, C)
    valid = torch.arange(C, device=dev) < cnt.unsqueeze(-1)
    rel = torch.where(valid, tails[..., 1:].long() - c0, Lc).clamp(0, Lc)
    b = (torch.arange(rows, device=dev) // T).view(rows, 1, 1)
    flags = torch.zeros(B * (Lc + 1), dtype=torch.bool, device=dev)
    flags[(b * (Lc + 1) + rel).view(-1)] = True
    return flags.view(B, Lc + 1)[:, :Lc].reshape(-1).nonzero().squeeze(1)


def compact_tails(tails):
    """The non-empty bucket tails of a chunk: flat indices row * 2^nb + bucket (int64) and their (count, positions)
    entries as raw bytes (n, (C + 1) * 4). In the heavy regime few buckets are used, so this is far smaller than the
    dense (rows, 2^nb, C + 1) array the merge kernel reads."""
    flat = tails.reshape(-1, tails.shape[-1])
    nz = (flat[:, 0] != 0).nonzero().squeeze(1)
    return flat[nz].contiguous().view(torch.uint8), nz


def expand_tails(ent_all, idx_all, shape):
    """(world, m, bytes) entries and (world, m) indices (-1 = padding) -> dense (world,) + shape int32 tails, zeros
    (empty tails) elsewhere."""
    world = ent_all.shape[0]
    dense = torch.zeros((world,) + tuple(shape), dtype=torch.int32, device=ent_all.device)
    for q in range(world):
        keep = idx_all[q] >= 0
        rows = ent_all[q][keep].contiguous().view(torch.int32).view(-1, shape[-1])
        dense[q].view(-1, shape[-1]).index_copy_(0, idx_all[q][keep], rows)
    return dense


def _row_payload(loc, sel, Ea_next):
    """(n, row bytes) uint8: for each selected local position its phi, Qc and Kc rows and the bf16 E row of the
    next position (its value row), as raw bytes."""
    parts = []
    for k in _ROW_KEYS:
        x = loc[k]
        parts.append(x.reshape(-1, x.shape[-1])[sel].contiguous().view(torch.uint8))
    parts.append(Ea_next.reshape(-1, Ea_next.shape[-1])[sel].contiguous().view(torch.uint8))
    return torch.cat(parts, 1)


def _row_widths(loc, Ea_next):
    return [loc[k].shape[-1] * loc[k].element_size() for k in _ROW_KEYS] + \
        [Ea_next.shape[-1] * Ea_next.element_size()]


def _full_rows(loc, B, L, c0, c1, Ea_first_next):
    """Zero-filled (B, L, .) feature tensors holding this chunk's own rows and, at c1, the next chunk's first value
    row; the earlier chunks' rows are scattered in by _scatter_rows."""
    full = {}
    for k in _ROW_KEYS + ('Ea',):
        x = loc[k]
        t = torch.zeros((B, L) + tuple(x.shape[2:]), dtype=x.dtype, device=x.device)
        t[:, c0:c1] = x
        full[k] = t
    if Ea_first_next is not None and c1 < L:
        full['Ea'][:, c1] = Ea_first_next
    return full


def _scatter_rows(full, payload, gidx, widths, L):
    """Rows of another chunk (payload (n, bytes), global flat indices b * L + p, -1 = padding) into full: phi, Qc, Kc
    at p, the value row at p + 1 (where the scoring kernel reads the value of key p)."""
    keep = gidx >= 0
    gidx, payload = gidx[keep], payload[keep]
    off = 0
    for k, w in zip(_ROW_KEYS + ('Ea',), widths):
        t = full[k]
        rows = payload[:, off:off + w].contiguous().view(t.dtype).view(-1, t.shape[-1])
        dst = gidx + 1 if k == 'Ea' else gidx
        if k == 'Ea':                                   # the value row of the sequence's last position is unused
            ok = (dst % L) != 0
            dst, rows = dst[ok], rows[ok]
        t.view(-1, t.shape[-1]).index_copy_(0, dst, rows)
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
        flip = torch.bitwise_xor(k, torch.tensor(-(1 << 63), dtype=torch.int64, device=k.device))
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


def _phase1(layer, E, h, tokens, E_halo, half, c0):
    """Local stages of one chunk starting at position c0. E, h (B, Lc, d) fp32, tokens (B, Lc) or None, E_halo (B, d):
    E of the position before the chunk."""
    ctx = stages.context(layer, h, tokens, E=None if tokens is not None else E, half=half)
    Bt = stages.clock(ctx['beta'])
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


def exchange_varlen_async(items, world, group=None):
    """Variable-length exchange of several items, each this rank's (n, bytes) uint8 payload and (n,) int64 indices:
    returns per item (payloads (world, m, bytes), indices (world, m)) padded to the largest n of any rank (index -1
    marks padding), and finish(), which makes the current stream wait for the collectives. The counts of all items go
    in one small all-gather that the host reads (the padded sizes must be known to allocate); the rest is issued
    without waiting."""
    import torch.distributed as dist
    dev = items[0][0].device
    n = torch.tensor([p.shape[0] for p, _ in items], dtype=torch.int64, device=dev)
    counts = torch.empty(world, len(items), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(counts.view(-1), n, group=group)
    ms = [max(1, int(m)) for m in counts.max(0).values.tolist()]
    out, works = [], []
    for (payload, gidx), m in zip(items, ms):
        pad = torch.zeros(m, payload.shape[1], dtype=torch.uint8, device=dev)
        pad[:payload.shape[0]] = payload
        idx = torch.full((m,), -1, dtype=torch.int64, device=dev)
        idx[:gidx.shape[0]] = gidx
        pay_all = torch.empty(world, m, payload.shape[1], dtype=torch.uint8, device=dev)
        idx_all = torch.empty(world, m, dtype=torch.int64, device=dev)
        works.append(dist.all_gather_into_tensor(pay_all.view(-1), pad.view(-1), group=group, async_op=True))
        works.append(dist.all_gather_into_tensor(idx_all.view(-1), idx, group=group, async_op=True))
        out.append((pay_all, idx_all))

    def finish():
        for w in works:
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
    lasts = [torch.empty_like(last) for _ in range(world)]
    dist.all_gather(lasts, last.contiguous(), group=group)
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
    same shapes; the collectives are the same on every rank, in the same order."""
    import torch.distributed as dist
    _check(layer, E, h, tokens)
    _raise_reported(E.device, block=False)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    half = compute_half('cuda')
    B, Lc, d = E.shape
    L = world * Lc
    c0, c1 = rank * Lc, (rank + 1) * Lc
    E, h = E.float().contiguous(), h.float().contiguous()
    if world == 1:
        return layer(E, h, tokens)
    # (1) halo rows: E of every chunk's last position
    halo = exchange_halo(E[:, -1], world, rank, group)
    loc = _phase1(layer, E, h, tokens, halo, half, c0)
    # (2) chunk sums of beta (= the last local clock value) -> clock offsets
    sums = exchange_chunk_sums(loc['Bt'][:, -1], world, group)
    # (3) bucket tails, (4) the per-position scalars of every position, (5) the feature and value rows of the tail
    # positions only (gathered while the n-gram memory sorts its chunk)
    full = {k: _gather_seq(loc[k], world, group) for k in _SCALAR_KEYS}
    firsts = exchange_first_rows(loc['Ea'][:, 0], world, group)
    nxt = firsts[rank + 1].unsqueeze(1) if rank + 1 < world else torch.zeros_like(loc['Ea'][:, :1])
    Ea_next = torch.cat([loc['Ea'][:, 1:], nxt], 1)
    sel = tail_index(loc['tails'], c0, Lc, B, layer.n_tablas)
    payload = _row_payload(loc, sel, Ea_next)
    gidx = (sel // Lc) * L + c0 + sel % Lc
    widths = _row_widths(loc, Ea_next)
    t_ent, t_idx = compact_tails(loc['tails'])
    ((ent_all, tidx_all), (pay_all, gidx_all)), finish = exchange_varlen_async([(t_ent, t_idx), (payload, gidx)],
                                                                                world, group)
    last_exchange.update(rows_sent=int(payload.shape[0]), rows_padded=int(pay_all.shape[1]), rows_chunk=B * Lc,
                         row_bytes=int(payload.shape[1]), tails_sent=int(t_idx.shape[0]),
                         tails_padded=int(tidx_all.shape[1]), tails_dense=int(loc['tails'][..., 0].numel()))
    _apply_clock_offsets(full['Bt'], sums, Lc)
    # (6) n-gram memory: per-group summaries of every chunk, then the streak maps
    ng = ngram_sort(layer, full, c0, Lc, half)
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
    status = carry_violations(sums=sums, maps=maps, keys=keys).clamp(max=1).to(torch.int32).mul(
        _lib.ASRN_ERR_DATA).view(1)
    out = _phase2(layer, loc, full, tails, (vistos, hawkes, racha), h, c0, c1, half,
                  status)
    _defer_status(status)
    return out
