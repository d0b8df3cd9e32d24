// Sequence-chunk sharding (one long sequence over several GPUs): the sorted rows of one shard.
// After the exchange every shard holds the whole sequence's bucket ids and features, sorts the full rows (one per
// (sequence, table)) and keeps only what its own queries need: the slots of its positions [q_lo, q_hi), and before
// each bucket's run of local slots the up to C slots of earlier shards that some local query has as a candidate (the
// "exclusive ring" of the bucket: the C most recent earlier positions). Within a bucket positions ascend, so a query's
// candidates -- its <= C nearest same-bucket predecessors (asrn/estable.py:232-236, 262-265) -- are the same in the
// shard's row as in the full row. Rows are compacted in order and padded to a common length Lv with a slot whose id
// matches no bucket (0xFFFF) at a position that is neither a query nor a candidate (pad_pos).
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {
constexpr int kShardThreads = 1024, kShardItems = 4;

__device__ __forceinline__ bool shard_keep(const int32_t* ord, const uint16_t* ids, int64_t L, int64_t s, int C,
                                           int64_t q_lo, int64_t q_hi) {
  const int64_t pos = ord[s];
  if (pos >= q_lo && pos < q_hi) return true;
  if (pos >= q_lo) return false;                 // a later shard's position: never a candidate of ours
  const uint16_t id = ids[s];
  for (int k = 1; k <= C && s + k < L; ++k) {
    if (ids[s + k] != id) return false;
    const int64_t p2 = ord[s + k];
    if (p2 >= q_lo) return p2 < q_hi;            // the bucket's first non-earlier slot: local or later
  }
  return false;
}
}  // namespace

// One block per row. With orden_v: compacts the kept slots into (orden_v, ids_v) of length Lv (a row keeping more
// than Lv slots is cut at Lv); with counts: writes the row's kept count (both may be given).
__global__ void __launch_bounds__(kShardThreads) k_shard_rows(int64_t L, int C, int64_t q_lo, int64_t q_hi,
                                                              const int32_t* __restrict__ orden,
                                                              const uint16_t* __restrict__ ids_o, int64_t Lv,
                                                              int32_t* __restrict__ orden_v,
                                                              uint16_t* __restrict__ ids_v, int64_t* counts,
                                                              int32_t pad_pos) {
  const int64_t row = blockIdx.x;
  const int32_t* ord = orden + row * L;
  const uint16_t* ids = ids_o + row * L;
  __shared__ int warp_tot[32];
  __shared__ int64_t carry_s;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int64_t base = 0; base < L; base += (int64_t)kShardThreads * kShardItems) {
    bool keep[kShardItems];
    int cnt = 0;
#pragma unroll
    for (int k = 0; k < kShardItems; ++k) {
      const int64_t s = base + (int64_t)tid * kShardItems + k;
      keep[k] = s < L && shard_keep(ord, ids, L, s, C, q_lo, q_hi);
      cnt += keep[k] ? 1 : 0;
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    if (wid == 0) {
      int w = lane < kShardThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    const int64_t carry = carry_s;
    int64_t at = carry + (wid > 0 ? warp_tot[wid - 1] : 0) + (incl - cnt);
    if (orden_v) {
#pragma unroll
      for (int k = 0; k < kShardItems; ++k) {
        if (!keep[k]) continue;
        const int64_t s = base + (int64_t)tid * kShardItems + k;
        if (at < Lv) {
          orden_v[row * Lv + at] = ord[s];
          ids_v[row * Lv + at] = ids[s];
        }
        ++at;
      }
    }
    __syncthreads();
    if (tid == 0) carry_s = carry + warp_tot[kShardThreads / 32 - 1];
    __syncthreads();
  }
  const int64_t n = carry_s;
  if (counts && tid == 0) counts[row] = n;
  if (!orden_v) return;
  for (int64_t i = n + tid; i < Lv; i += kShardThreads) {
    orden_v[row * Lv + i] = pad_pos;
    ids_v[row * Lv + i] = 0xFFFF;
  }
}

int launch_shard_rows(int64_t rows, int64_t L, int C, int64_t q_lo, int64_t q_hi, const int32_t* orden,
                      const uint16_t* ids_o, int64_t Lv, int32_t* orden_v, uint16_t* ids_v, int64_t* counts,
                      int32_t pad_pos, cudaStream_t s) {
  if (rows == 0) return ASRN_OK;
  k_shard_rows<<<(unsigned)rows, kShardThreads, 0, s>>>(L, C, q_lo, q_hi, orden, ids_o, Lv, orden_v, ids_v, counts,
                                                        pad_pos);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}


// ---- shard rows from local sorts and exchanged bucket tails ----------------------------------------------------------
// The same rows as k_shard_rows, without sorting the whole sequence on every shard. Each shard sorts its own chunk
// (asrn_bucket_sort on (rows, Lc)); per (row, bucket) it publishes the bucket's tail, its last <= C positions
// (asrn_shard_tails); the tails of every shard are all-gathered; a shard's row is then, for every bucket with local
// slots, the bucket's C most recent earlier-chunk positions (walking the earlier shards' tails from the nearest one
// back) followed by its local run (asrn_shard_merge). Within a bucket positions ascend across chunks in rank order,
// so this is the slot set and order of the full row restricted as k_shard_rows restricts it.
namespace {
constexpr int kBinT = 256;

// run_beg[row][bucket] = first local slot, run_end[row][bucket] = one past the last (both zero-initialised: empty)
__global__ void k_shard_runs(int64_t rows, int64_t Lc, int nbins, const uint16_t* __restrict__ ids_loc,
                             int32_t* __restrict__ run_beg, int32_t* __restrict__ run_end) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * Lc) return;
  const int64_t row = i / Lc, s = i % Lc;
  const uint16_t* ids = ids_loc + row * Lc;
  const int id = ids[s];
  if (s == 0 || ids[s - 1] != id) run_beg[row * nbins + id] = (int32_t)s;
  if (s == Lc - 1 || ids[s + 1] != id) run_end[row * nbins + id] = (int32_t)(s + 1);
}

// tails (rows, nbins, C + 1): [0] = count, [1 .. count] = the bucket's last count global positions, ascending
__global__ void k_shard_tails(int64_t rows, int nbins, int C, int64_t c0, const int32_t* __restrict__ orden_loc,
                              int64_t Lc, const int32_t* __restrict__ run_beg, const int32_t* __restrict__ run_end,
                              int32_t* __restrict__ tails) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nbins) return;
  const int64_t row = i / nbins;
  const int beg = run_beg[i], end = run_end[i];
  const int cnt = min(C, end - beg);
  int32_t* t = tails + i * (C + 1);
  t[0] = cnt;
  for (int j = 0; j < cnt; ++j) t[1 + j] = (int32_t)(c0 + orden_loc[row * Lc + end - cnt + j]);
}

// A tail received from shard p (chunk [p Lc, (p + 1) Lc)) is used only if it is consistent: count in [0, C] and its
// positions strictly ascending inside the sender's chunk. Anything else (a carry corrupted in transit, a faulty rank)
// would index features out of range later: such a tail is treated as empty and ASRN_ERR_DATA is recorded.
__device__ __forceinline__ bool tail_valid(const int32_t* t, int C, int64_t lo, int64_t hi) {
  const int cnt = t[0];
  if (cnt < 0 || cnt > C) return false;
  int64_t prev = lo - 1;
  for (int e = 1; e <= cnt; ++e) {
    const int64_t q = t[e];
    if (q <= prev || q >= hi) return false;
    prev = q;
  }
  return true;
}

// per (row, bucket): ring length (0 without local slots) and ring + local length
__global__ void k_shard_sizes(int64_t rows, int64_t Lc, int nbins, int C, int n_prev,
                              const int32_t* __restrict__ tails_prev, const int32_t* __restrict__ run_beg,
                              const int32_t* __restrict__ run_end, int32_t* __restrict__ ring,
                              int32_t* __restrict__ tot, int* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nbins) return;
  const int local = run_end[i] - run_beg[i];
  int r = 0;
  if (local > 0)
    for (int p = n_prev - 1; p >= 0 && r < C; --p) {
      const int32_t* t = tails_prev + ((int64_t)p * rows * nbins + i) * (C + 1);
      if (!tail_valid(t, C, p * Lc, (p + 1) * Lc)) {
        if (status) atomicCAS(status, ASRN_OK, ASRN_ERR_DATA);
        continue;
      }
      r += t[0];
    }
  r = min(r, C);
  ring[i] = r;
  tot[i] = r + local;
}

// per row: exclusive scan of tot over the buckets (in place) and the row's length
__global__ void __launch_bounds__(1024) k_shard_scan(int32_t* __restrict__ tot, int nbins, int64_t* row_len) {
  const int64_t row = blockIdx.x;
  const int per = (nbins + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int32_t* t = tot + row * nbins;
  int local = 0;
  for (int k = 0; k < per && b0 + k < nbins; ++k) local += t[b0 + k];
  __shared__ int wsum[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    int w = (lane < (int)(blockDim.x >> 5)) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;
  }
  __syncthreads();
  int run = (wid > 0 ? wsum[wid - 1] : 0) + incl - local;
  for (int k = 0; k < per && b0 + k < nbins; ++k) {
    const int c = t[b0 + k];
    t[b0 + k] = run;
    run += c;
  }
  if (threadIdx.x == blockDim.x - 1) row_len[row] = run;
}

__global__ void k_shard_pad(int64_t n, int32_t pad_pos, int32_t* __restrict__ orden_v, uint16_t* __restrict__ ids_v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  orden_v[i] = pad_pos;
  ids_v[i] = 0xFFFF;
}

// ring entries: the j-th most recent earlier position of the bucket goes to slot off + ring - 1 - j
__global__ void k_shard_write_ring(int64_t rows, int64_t Lc, int nbins, int C, int n_prev,
                                   const int32_t* __restrict__ tails_prev, const int32_t* __restrict__ ring,
                                   const int32_t* __restrict__ off, int64_t Lv, int32_t* __restrict__ orden_v,
                                   uint16_t* __restrict__ ids_v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nbins) return;
  const int r = ring[i];
  if (r == 0) return;
  const int64_t row = i / nbins;
  const int bucket = (int)(i % nbins);
  const int64_t base = row * Lv + off[i];
  int j = 0;
  for (int p = n_prev - 1; p >= 0 && j < r; --p) {
    const int32_t* t = tails_prev + ((int64_t)p * rows * nbins + i) * (C + 1);
    if (!tail_valid(t, C, p * Lc, (p + 1) * Lc)) continue;      // skipped by k_shard_sizes too
    for (int e = t[0]; e >= 1 && j < r; --e, ++j) {
      orden_v[base + r - 1 - j] = t[e];
      ids_v[base + r - 1 - j] = (uint16_t)bucket;
    }
  }
}

__global__ void k_shard_write_local(int64_t rows, int64_t Lc, int nbins, int64_t c0,
                                    const int32_t* __restrict__ orden_loc, const uint16_t* __restrict__ ids_loc,
                                    const int32_t* __restrict__ run_beg, const int32_t* __restrict__ ring,
                                    const int32_t* __restrict__ off, int64_t Lv, int32_t* __restrict__ orden_v,
                                    uint16_t* __restrict__ ids_v) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * Lc) return;
  const int64_t row = i / Lc, s = i % Lc;
  const int id = ids_loc[i];
  const int64_t k = row * nbins + id;
  const int64_t dst = row * Lv + off[k] + ring[k] + (s - run_beg[k]);
  orden_v[dst] = (int32_t)(c0 + orden_loc[i]);
  ids_v[dst] = (uint16_t)id;
}

inline unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }
}  // namespace

size_t shard_merge_workspace(int64_t rows, int nb) {
  return 4 * align_up((size_t)rows * ((size_t)1 << nb) * 4);
}

int launch_shard_tails(int64_t rows, int64_t Lc, int nb, int C, int64_t c0, const int32_t* orden_loc,
                       const uint16_t* ids_loc, int32_t* tails, void* ws, cudaStream_t s) {
  const int nbins = 1 << nb;
  const size_t part = align_up((size_t)rows * nbins * 4);
  int32_t* beg = reinterpret_cast<int32_t*>(ws);
  int32_t* end = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(ws) + part);
  if (cudaMemsetAsync(ws, 0, 2 * part, s) != cudaSuccess) return ASRN_ERR_CUDA;
  if (rows * Lc > 0) k_shard_runs<<<blocks_for(rows * Lc, kBinT), kBinT, 0, s>>>(rows, Lc, nbins, ids_loc, beg, end);
  k_shard_tails<<<blocks_for(rows * nbins, kBinT), kBinT, 0, s>>>(rows, nbins, C, c0, orden_loc, Lc, beg, end, tails);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_shard_merge(int64_t rows, int64_t Lc, int nb, int C, int64_t c0, int n_prev, const int32_t* tails_prev,
                       const int32_t* orden_loc, const uint16_t* ids_loc, int64_t Lv, int32_t* orden_v,
                       uint16_t* ids_v, int64_t* row_len, int32_t pad_pos, int* status, void* ws, cudaStream_t s) {
  const int nbins = 1 << nb;
  const size_t part = align_up((size_t)rows * nbins * 4);
  char* w = reinterpret_cast<char*>(ws);
  int32_t* beg = reinterpret_cast<int32_t*>(w);
  int32_t* end = reinterpret_cast<int32_t*>(w + part);
  int32_t* ring = reinterpret_cast<int32_t*>(w + 2 * part);
  int32_t* off = reinterpret_cast<int32_t*>(w + 3 * part);
  if (cudaMemsetAsync(ws, 0, 2 * part, s) != cudaSuccess) return ASRN_ERR_CUDA;
  const unsigned gb = blocks_for(rows * nbins, kBinT);
  if (rows * Lc > 0) k_shard_runs<<<blocks_for(rows * Lc, kBinT), kBinT, 0, s>>>(rows, Lc, nbins, ids_loc, beg, end);
  k_shard_sizes<<<gb, kBinT, 0, s>>>(rows, Lc, nbins, C, n_prev, tails_prev, beg, end, ring, off, status);
  k_shard_scan<<<(unsigned)rows, 1024, 0, s>>>(off, nbins, row_len);
  k_shard_pad<<<blocks_for(rows * Lv, kBinT), kBinT, 0, s>>>(rows * Lv, pad_pos, orden_v, ids_v);
  k_shard_write_ring<<<gb, kBinT, 0, s>>>(rows, Lc, nbins, C, n_prev, tails_prev, ring, off, Lv, orden_v, ids_v);
  if (rows * Lc > 0)
    k_shard_write_local<<<blocks_for(rows * Lc, kBinT), kBinT, 0, s>>>(rows, Lc, nbins, c0, orden_loc, ids_loc, beg,
                                                                       ring, off, Lv, orden_v, ids_v);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
