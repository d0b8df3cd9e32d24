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

// One block per row. counts != null: writes the row's kept count; else compacts into (orden_v, ids_v) of length Lv.
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
  if (!orden_v) {
    if (tid == 0) counts[row] = n;
    return;
  }
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

}  // namespace asrn
