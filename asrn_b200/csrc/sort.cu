// Per-table stable bucket sort: for every row r = b * T + tau, the text positions ordered by bucket id, ties by
// position. Reference: ids.transpose(1, 2).reshape(B*T, L).argsort(dim=-1, stable=True) (asrn/estable.py:220-221).
//
// Design: a row is cut into tiles of at most kTile positions, one block per tile. The block sorts composite 32-bit
// keys (id << 13 | local position) in shared memory with an LSD radix sort on the id: one pass per digit of at most
// 8 bits (two passes for 14-bit ids). A pass is a stable counting sort: each warp owns a contiguous segment of the
// keys and walks it 32 keys at a time; __match_any_sync groups the lanes of equal digits, so the warp's count of a
// digit (a per-warp histogram in shared memory, no atomics) and each key's rank among the equal digits before it come
// from one ballot-like instruction; an exclusive scan over (digit, warp) gives every warp's first slot per digit, and
// the warps scatter in position order, which keeps the sort stable.
// A single-tile row is written out directly. Longer rows add a per-tile histogram of the 2^nb buckets, the global
// slot where each tile's run of a bucket starts (bucket totals over the tiles, a scan over the buckets, running
// offsets over the tiles), and a scatter of every tile's runs to their slots.
#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kTile = 8192;
constexpr int kPosBits = 13;
constexpr uint32_t kPosMask = (1u << kPosBits) - 1;
constexpr int kSortThreads = 1024;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kMaxDigitBits = 8;
constexpr int kMaxGridY = 65535;

// Shared memory of k_bsort_tile: two key buffers of kTile and the (warp, digit) table of 16-bit counts / offsets.
constexpr size_t kSortSmem = 2 * (size_t)kTile * 4 + (size_t)kSortWarps * (1 << kMaxDigitBits) * 2;

// One stable counting-sort pass of src[0, n_pad) into dst by the digit (key >> shift) & (2^bits - 1).
__device__ __forceinline__ void radix_pass(const uint32_t* src, uint32_t* dst, uint16_t* tab, int n_pad, int shift,
                                           int bits) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nd = 1 << bits;
  const uint32_t dmask = (uint32_t)nd - 1;
  const int seg = n_pad / kSortWarps;                 // a multiple of 32
  const uint32_t lt = (1u << lane) - 1;
  for (int i = threadIdx.x; i < kSortWarps * nd; i += kSortThreads) tab[i] = 0;
  __syncthreads();
  // counts: tab[d * 32 + w] = keys of warp w's segment with digit d
  for (int j = 0; j < seg; j += 32) {
    const uint32_t d = (src[w * seg + j + lane] >> shift) & dmask;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    if ((peers & lt) == 0) tab[d * kSortWarps + w] += (uint16_t)__popc(peers);
  }
  __syncthreads();
  // exclusive scan of tab in (digit, warp) order; every thread scans a run of `per` consecutive entries
  {
    __shared__ int wsum[kSortWarps];
    const int total = kSortWarps * nd;
    const int per = (total + kSortThreads - 1) / kSortThreads;
    const int e0 = threadIdx.x * per;
    int local = 0;
    for (int k = 0; k < per && e0 + k < total; ++k) local += tab[e0 + k];
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) wsum[w] = incl;
    __syncthreads();
    if (w == 0) {
      int v = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      wsum[lane] = v;
    }
    __syncthreads();
    int run = (w > 0 ? wsum[w - 1] : 0) + incl - local;
    for (int k = 0; k < per && e0 + k < total; ++k) {
      const int c = tab[e0 + k];
      tab[e0 + k] = (uint16_t)run;
      run += c;
    }
  }
  __syncthreads();
  // scatter in position order: key rank = the warp's next slot for its digit + equal digits on lower lanes
  for (int j = 0; j < seg; j += 32) {
    const uint32_t k = src[w * seg + j + lane];
    const uint32_t d = (k >> shift) & dmask;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const int base = tab[d * kSortWarps + w];
    dst[base + __popc(peers & lt)] = k;
    __syncwarp();
    if ((peers & lt) == 0) tab[d * kSortWarps + w] = (uint16_t)(base + __popc(peers));
    __syncwarp();
  }
  __syncthreads();
}

// first index in keys[0, n) whose key >= v (keys ascending)
__device__ __forceinline__ int lower_bound_u32(const uint32_t* keys, int n, uint32_t v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (keys[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(kSortThreads) k_bsort_tile(const uint16_t* __restrict__ ids_rows, int64_t L,
                                                             int ntiles, int n_pad, int nb,
                                                             int32_t* __restrict__ orden, uint16_t* __restrict__ ids_o,
                                                             uint32_t* __restrict__ tmp, int32_t* __restrict__ hist) {
  extern __shared__ __align__(16) uint32_t sm[];
  uint32_t* ka = sm;
  uint32_t* kb = sm + kTile;
  uint16_t* tab = reinterpret_cast<uint16_t*>(sm + 2 * kTile);
  const int tile = blockIdx.x;
  const int64_t row = blockIdx.y;
  const int64_t base = (int64_t)tile * kTile;
  const int n = (int)min((int64_t)kTile, L - base);
  const uint16_t* src = ids_rows + row * L + base;
  for (int i = threadIdx.x; i < n_pad; i += kSortThreads)
    ka[i] = (i < n) ? (((uint32_t)src[i] << kPosBits) | (uint32_t)i) : 0xFFFFFFFFu;   // padding sorts last
  __syncthreads();
  // digits of the id, low first (at most 8 bits each)
  const int passes = (nb + kMaxDigitBits - 1) / kMaxDigitBits;
  uint32_t* cur = ka;
  uint32_t* nxt = kb;
  int done = 0;
  for (int p = 0; p < passes; ++p) {
    const int bits = (nb - done + (passes - p) - 1) / (passes - p);        // split nb evenly over the passes
    radix_pass(cur, nxt, tab, n_pad, kPosBits + done, bits);
    done += bits;
    uint32_t* t = cur; cur = nxt; nxt = t;
  }
  if (ntiles == 1) {
    for (int i = threadIdx.x; i < n; i += kSortThreads) {
      const uint32_t k = cur[i];
      orden[row * L + i] = (int32_t)(k & kPosMask);
      ids_o[row * L + i] = (uint16_t)(k >> kPosBits);
    }
    return;
  }
  uint32_t* t = tmp + row * L + base;
  int32_t* hrow = hist + (row * ntiles + tile) * ((int64_t)1 << nb);
  for (int i = threadIdx.x; i < n; i += kSortThreads) {
    const uint32_t k = cur[i];
    t[i] = k;
    const uint32_t id = k >> kPosBits;
    if (i == n - 1 || (cur[i + 1] >> kPosBits) != id) {
      const int first = lower_bound_u32(cur, n, id << kPosBits);
      hrow[id] = i - first + 1;
    }
  }
}

// hist[row][tile][bin] (counts) -> the global slot where the tile's run of bin starts, in three passes that keep
// every SM busy (a row has 2^nb bins, up to 65536): (1) per bin its total over the tiles, a thread per bin, the
// tiles' counts read coalesced across the bins; (2) per row an exclusive scan of the totals, one block per row;
// (3) per bin the running offsets over the tiles, written in place.
constexpr int kBinThreads = 256;

__global__ void __launch_bounds__(kBinThreads) k_bsort_bin_totals(const int32_t* __restrict__ hist, int ntiles,
                                                                  int nbins, int32_t* __restrict__ tot) {
  const int64_t row = blockIdx.y;
  const int bin = blockIdx.x * kBinThreads + threadIdx.x;
  if (bin >= nbins) return;
  const int32_t* h = hist + row * (int64_t)ntiles * nbins + bin;
  int run = 0;
  for (int tl = 0; tl < ntiles; ++tl) run += h[(int64_t)tl * nbins];
  tot[row * nbins + bin] = run;
}

__global__ void __launch_bounds__(1024) k_bsort_bin_scan(int32_t* __restrict__ tot, int nbins) {
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
}

__global__ void __launch_bounds__(kBinThreads) k_bsort_bin_offsets(int32_t* __restrict__ hist, int ntiles, int nbins,
                                                                   const int32_t* __restrict__ tot) {
  const int64_t row = blockIdx.y;
  const int bin = blockIdx.x * kBinThreads + threadIdx.x;
  if (bin >= nbins) return;
  int32_t* h = hist + row * (int64_t)ntiles * nbins + bin;
  int off = tot[row * nbins + bin];
  for (int tl = 0; tl < ntiles; ++tl) {
    const int c = h[(int64_t)tl * nbins];
    h[(int64_t)tl * nbins] = off;
    off += c;
  }
}

__global__ void __launch_bounds__(1024) k_bsort_scatter(const uint32_t* __restrict__ tmp,
                                                        const int32_t* __restrict__ hist, int64_t L, int ntiles,
                                                        int nb, int32_t* __restrict__ orden,
                                                        uint16_t* __restrict__ ids_o) {
  extern __shared__ uint32_t keys[];
  const int tile = blockIdx.x;
  const int64_t row = blockIdx.y;
  const int64_t base = (int64_t)tile * kTile;
  const int n = (int)min((int64_t)kTile, L - base);
  const uint32_t* t = tmp + row * L + base;
  for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = t[i];
  __syncthreads();
  const int32_t* hrow = hist + (row * ntiles + tile) * ((int64_t)1 << nb);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t k = keys[i];
    const uint32_t id = k >> kPosBits;
    const int first = lower_bound_u32(keys, n, id << kPosBits);
    const int64_t dst = row * L + hrow[id] + (i - first);
    orden[dst] = (int32_t)(base + (k & kPosMask));
    ids_o[dst] = (uint16_t)id;
  }
}

static int ntiles_of(int64_t L) { return (int)((L + kTile - 1) / kTile); }

size_t bucket_sort_workspace(int64_t rows, int64_t L, int nb) {
  if (rows <= 0 || L <= 0 || nb < 1 || nb > 16) return 0;
  const int nt = ntiles_of(L);
  if (nt <= 1) return 0;
  return align_up((size_t)rows * L * 4) + align_up((size_t)rows * nt * ((size_t)1 << nb) * 4) +
         align_up((size_t)rows * ((size_t)1 << nb) * 4);
}

int launch_bucket_sort(int64_t rows, int64_t L, int nb, const uint16_t* ids_rows, int32_t* orden, uint16_t* ids_o,
                       void* ws, size_t ws_bytes, cudaStream_t s) {
  if (rows < 0 || L < 0) return ASRN_ERR_ARG;
  if (rows == 0 || L == 0) return ASRN_OK;
  // sizes whose byte counts would overflow, or a position that does not fit int32
  if (nb < 1 || nb > 16 || L > ((int64_t)1 << 31) - 1 || rows > ((int64_t)1 << 40) / L) return ASRN_ERR_ARG;
  const int nt = ntiles_of(L);
  const int64_t tile_len = L < kTile ? L : (int64_t)kTile;
  const int n_pad = (int)((tile_len + kSortThreads - 1) / kSortThreads * kSortThreads);
  cudaFuncSetAttribute(k_bsort_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSortSmem);
  cudaFuncSetAttribute(k_bsort_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize, kTile * 4);
  if (nt == 1) {
    for (int64_t r0 = 0; r0 < rows; r0 += kMaxGridY) {        // grid.y holds at most 65535 rows per launch
      const unsigned nr = (unsigned)(rows - r0 < kMaxGridY ? rows - r0 : kMaxGridY);
      k_bsort_tile<<<dim3(1, nr), kSortThreads, kSortSmem, s>>>(ids_rows + r0 * L, L, 1, n_pad, nb, orden + r0 * L,
                                                                ids_o + r0 * L, nullptr, nullptr);
    }
    return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
  }
  if (ws_bytes < bucket_sort_workspace(rows, L, nb) || ws == nullptr) return ASRN_ERR_WORKSPACE;
  const int nbins = 1 << nb;
  uint32_t* tmp = reinterpret_cast<uint32_t*>(ws);
  int32_t* hist = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(ws) + align_up((size_t)rows * L * 4));
  const size_t hist_bytes = (size_t)rows * nt * nbins * 4;
  int32_t* tot = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(hist) + align_up(hist_bytes));
  if (cudaMemsetAsync(hist, 0, hist_bytes, s) != cudaSuccess) return ASRN_ERR_CUDA;
  for (int64_t r0 = 0; r0 < rows; r0 += kMaxGridY) {
    const unsigned nr = (unsigned)(rows - r0 < kMaxGridY ? rows - r0 : kMaxGridY);
    const uint16_t* ir = ids_rows + r0 * L;
    int32_t* ho = hist + r0 * nt * nbins;
    int32_t* to = tot + r0 * nbins;
    uint32_t* tm = tmp + r0 * L;
    k_bsort_tile<<<dim3(nt, nr), kSortThreads, kSortSmem, s>>>(ir, L, nt, n_pad, nb, nullptr, nullptr, tm, ho);
    const dim3 bin_grid((unsigned)((nbins + kBinThreads - 1) / kBinThreads), nr);
    k_bsort_bin_totals<<<bin_grid, kBinThreads, 0, s>>>(ho, nt, nbins, to);
    k_bsort_bin_scan<<<nr, 1024, 0, s>>>(to, nbins);
    k_bsort_bin_offsets<<<bin_grid, kBinThreads, 0, s>>>(ho, nt, nbins, to);
    k_bsort_scatter<<<dim3(nt, nr), 1024, kTile * 4, s>>>(tm, ho, L, nt, nb, orden + r0 * L, ids_o + r0 * L);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

// ---- allocation-free variant -----------------------------------------------------------------------------------
// For callers that cannot allocate device memory at the time they sort: a plug-in that runs inside a host process
// whose allocator it does not own, a serving loop that must keep a fixed memory footprint after start-up, or code that
// runs while other work holds the allocator. The scratch of rows longer than one tile (the tiles' sorted keys and their
// bucket histograms) lives in a fixed device array of this library instead of a caller-provided workspace.
// Every GPU that loads the library keeps this array until the process exits. All calls share it and it keeps the last
// call's contents: the histogram part is cleared on the stream before each use, and calls that overlap on the GPU (two
// streams, or two host threads) race on it -- order them on one stream.
constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;   // 32 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array in the current CUDA context. In host code the array's name only stands for the
// symbol; kernels must be given this address. It is looked up on every call (a host-side query, no stream work), so
// it stays right after a context is destroyed and created again (cudaDeviceReset), where the array may have moved.
static int noalloc_scratch(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return ASRN_ERR_CUDA;
  *out = p;
  return ASRN_OK;
}

int launch_bucket_sort_noalloc(int64_t rows, int64_t L, int nb, const uint16_t* ids_rows, int32_t* orden,
                               uint16_t* ids_o, cudaStream_t s) {
  if (rows < 0 || L < 0) return ASRN_ERR_ARG;
  if (rows == 0 || L == 0) return ASRN_OK;                  // as asrn_bucket_sort: nothing to sort, nothing checked
  if (nb < 1 || nb > 16 || L > ((int64_t)1 << 31) - 1 || rows > ((int64_t)1 << 40) / L) return ASRN_ERR_ARG;
  const size_t need = bucket_sort_workspace(rows, L, nb);
  if (need > kNoAllocScratchBytes) return ASRN_ERR_WORKSPACE;
  void* ws = nullptr;
  if (need > 0) {
    const int st = noalloc_scratch(&ws);
    if (st != ASRN_OK) return st;
  }
  return launch_bucket_sort(rows, L, nb, ids_rows, orden, ids_o, ws, need, s);
}

}  // namespace asrn
