// Repetition memory: "seen" flags, Hawkes intensity per n-gram order, and the repetition streak.
// Reference: CapaASRNEstable._repeticion (asrn/estable.py:304-321) with _claves_de (asrn/nucleo.py:175-185),
// _ordenar_claves (asrn/nucleo.py:693-701) and escaneo (asrn/nucleo.py:188-257):
//   key_n(t) = ((0 + s_t c_0) + s_{t-1} c_1) + ... + s_{t-n} c_n   in fp64, this order, no FMA; NaN before the start
//   per (b, n): stable sort by key (NaN last); repetido_i = key_i == key_{i-1}
//   a_i = repetido_i * exp(-kappa_n * float(max(0, B_i - B_{i-1}))),  lambda_i = a_i (lambda_{i-1} + alfa_{i-1})
//   hawkes / vistos scattered back to text order; streak S_t = r_t exp(-kappa_r beta_t) S_{t-1} + r_t with
//   r_t = vistos of the longest order.
// Rows of at most 8192 positions: one block per (b, n) row sorts (key, position) pairs in shared memory with an LSD
// radix sort on the 64-bit order-preserving key (8-bit digits, per-warp histograms, __match_any_sync ranking; a pass
// whose digit is the same for every key is skipped), then runs a block-wide scan of affine maps over the sorted row.
// Longer rows (workspace from repetition_workspace): tiles are sorted with a bitonic network and written out, runs are
// merged pairwise (merge path, log2(tiles) passes), then a tiled scan writes each tile's local inclusive maps and its
// aggregate, and a last pass composes the aggregates of the earlier tiles into each element and scatters to text
// order. Keys are unique as (key, position) pairs, so every correct sort gives the stable argsort of the reference.
#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kRepMaxL = 16384;   // tile of the long-row path (16384 x 12 B of shared memory)
constexpr int kRepRowMaxL = 8192; // rows radix-sorted in one block: 2 x 8192 x 12 B of key / position buffers
constexpr int kRxThreads = 1024, kRxWarps = kRxThreads / 32;
constexpr size_t kRxTabBytes = (size_t)kRxWarps * 256 * 2;   // (digit, warp) counts / offsets, 16-bit

// One stable counting-sort pass of n_pad (key, position) pairs by the digit (key >> shift) & 255, src -> dst, with
// the rank of each key among equal digits of its 32-key group from __match_any_sync. Returns false (and moves
// nothing) when every key has the same digit: the order is already sorted by it.
__device__ __forceinline__ bool radix_pass64(const uint64_t* sk, const uint32_t* sp, uint64_t* dk, uint32_t* dp,
                                             uint16_t* tab, int n_pad, int shift) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int seg = n_pad / kRxWarps;                   // a multiple of 32
  const uint32_t lt = (1u << lane) - 1;
  const uint32_t d0 = (uint32_t)(sk[0] >> shift) & 255u;
  for (int i = threadIdx.x; i < kRxWarps * 256; i += kRxThreads) tab[i] = 0;
  __syncthreads();
  int differs = 0;
  for (int j = 0; j < seg; j += 32) {
    const uint32_t d = (uint32_t)(sk[w * seg + j + lane] >> shift) & 255u;
    differs |= d != d0;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    if ((peers & lt) == 0) tab[d * kRxWarps + w] += (uint16_t)__popc(peers);
  }
  if (!__syncthreads_or(differs)) return false;
  {   // exclusive scan of tab in (digit, warp) order, 8 consecutive entries per thread
    __shared__ int wsum[kRxWarps];
    const int e0 = threadIdx.x * 8;
    int local = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) local += tab[e0 + k];
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
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = tab[e0 + k];
      tab[e0 + k] = (uint16_t)run;
      run += c;
    }
  }
  __syncthreads();
  for (int j = 0; j < seg; j += 32) {
    const int i = w * seg + j + lane;
    const uint64_t k = sk[i];
    const uint32_t d = (uint32_t)(k >> shift) & 255u;
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    const int base = tab[d * kRxWarps + w];
    const int at = base + __popc(peers & lt);
    dk[at] = k;
    dp[at] = sp[i];
    __syncwarp();
    if ((peers & lt) == 0) tab[d * kRxWarps + w] = (uint16_t)(base + __popc(peers));
    __syncwarp();
  }
  __syncthreads();
  return true;
}

__device__ __forceinline__ bool pair_less(uint64_t ka, uint32_t pa, uint64_t kb, uint32_t pb) {
  return ka < kb || (ka == kb && pa < pb);
}

// Block-wide inclusive scan of affine maps; each thread holds `items` consecutive elements in v[].
template <int kItems>
__device__ __forceinline__ void block_scan_affine(Affine* v, Affine* warp_agg) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int k = 1; k < kItems; ++k) v[k] = compose(v[k - 1], v[k]);
  Affine tot = v[kItems - 1];
  // warp inclusive scan of thread aggregates
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    Affine y;
    y.a = __shfl_up_sync(0xffffffffu, tot.a, o);
    y.b = __shfl_up_sync(0xffffffffu, tot.b, o);
    if (lane >= o) tot = compose(y, tot);
  }
  if (lane == 31) warp_agg[wid] = tot;
  __syncthreads();
  if (wid == 0) {
    Affine w = (lane < (int)(blockDim.x >> 5)) ? warp_agg[lane] : Affine{1.f, 0.f};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      Affine y;
      y.a = __shfl_up_sync(0xffffffffu, w.a, o);
      y.b = __shfl_up_sync(0xffffffffu, w.b, o);
      if (lane >= o) w = compose(y, w);
    }
    warp_agg[lane] = w;
  }
  __syncthreads();
  // exclusive prefix of this thread = (previous warps) o (previous lanes of this warp)
  Affine pre = Affine{1.f, 0.f};
  if (wid > 0) pre = warp_agg[wid - 1];
  Affine lanepre;
  lanepre.a = __shfl_up_sync(0xffffffffu, tot.a, 1);
  lanepre.b = __shfl_up_sync(0xffffffffu, tot.b, 1);
  if (lane > 0) pre = compose(pre, lanepre);
#pragma unroll
  for (int k = 0; k < kItems; ++k) v[k] = compose(pre, v[k]);
}

// The signature at t of a row: the token id as fp32 when the row's tokens are given, else sig (firmas_de_piezas,
// asrn/nucleo.py:161-164, or E . r_firma).
__device__ __forceinline__ double sig_at(const float* sig, const int64_t* tok, int64_t t) {
  return tok ? (double)(float)tok[t] : (double)sig[t];
}

__device__ __forceinline__ double ngram_key_at(const float* sig, const int64_t* tok, int64_t i, int ni,
                                               const double* c) {
  double key = 0.0;
  for (int j = 0; j <= ni; ++j) {
    const int64_t t = i - j;
    const double s = (t >= 0) ? sig_at(sig, tok, t) : __longlong_as_double(0x7ff8000000000000ll);
    key = __dadd_rn(key, __dmul_rn(s, c[j]));
  }
  return key;
}

template <int kItems>
__global__ void __launch_bounds__(kRxThreads) k_ngram_row(RepetitionArgs a, int n2) {
  // n2: the row length rounded up to a multiple of 1024 (the sort's padding keys are all ones: they sort last)
  extern __shared__ __align__(16) char smem_raw[];
  __shared__ Affine warp_agg[32];
  const int64_t b = blockIdx.x / a.n;
  const int ni = (int)(blockIdx.x % a.n);
  const int64_t L = a.L;
  const uint64_t* sk;
  const uint32_t* sp;
  if (a.ng_mode == kNgScanOnly) {
    sk = a.ng_keys + (int64_t)blockIdx.x * L;
    sp = a.ng_pos + (int64_t)blockIdx.x * L;
  } else {
    uint64_t* k0 = reinterpret_cast<uint64_t*>(smem_raw);
    uint64_t* k1 = k0 + n2;
    uint32_t* p0 = reinterpret_cast<uint32_t*>(k1 + n2);
    uint32_t* p1 = p0 + n2;
    uint16_t* tab = reinterpret_cast<uint16_t*>(p1 + n2);
    const float* sig = a.sig ? a.sig + b * L : nullptr;
    const int64_t* tok = a.tok ? a.tok + b * L : nullptr;
    // keys of the (ni + 1)-token groups ending at t (asrn/nucleo.py:175-185)
    for (int i = threadIdx.x; i < n2; i += blockDim.x) {
      if (i < L) {
        const double key = ngram_key_at(sig, tok, i, ni, a.c);
        if (a.keys) a.keys[(b * L + i) * a.n + ni] = key;
        k0[i] = sortable_key(key);
        p0[i] = (uint32_t)i;
      } else {
        k0[i] = 0xFFFFFFFFFFFFFFFFull;
        p0[i] = 0xFFFFFFFFu;
      }
    }
    __syncthreads();
    // stable LSD radix sort by key: positions start ascending, so equal keys keep position order
    uint64_t* ck = k0;
    uint32_t* cp = p0;
    for (int shift = 0; shift < 64; shift += 8) {
      uint64_t* dk = ck == k0 ? k1 : k0;
      uint32_t* dp = cp == p0 ? p1 : p0;
      if (radix_pass64(ck, cp, dk, dp, tab, n2, shift)) {
        ck = dk;
        cp = dp;
      }
    }
    if (a.ng_mode == kNgSortOnly) {
      for (int i = threadIdx.x; i < L; i += blockDim.x) {
        a.ng_keys[(int64_t)blockIdx.x * L + i] = ck[i];
        a.ng_pos[(int64_t)blockIdx.x * L + i] = cp[i];
      }
      return;
    }
    sk = ck;
    sp = cp;
  }
  // affine elements in sorted order; thread owns kItems consecutive slots
  const float kappa = a.kappa[ni];
  Affine v[kItems];
  bool rep[kItems];
  const int i0 = threadIdx.x * kItems;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int i = i0 + k;
    rep[k] = false;
    v[k] = Affine{0.f, 0.f};
    if (i < L) {
      rep[k] = i > 0 && sk[i] == sk[i - 1] && sk[i] != 0xFFFFFFFFFFFFFFFFull;
      if (rep[k]) {
        const int64_t pc = sp[i], pp = sp[i - 1];
        const double dB = fmax(a.Bt[b * L + pc] - a.Bt[b * L + pp], 0.0);
        const float av = expf(__fmul_rn(-kappa, __double2float_rn(dB)));
        v[k] = Affine{av, __fmul_rn(av, expf(a.log_alfa[b * L + pp]))};
      }
    } else {
      v[k] = Affine{1.f, 0.f};
    }
  }
  block_scan_affine<kItems>(v, warp_agg);
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int i = i0 + k;
    if (i < L) {
      const int64_t pc = sp[i];
      a.hawkes[(b * L + pc) * a.n + ni] = v[k].b;
      a.vistos[(b * L + pc) * a.n + ni] = rep[k] ? 1 : 0;
      if (a.orden_ng) a.orden_ng[(b * a.n + ni) * L + i] = (int32_t)pc;
      if (a.repetido) a.repetido[(b * a.n + ni) * L + i] = rep[k] ? 1 : 0;
    }
  }
}

// Streak scan in text order, one block per batch row, chunks of 1024 * 4 with a carried affine map.
__global__ void __launch_bounds__(1024) k_racha(RepetitionArgs a) {
  const int64_t b = blockIdx.x;
  const int64_t L = a.L;
  const float kr = a.kappa[a.n];
  __shared__ Affine warp_agg[32];
  __shared__ Affine carry_s;
  // the map from the streak before the row (0, or racha_in) to each position; with racha_in the carry is constant
  if (threadIdx.x == 0) carry_s = a.racha_in ? Affine{0.f, a.racha_in[b]} : Affine{1.f, 0.f};
  __syncthreads();
  constexpr int kItems = 4;
  for (int64_t base = 0; base < L; base += 1024 * kItems) {
    Affine v[kItems];
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int64_t t = base + (int64_t)threadIdx.x * kItems + k;
      if (t < L) {
        const float r = (float)a.vistos[(b * L + t) * a.n + (a.n - 1)];
        const float e = expf(__fmul_rn(-kr, (float)a.beta[b * L + t]));
        v[k] = Affine{__fmul_rn(r, e), r};
      } else {
        v[k] = Affine{1.f, 0.f};
      }
    }
    block_scan_affine<kItems>(v, warp_agg);
    const Affine carry = carry_s;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int64_t t = base + (int64_t)threadIdx.x * kItems + k;
      const Affine s = compose(carry, v[k]);
      if (t < L && a.racha) a.racha[b * L + t] = s.b;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry_s = compose(carry, v[kItems - 1]);
    __syncthreads();
  }
  if (a.racha_map && threadIdx.x == 0) {
    a.racha_map[2 * b] = carry_s.a;
    a.racha_map[2 * b + 1] = carry_s.b;
  }
}

// Streak over long rows of few sequences, in parallel over tiles of kRachaTile positions: each tile's local maps and
// its aggregate, then each tile composes the aggregates before it (and racha_in) into its positions.
constexpr int kRachaItems = 4;
constexpr int kRachaTile = 1024 * kRachaItems;

__global__ void __launch_bounds__(1024) k_racha_tile(RepetitionArgs a, int64_t tiles, float2* vloc, float2* agg) {
  __shared__ Affine warp_agg[32];
  const int64_t b = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t L = a.L;
  const float kr = a.kappa[a.n];
  Affine v[kRachaItems];
  const int64_t t0 = tile * kRachaTile + (int64_t)threadIdx.x * kRachaItems;
#pragma unroll
  for (int k = 0; k < kRachaItems; ++k) {
    const int64_t t = t0 + k;
    if (t < L) {
      const float r = (float)a.vistos[(b * L + t) * a.n + (a.n - 1)];
      const float e = expf(__fmul_rn(-kr, (float)a.beta[b * L + t]));
      v[k] = Affine{__fmul_rn(r, e), r};
    } else {
      v[k] = Affine{1.f, 0.f};
    }
  }
  block_scan_affine<kRachaItems>(v, warp_agg);
#pragma unroll
  for (int k = 0; k < kRachaItems; ++k) {
    const int64_t t = t0 + k;
    if (t < L) vloc[b * L + t] = make_float2(v[k].a, v[k].b);
  }
  if (threadIdx.x == blockDim.x - 1) agg[b * tiles + tile] = make_float2(v[kRachaItems - 1].a, v[kRachaItems - 1].b);
}

__global__ void __launch_bounds__(1024) k_racha_apply(RepetitionArgs a, int64_t tiles, const float2* vloc,
                                                      const float2* agg) {
  __shared__ Affine carry_s;
  const int64_t b = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t L = a.L;
  if (threadIdx.x == 0) {
    Affine c = a.racha_in ? Affine{0.f, a.racha_in[b]} : Affine{1.f, 0.f};
    for (int64_t q = 0; q < tile; ++q) {
      const float2 g = agg[b * tiles + q];
      c = compose(c, Affine{g.x, g.y});
    }
    carry_s = c;
  }
  __syncthreads();
  const Affine c = carry_s;
  const int64_t end = (tile + 1) * kRachaTile < L ? (tile + 1) * kRachaTile : L;
  for (int64_t t = tile * kRachaTile + threadIdx.x; t < end; t += blockDim.x) {
    const float2 lv = vloc[b * L + t];
    const Affine s = compose(c, Affine{lv.x, lv.y});
    if (a.racha) a.racha[b * L + t] = s.b;
  }
  if (a.racha_map && tile == tiles - 1 && threadIdx.x == 0) {
    const float2 lv = vloc[b * L + L - 1];
    const Affine s = compose(c, Affine{lv.x, lv.y});
    a.racha_map[2 * b] = s.a;
    a.racha_map[2 * b + 1] = s.b;
  }
}

// ---- rows longer than kRepMaxL ---------------------------------------------------------------------------------------

constexpr int kRepTile = kRepMaxL;   // scan tiles
constexpr int kSortTile = 4096;      // sort tiles: 4 keys per thread, 48 KB of shared memory, many blocks per row
constexpr int kMergeItems = 8;

struct RepLong {
  uint64_t *k0, *k1;   // (rows, L) sortable keys, ping-pong
  uint32_t *p0, *p1;   // (rows, L) positions, ping-pong
  float2* vloc;        // (rows, L) tile-local inclusive maps (a, b)
  float2* agg;         // (rows, tiles) tile aggregates
};


__global__ void __launch_bounds__(1024) k_ngram_tile_sort(RepetitionArgs a, int64_t tiles, uint64_t* K, uint32_t* Pp) {
  extern __shared__ __align__(16) char smem_raw[];
  uint64_t* sk = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* sp = reinterpret_cast<uint32_t*>(sk + kSortTile);
  const int64_t row = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const int64_t L = a.L, base = tile * kSortTile;
  const float* sig = a.sig ? a.sig + b * a.Lf : nullptr;
  const int64_t* tok = a.tok ? a.tok + b * a.Lf : nullptr;
  for (int i = threadIdx.x; i < kSortTile; i += blockDim.x) {
    const int64_t p = base + i;
    if (p < L) {
      const double key = ngram_key_at(sig, tok, a.pos0 + p, ni, a.c);
      if (a.keys) a.keys[(b * L + p) * a.n + ni] = key;
      sk[i] = sortable_key(key);
      sp[i] = (uint32_t)(a.pos0 + p);
    } else {
      sk[i] = 0xFFFFFFFFFFFFFFFFull;
      sp[i] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();
  for (int k = 2; k <= kSortTile; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < kSortTile; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t ka = sk[i], kb = sk[ixj];
          const uint32_t pa = sp[i], pb = sp[ixj];
          const bool up = (i & k) == 0;
          if (pair_less(kb, pb, ka, pa) == up) {
            sk[i] = kb; sk[ixj] = ka;
            sp[i] = pb; sp[ixj] = pa;
          }
        }
      }
      __syncthreads();
    }
  }
  const int64_t cnt = L - base < kSortTile ? L - base : kSortTile;
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
    K[row * L + base + i] = sk[i];
    Pp[row * L + base + i] = sp[i];
  }
}

// Merge sorted runs of width w pairwise; each thread writes kMergeItems consecutive outputs of one pair, starting from
// its merge-path diagonal (binary search).
__global__ void __launch_bounds__(256) k_ngram_merge(const uint64_t* __restrict__ Kin, const uint32_t* __restrict__ Pin,
                                                     uint64_t* __restrict__ Kout, uint32_t* __restrict__ Pout,
                                                     int64_t rows, int64_t L, int64_t w) {
  const int64_t per_row = (L + kMergeItems - 1) / kMergeItems;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= rows * per_row) return;
  const int64_t row = gid / per_row;
  const int64_t o0 = (gid % per_row) * kMergeItems;
  const int64_t s = (o0 / (2 * w)) * (2 * w);
  const int64_t la = L - s < w ? L - s : w;
  const int64_t lb = L - s - la < w ? L - s - la : w;
  const uint64_t* KA = Kin + row * L + s;
  const uint32_t* PA = Pin + row * L + s;
  const uint64_t* KB = KA + la;
  const uint32_t* PB = PA + la;
  const int64_t k = o0 - s;
  const int64_t kend = (k + kMergeItems < la + lb) ? k + kMergeItems : la + lb;
  int64_t lo = k - lb > 0 ? k - lb : 0, hi = k < la ? k : la;
  while (lo < hi) {          // first i with A[i] > B[k - 1 - i]
    const int64_t mid = (lo + hi) >> 1;
    if (pair_less(KA[mid], PA[mid], KB[k - 1 - mid], PB[k - 1 - mid])) lo = mid + 1;
    else hi = mid;
  }
  int64_t i = lo, j = k - lo;
  uint64_t* ko = Kout + row * L + s;
  uint32_t* po = Pout + row * L + s;
  for (int64_t o = k; o < kend; ++o) {
    const bool take_a = j >= lb || (i < la && pair_less(KA[i], PA[i], KB[j], PB[j]));
    if (take_a) { ko[o] = KA[i]; po[o] = PA[i]; ++i; }
    else { ko[o] = KB[j]; po[o] = PB[j]; ++j; }
  }
}

// Affine element of sorted index i (asrn/estable.py:304-321).
__device__ __forceinline__ Affine ngram_elem(const RepetitionArgs& a, const uint64_t* K, const uint32_t* Pp, int64_t b,
                                             int64_t i, float kappa, bool* rep) {
  const int64_t L = a.L;
  *rep = i > 0 && K[i] == K[i - 1] && K[i] != 0xFFFFFFFFFFFFFFFFull;
  if (!*rep) return Affine{0.f, 0.f};
  const int64_t pc = Pp[i], pp = Pp[i - 1];
  const double dB = fmax(a.Bt[b * L + pc] - a.Bt[b * L + pp], 0.0);
  const float av = expf(__fmul_rn(-kappa, __double2float_rn(dB)));
  return Affine{av, __fmul_rn(av, expf(a.log_alfa[b * L + pp]))};
}

constexpr int kScanItems = kRepTile / 1024;

__global__ void __launch_bounds__(1024) k_ngram_scan_tile(RepetitionArgs a, int64_t tiles, const uint64_t* K,
                                                          const uint32_t* Pp, float2* vloc, float2* agg) {
  __shared__ Affine warp_agg[32];
  const int64_t row = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const int64_t L = a.L;
  const float kappa = a.kappa[ni];
  const uint64_t* Kr = K + row * L;
  const uint32_t* Pr = Pp + row * L;
  Affine v[kScanItems];
  const int64_t i0 = tile * kRepTile + (int64_t)threadIdx.x * kScanItems;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = i0 + k;
    bool rep;
    v[k] = (i < L) ? ngram_elem(a, Kr, Pr, b, i, kappa, &rep) : Affine{1.f, 0.f};
  }
  block_scan_affine<kScanItems>(v, warp_agg);
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = i0 + k;
    if (i < L) vloc[row * L + i] = make_float2(v[k].a, v[k].b);
  }
  if (threadIdx.x == blockDim.x - 1) agg[row * tiles + tile] = make_float2(v[kScanItems - 1].a, v[kScanItems - 1].b);
}

__global__ void __launch_bounds__(1024) k_ngram_apply(RepetitionArgs a, int64_t tiles, const uint64_t* K,
                                                      const uint32_t* Pp, const float2* vloc, const float2* agg) {
  __shared__ Affine carry_s;
  const int64_t row = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const int64_t L = a.L;
  if (threadIdx.x == 0) {
    Affine c{1.f, 0.f};
    for (int64_t q = 0; q < tile; ++q) {
      const float2 g = agg[row * tiles + q];
      c = compose(c, Affine{g.x, g.y});
    }
    carry_s = c;
  }
  __syncthreads();
  const Affine carry = carry_s;
  const uint64_t* Kr = K + row * L;
  const uint32_t* Pr = Pp + row * L;
  const int64_t end = (tile + 1) * kRepTile < L ? (tile + 1) * kRepTile : L;
  for (int64_t i = tile * kRepTile + threadIdx.x; i < end; i += blockDim.x) {
    const float2 lv = vloc[row * L + i];
    const Affine s = compose(carry, Affine{lv.x, lv.y});
    const bool rep = i > 0 && Kr[i] == Kr[i - 1] && Kr[i] != 0xFFFFFFFFFFFFFFFFull;
    const int64_t pc = Pr[i];
    a.hawkes[(b * L + pc) * a.n + ni] = s.b;
    a.vistos[(b * L + pc) * a.n + ni] = rep ? 1 : 0;
    if (a.orden_ng) a.orden_ng[(b * a.n + ni) * L + i] = (int32_t)pc;
    if (a.repetido) a.repetido[(b * a.n + ni) * L + i] = rep ? 1 : 0;
  }
}

static RepLong rep_long_layout(void* ws, int64_t rows, int64_t L) {
  char* p = reinterpret_cast<char*>(ws);
  const size_t E = (size_t)rows * L;
  RepLong r;
  size_t o = 0;
  r.k0 = reinterpret_cast<uint64_t*>(p + o); o = align_up(o + E * 8);
  r.k1 = reinterpret_cast<uint64_t*>(p + o); o = align_up(o + E * 8);
  r.p0 = reinterpret_cast<uint32_t*>(p + o); o = align_up(o + E * 4);
  r.p1 = reinterpret_cast<uint32_t*>(p + o); o = align_up(o + E * 4);
  r.vloc = reinterpret_cast<float2*>(p + o); o = align_up(o + E * 8);
  r.agg = reinterpret_cast<float2*>(p + o);
  return r;
}

// Rows longer than one block's shared-memory sort take the tiled path (tile sorts, merges, tiled scans); shorter rows
// are sorted and scanned by one block each (measured as fast as the tiled path at 32 x 4 rows of 8192 positions).
static bool rep_tiled(int64_t L) { return L > kRepRowMaxL; }

size_t repetition_workspace(int64_t B, int64_t L, int n) {
  if (!rep_tiled(L)) return 0;
  const size_t rows = (size_t)B * n, E = rows * (size_t)L;
  const size_t tiles = (size_t)((L + kRepTile - 1) / kRepTile);
  return align_up(E * 8) * 2 + align_up(E * 4) * 2 + align_up(E * 8) + align_up(rows * tiles * 8);
}

static int launch_repetition_long(const RepetitionArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (a.L >= ((int64_t)1 << 31)) return ASRN_ERR_UNSUPPORTED;
  if (!ws || ws_bytes < repetition_workspace(a.B, a.L, a.n)) return ASRN_ERR_WORKSPACE;
  const int64_t rows = a.B * a.n, L = a.L;
  const int64_t tiles = (L + kRepTile - 1) / kRepTile;
  const int64_t stiles = (L + kSortTile - 1) / kSortTile;
  RepLong r = rep_long_layout(ws, rows, L);
  uint64_t* kin = r.k0;
  uint32_t* pin = r.p0;
  if (a.ng_mode == kNgScanOnly) {
    kin = a.ng_keys;
    pin = a.ng_pos;
  } else {
    const size_t smem = (size_t)kSortTile * 12;
    cudaFuncSetAttribute(k_ngram_tile_sort, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_tile_sort<<<(unsigned)(rows * stiles), 1024, smem, s>>>(a, stiles, r.k0, r.p0);
    uint64_t* kout = r.k1;
    uint32_t* pout = r.p1;
    const int64_t per_row = (L + kMergeItems - 1) / kMergeItems;
    for (int64_t w = kSortTile; w < L; w <<= 1) {
      k_ngram_merge<<<(unsigned)((rows * per_row + 255) / 256), 256, 0, s>>>(kin, pin, kout, pout, rows, L, w);
      uint64_t* tk = kin; kin = kout; kout = tk;
      uint32_t* tp = pin; pin = pout; pout = tp;
    }
    if (a.ng_mode == kNgSortOnly) {
      if (cudaMemcpyAsync(a.ng_keys, kin, (size_t)rows * L * 8, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
          cudaMemcpyAsync(a.ng_pos, pin, (size_t)rows * L * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return ASRN_ERR_CUDA;
      return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
    }
  }
  k_ngram_scan_tile<<<(unsigned)(rows * tiles), 1024, 0, s>>>(a, tiles, kin, pin, r.vloc, r.agg);
  k_ngram_apply<<<(unsigned)(rows * tiles), 1024, 0, s>>>(a, tiles, kin, pin, r.vloc, r.agg);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

// ---- chunk of a sequence-sharded row ---------------------------------------------------------------------------
// Shard r owns positions [pos0, pos0 + Lc) of every sequence; the per-position inputs (signatures, clock, log alfa)
// are the gathered full rows. The n-gram memory of the chunk (asrn/estable.py:304-321) in two calls around one
// exchange:
//   sort    the chunk's (key, position) pairs per (b, n) row (tile sort + merges), then two scans over the sorted row:
//           lambda with the chunk alone (a group's first slot starts from 0) and P_i, the product of a_j over the
//           group's slots after its first up to i. Out: the sorted keys and, at each group's first slot, its summary
//           {B of its first and last occurrence, lambda and P at its last slot, alfa of its last occurrence}.
//   finish  per group, the state after the earlier chunks: walk the earlier shards in order, find the key in each
//           one's sorted keys (binary search) and fold its summary: lambda <- P_L * a(B_first - B) * (lambda + alfa)
//           + lambda_L, then alfa, B <- the last occurrence's. The chunk's first occurrence of a key seen before is
//           a repeat (vistos = 1) and every slot of its group gets lambda_i + P_i * a(B_first - B) * (lambda + alfa):
//           the recursion lambda_i = a_i (lambda_{i-1} + alfa_{i-1}) is linear in the incoming state.
// The streak (racha) carries across chunks as an affine map (k_racha with racha_in / racha_map).
struct NgcSummary {
  double b_first, b_last;
  float lam, prod, alfa, pad;
};

struct NgcLayout {
  uint64_t *k0, *k1;
  uint32_t *p0, *p1;
  float4* vloc;        // (rows, Lc) tile-local inclusive maps of both scans (lambda a, b; product a, b)
  float4* agg;         // (rows, tiles)
  float2* lp;          // (rows, Lc) (lambda, P) per sorted slot
  float2* carry;       // (rows, Lc) at group-first slots: (c, seen)
  uint32_t* pos;       // (rows, Lc) sorted positions (the final ping-pong buffer's copy)
};

static NgcLayout ngc_layout(void* ws, int64_t rows, int64_t Lc) {
  char* p = reinterpret_cast<char*>(ws);
  const size_t E = (size_t)rows * Lc;
  const size_t tiles = (size_t)((Lc + kRepTile - 1) / kRepTile);
  NgcLayout r;
  size_t o = 0;
  r.k0 = reinterpret_cast<uint64_t*>(p + o); o = align_up(o + E * 8);
  r.k1 = reinterpret_cast<uint64_t*>(p + o); o = align_up(o + E * 8);
  r.p0 = reinterpret_cast<uint32_t*>(p + o); o = align_up(o + E * 4);
  r.p1 = reinterpret_cast<uint32_t*>(p + o); o = align_up(o + E * 4);
  r.vloc = reinterpret_cast<float4*>(p + o); o = align_up(o + E * 16);
  r.agg = reinterpret_cast<float4*>(p + o); o = align_up(o + rows * tiles * 16);
  r.lp = reinterpret_cast<float2*>(p + o); o = align_up(o + E * 8);
  r.carry = reinterpret_cast<float2*>(p + o); o = align_up(o + E * 8);
  r.pos = reinterpret_cast<uint32_t*>(p + o);
  return r;
}

size_t ngram_chunk_workspace(int64_t B, int64_t Lc, int n) {
  const size_t rows = (size_t)B * n, E = rows * (size_t)Lc;
  const size_t tiles = (size_t)((Lc + kRepTile - 1) / kRepTile);
  return 2 * align_up(E * 8) + 2 * align_up(E * 4) + align_up(E * 16) + align_up(rows * tiles * 16) +
         2 * align_up(E * 8) + align_up(E * 4);
}

// elements of the two scans at sorted slot i: lambda (as ngram_elem) and the in-group product
__device__ __forceinline__ void ngc_elems(const RepetitionArgs& a, const uint64_t* K, const uint32_t* P, int64_t b,
                                          int64_t i, float kappa, Affine* lam, Affine* prod) {
  const bool rep = i > 0 && K[i] == K[i - 1] && K[i] != 0xFFFFFFFFFFFFFFFFull;
  if (!rep) {
    *lam = Affine{0.f, 0.f};
    *prod = Affine{0.f, 1.f};
    return;
  }
  const int64_t pc = P[i], pp = P[i - 1];
  const double dB = fmax(a.Bt[b * a.Lf + pc] - a.Bt[b * a.Lf + pp], 0.0);
  const float av = expf(__fmul_rn(-kappa, __double2float_rn(dB)));
  *lam = Affine{av, __fmul_rn(av, expf(a.log_alfa[b * a.Lf + pp]))};
  *prod = Affine{av, 0.f};
}

__global__ void __launch_bounds__(1024) k_ngc_scan_tile(RepetitionArgs a, int64_t tiles, const uint64_t* K,
                                                        const uint32_t* Pp, float4* vloc, float4* agg) {
  __shared__ Affine warp_agg[32];
  const int64_t row = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const int64_t L = a.L;
  const float kappa = a.kappa[ni];
  const uint64_t* Kr = K + row * L;
  const uint32_t* Pr = Pp + row * L;
  Affine v[kScanItems], w[kScanItems];
  const int64_t i0 = tile * kRepTile + (int64_t)threadIdx.x * kScanItems;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = i0 + k;
    if (i < L) ngc_elems(a, Kr, Pr, b, i, kappa, &v[k], &w[k]);
    else v[k] = w[k] = Affine{1.f, 0.f};
  }
  block_scan_affine<kScanItems>(v, warp_agg);
  __syncthreads();
  block_scan_affine<kScanItems>(w, warp_agg);
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = i0 + k;
    if (i < L) vloc[row * L + i] = make_float4(v[k].a, v[k].b, w[k].a, w[k].b);
  }
  if (threadIdx.x == blockDim.x - 1)
    agg[row * tiles + tile] = make_float4(v[kScanItems - 1].a, v[kScanItems - 1].b, w[kScanItems - 1].a,
                                          w[kScanItems - 1].b);
}

__global__ void __launch_bounds__(1024) k_ngc_apply(RepetitionArgs a, int64_t tiles, const float4* vloc,
                                                    const float4* agg, float2* lp, const uint32_t* Pin,
                                                    uint32_t* Pout) {
  __shared__ Affine carry_s[2];
  const int64_t row = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  const int64_t L = a.L;
  if (threadIdx.x == 0) {
    Affine c{1.f, 0.f}, e{1.f, 0.f};
    for (int64_t q = 0; q < tile; ++q) {
      const float4 g = agg[row * tiles + q];
      c = compose(c, Affine{g.x, g.y});
      e = compose(e, Affine{g.z, g.w});
    }
    carry_s[0] = c;
    carry_s[1] = e;
  }
  __syncthreads();
  const Affine c = carry_s[0], e = carry_s[1];
  const int64_t end = (tile + 1) * kRepTile < L ? (tile + 1) * kRepTile : L;
  for (int64_t i = tile * kRepTile + threadIdx.x; i < end; i += blockDim.x) {
    const float4 v = vloc[row * L + i];
    lp[row * L + i] = make_float2(compose(c, Affine{v.x, v.y}).b, compose(e, Affine{v.z, v.w}).b);
    Pout[row * L + i] = Pin[row * L + i];
  }
}

// first index in K[lo, hi) with K[idx] >= v / > v
__device__ __forceinline__ int64_t lower_u64(const uint64_t* K, int64_t lo, int64_t hi, uint64_t v) {
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (K[mid] < v) lo = mid + 1; else hi = mid;
  }
  return lo;
}
__device__ __forceinline__ int64_t upper_u64(const uint64_t* K, int64_t lo, int64_t hi, uint64_t v) {
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (K[mid] <= v) lo = mid + 1; else hi = mid;
  }
  return lo;
}

__global__ void k_ngc_summary(RepetitionArgs a, const uint64_t* K, const uint32_t* P, const float2* lp,
                              uint64_t* keys_out, NgcSummary* summ) {
  const int64_t L = a.L;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= a.B * a.n * L) return;
  const int64_t row = g / L, i = g % L;
  const int64_t b = row / a.n;
  const uint64_t* Kr = K + row * L;
  const uint64_t k = Kr[i];
  keys_out[g] = k;
  if (k == 0xFFFFFFFFFFFFFFFFull || (i > 0 && Kr[i - 1] == k)) return;
  const int64_t last = upper_u64(Kr, i, L, k) - 1;
  const uint32_t* Pr = P + row * L;
  NgcSummary r;
  r.b_first = a.Bt[b * a.Lf + Pr[i]];
  r.b_last = a.Bt[b * a.Lf + Pr[last]];
  r.lam = lp[row * L + last].x;
  r.prod = lp[row * L + last].y;
  r.alfa = expf(a.log_alfa[b * a.Lf + Pr[last]]);
  r.pad = 0.f;
  summ[g] = r;
}

// per group-first slot of this chunk: (c, seen) from the earlier chunks' summaries, in rank order
__global__ void k_ngc_resolve(RepetitionArgs a, int n_prev, const uint64_t* keys_prev, const NgcSummary* summ_prev,
                              const uint64_t* K, const uint32_t* P, float2* carry) {
  const int64_t L = a.L;
  const int64_t rows = a.B * a.n;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= rows * L) return;
  const int64_t row = g / L, i = g % L;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const uint64_t* Kr = K + row * L;
  const uint64_t k = Kr[i];
  if (k == 0xFFFFFFFFFFFFFFFFull || (i > 0 && Kr[i - 1] == k)) return;
  const float kappa = a.kappa[ni];
  bool seen = false;
  float lam = 0.f, alfa = 0.f;
  double bt = 0.0;
  for (int q = 0; q < n_prev; ++q) {
    const uint64_t* Kq = keys_prev + ((int64_t)q * rows + row) * L;
    const int64_t j = lower_u64(Kq, 0, L, k);
    if (j >= L || Kq[j] != k) continue;
    const NgcSummary r = summ_prev[((int64_t)q * rows + row) * L + j];
    if (seen) {
      const float a1 = expf(__fmul_rn(-kappa, __double2float_rn(fmax(r.b_first - bt, 0.0))));
      const float c = __fadd_rn(__fmul_rn(a1, lam), __fmul_rn(a1, alfa));
      lam = __fadd_rn(r.lam, __fmul_rn(r.prod, c));
    } else {
      lam = r.lam;
    }
    alfa = r.alfa;
    bt = r.b_last;
    seen = true;
  }
  float c = 0.f;
  if (seen) {
    const double b_first = a.Bt[b * a.Lf + P[row * L + i]];
    const float a1 = expf(__fmul_rn(-kappa, __double2float_rn(fmax(b_first - bt, 0.0))));
    c = __fadd_rn(__fmul_rn(a1, lam), __fmul_rn(a1, alfa));
  }
  carry[g] = make_float2(c, seen ? 1.f : 0.f);
}

// vistos / hawkes of every slot, scattered to the chunk's text order (B, Lc, n)
__global__ void k_ngc_final(RepetitionArgs a, const uint64_t* K, const uint32_t* P, const float2* lp,
                            const float2* carry) {
  const int64_t L = a.L;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= a.B * a.n * L) return;
  const int64_t row = g / L, i = g % L;
  const int64_t b = row / a.n;
  const int ni = (int)(row % a.n);
  const uint64_t* Kr = K + row * L;
  const uint64_t k = Kr[i];
  const int64_t t = (int64_t)P[g] - a.pos0;
  const float2 v = lp[g];
  float h = v.x;
  uint8_t vis = 0;
  if (k != 0xFFFFFFFFFFFFFFFFull) {
    const bool first = i == 0 || Kr[i - 1] != k;
    const int64_t f = first ? i : lower_u64(Kr, 0, i, k);
    const float2 cs = carry[row * L + f];
    h = __fadd_rn(v.x, __fmul_rn(v.y, cs.x));
    vis = first ? (cs.y != 0.f ? 1 : 0) : 1;
  }
  a.hawkes[(b * L + t) * a.n + ni] = h;
  a.vistos[(b * L + t) * a.n + ni] = vis;
}

int launch_ngram_chunk_sort(const RepetitionArgs& a, uint64_t* keys, void* summary, void* ws, size_t ws_bytes,
                            cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  if (a.n < 1 || a.n > kMaxSeen || a.pos0 + a.L > a.Lf || a.Lf >= ((int64_t)1 << 31)) return ASRN_ERR_ARG;
  if (!ws || ws_bytes < ngram_chunk_workspace(a.B, a.L, a.n)) return ASRN_ERR_WORKSPACE;
  const int64_t rows = a.B * a.n, L = a.L;
  const int64_t tiles = (L + kRepTile - 1) / kRepTile;
  const int64_t stiles = (L + kSortTile - 1) / kSortTile;
  NgcLayout r = ngc_layout(ws, rows, L);
  const size_t smem = (size_t)kSortTile * 12;
  cudaFuncSetAttribute(k_ngram_tile_sort, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  RepetitionArgs ak = a;
  ak.keys = nullptr;
  k_ngram_tile_sort<<<(unsigned)(rows * stiles), 1024, smem, s>>>(ak, stiles, r.k0, r.p0);
  uint64_t *kin = r.k0, *kout = r.k1;
  uint32_t *pin = r.p0, *pout = r.p1;
  const int64_t per_row = (L + kMergeItems - 1) / kMergeItems;
  for (int64_t w = kSortTile; w < L; w <<= 1) {
    k_ngram_merge<<<(unsigned)((rows * per_row + 255) / 256), 256, 0, s>>>(kin, pin, kout, pout, rows, L, w);
    uint64_t* tk = kin; kin = kout; kout = tk;
    uint32_t* tp = pin; pin = pout; pout = tp;
  }
  k_ngc_scan_tile<<<(unsigned)(rows * tiles), 1024, 0, s>>>(a, tiles, kin, pin, r.vloc, r.agg);
  k_ngc_apply<<<(unsigned)(rows * tiles), 1024, 0, s>>>(a, tiles, r.vloc, r.agg, r.lp, pin, r.pos);
  const unsigned gb = (unsigned)((rows * L + 255) / 256);
  k_ngc_summary<<<gb, 256, 0, s>>>(a, kin, r.pos, r.lp, keys, reinterpret_cast<NgcSummary*>(summary));
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_ngram_chunk_finish(const RepetitionArgs& a, int n_prev, const uint64_t* keys_prev, const void* summary_prev,
                              const uint64_t* keys, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  if (a.n < 1 || a.n > kMaxSeen || n_prev < 0 || a.pos0 + a.L > a.Lf) return ASRN_ERR_ARG;
  if (!ws || ws_bytes < ngram_chunk_workspace(a.B, a.L, a.n)) return ASRN_ERR_WORKSPACE;
  const int64_t rows = a.B * a.n, L = a.L;
  NgcLayout r = ngc_layout(ws, rows, L);
  const unsigned gb = (unsigned)((rows * L + 255) / 256);
  k_ngc_resolve<<<gb, 256, 0, s>>>(a, n_prev, keys_prev, reinterpret_cast<const NgcSummary*>(summary_prev), keys,
                                   r.pos, r.carry);
  k_ngc_final<<<gb, 256, 0, s>>>(a, keys, r.pos, r.lp, r.carry);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

size_t racha_workspace(int64_t B, int64_t L) {
  const int64_t tiles = (L + kRachaTile - 1) / kRachaTile;
  return align_up((size_t)B * L * 8) + align_up((size_t)B * tiles * 8);
}

// Streak of rows of L positions: one block per row, or (rows that are few and long, and a workspace given) the tiled
// scan over all SMs.
int launch_racha_ws(const RepetitionArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  const int64_t tiles = (a.L + kRachaTile - 1) / kRachaTile;
  if (ws && ws_bytes >= racha_workspace(a.B, a.L) && tiles >= 4 && a.B < 64) {
    float2* vloc = reinterpret_cast<float2*>(ws);
    float2* agg = reinterpret_cast<float2*>(reinterpret_cast<char*>(ws) + align_up((size_t)a.B * a.L * 8));
    k_racha_tile<<<(unsigned)(a.B * tiles), 1024, 0, s>>>(a, tiles, vloc, agg);
    k_racha_apply<<<(unsigned)(a.B * tiles), 1024, 0, s>>>(a, tiles, vloc, agg);
  } else {
    k_racha<<<(unsigned)a.B, 1024, 0, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_racha(const RepetitionArgs& a, cudaStream_t s) { return launch_racha_ws(a, nullptr, 0, s); }

int launch_repetition(const RepetitionArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  if (a.n < 1 || a.n > kMaxSeen) return ASRN_ERR_ARG;
  if (a.ng_mode != kNgFull && (!a.ng_keys || !a.ng_pos || a.pos0 != 0 || a.Lf != a.L)) return ASRN_ERR_ARG;
  if (rep_tiled(a.L)) {
    const int st = launch_repetition_long(a, ws, ws_bytes, s);
    if (st || a.ng_mode == kNgSortOnly) return st;
    return launch_racha_ws(a, ws, ws_bytes, s);   // the n-gram passes are done with the workspace
  }
  const int n2 = (int)((a.L + kRxThreads - 1) / kRxThreads * kRxThreads);
  const size_t smem = a.ng_mode == kNgScanOnly ? 0 : (size_t)n2 * 24 + kRxTabBytes;
  dim3 grid((unsigned)(a.B * a.n));
  const int items = n2 / 1024;
  if (items <= 1) {
    cudaFuncSetAttribute(k_ngram_row<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_row<1><<<grid, 1024, smem, s>>>(a, n2);
  } else if (items <= 2) {
    cudaFuncSetAttribute(k_ngram_row<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_row<2><<<grid, 1024, smem, s>>>(a, n2);
  } else if (items <= 4) {
    cudaFuncSetAttribute(k_ngram_row<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_row<4><<<grid, 1024, smem, s>>>(a, n2);
  } else if (items <= 8) {
    cudaFuncSetAttribute(k_ngram_row<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_row<8><<<grid, 1024, smem, s>>>(a, n2);
  } else {
    cudaFuncSetAttribute(k_ngram_row<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_ngram_row<16><<<grid, 1024, smem, s>>>(a, n2);
  }
  if (cudaGetLastError() != cudaSuccess) return ASRN_ERR_CUDA;
  if (a.ng_mode == kNgSortOnly) return ASRN_OK;
  k_racha<<<(unsigned)a.B, 1024, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

size_t ngram_shared_bytes(int64_t B, int64_t L, int n) {
  const size_t e = (size_t)B * n * L;
  return align_up(e * 8) + align_up(e * 4);
}

}  // namespace asrn
