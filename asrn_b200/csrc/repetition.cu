// Repetition memory: "seen" flags, Hawkes intensity per n-gram order, and the repetition streak.
// Reference: CapaASRNEstable._repeticion (asrn/estable.py:304-321) with _claves_de (asrn/nucleo.py:175-185),
// _ordenar_claves (asrn/nucleo.py:693-701) and escaneo (asrn/nucleo.py:188-257):
//   key_n(t) = ((0 + s_t c_0) + s_{t-1} c_1) + ... + s_{t-n} c_n   in fp64, this order, no FMA; NaN before the start
//   per (b, n): stable sort by key (NaN last); repetido_i = key_i == key_{i-1}
//   a_i = repetido_i * exp(-kappa_n * float(max(0, B_i - B_{i-1}))),  lambda_i = a_i (lambda_{i-1} + alfa_{i-1})
//   hawkes / vistos scattered back to text order; streak S_t = r_t exp(-kappa_r beta_t) S_{t-1} + r_t with
//   r_t = vistos of the longest order.
// One block per (b, n) row sorts (key, position) pairs in shared memory with a bitonic network, then runs a
// block-wide scan of affine maps over the sorted row.
#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kRepMaxL = 16384;   // rows sorted in one block (16384 x 12 B of shared memory)

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

template <int kItems>
__global__ void __launch_bounds__(1024) k_ngram_row(RepetitionArgs a, int n2) {
  extern __shared__ __align__(16) char smem_raw[];
  uint64_t* sk = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* sp = reinterpret_cast<uint32_t*>(sk + n2);
  __shared__ Affine warp_agg[32];
  const int64_t b = blockIdx.x / a.n;
  const int ni = (int)(blockIdx.x % a.n);
  const int64_t L = a.L;
  const float* sig = a.sig + b * L;
  // keys of the (ni + 1)-token groups ending at t (asrn/nucleo.py:175-185)
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    if (i < L) {
      double key = 0.0;
      for (int j = 0; j <= ni; ++j) {
        const int64_t t = i - j;
        const double s = (t >= 0) ? (double)sig[t] : __longlong_as_double(0x7ff8000000000000ll);
        key = __dadd_rn(key, __dmul_rn(s, a.c[j]));
      }
      if (a.keys) a.keys[(b * L + i) * a.n + ni] = key;
      sk[i] = sortable_key(key);
      sp[i] = (uint32_t)i;
    } else {
      sk[i] = 0xFFFFFFFFFFFFFFFFull;
      sp[i] = 0xFFFFFFFFu;
    }
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
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
  if (threadIdx.x == 0) carry_s = Affine{1.f, 0.f};
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
      if (t < L) a.racha[b * L + t] = s.b;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry_s = compose(carry, v[kItems - 1]);
    __syncthreads();
  }
}

size_t repetition_workspace(int64_t, int64_t, int) { return 0; }

int launch_repetition(const RepetitionArgs& a, void*, size_t, cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  if (a.n < 1 || a.n > kMaxSeen) return ASRN_ERR_ARG;
  if (a.L > kRepMaxL) return ASRN_ERR_UNSUPPORTED;
  int n2 = 1;
  while (n2 < a.L) n2 <<= 1;
  const size_t smem = (size_t)n2 * 12;
  dim3 grid((unsigned)(a.B * a.n));
  const int items = (n2 + 1023) / 1024;
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
  k_racha<<<(unsigned)a.B, 1024, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
