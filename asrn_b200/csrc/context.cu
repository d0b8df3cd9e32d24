// Context stage: LN(h) -> Qc, Kc, beta, log_alfa; g(h); token signatures; and the fp64 clock Bt = cumsum(beta).
// Reference: CapaASRNEstable._contexto (asrn/estable.py:153-194), firmas_de_piezas (asrn/nucleo.py:161-164),
// CapaASRN._firma (asrn/nucleo.py:634-637), the clock Bt = beta.cumsum(1) (asrn/estable.py:418) and the gate's
// g(h) term computed in the precision of h (asrn/estable.py:393-394).
#include "common.cuh"
#include "layout.h"

namespace asrn {

// One warp per token. Each lane owns the elements j = lane + 32 i of the row (coalesced across the warp).
template <bool Half>
__global__ void __launch_bounds__(256) k_context(ContextArgs a) {
  using A = Act<Half>;
  const int64_t M = a.B * a.L;
  const int d = a.d, cf = a.cf;
  const int lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= M) return;
  const float* hrow = a.h + tok * d;
  constexpr int kMaxPer = 32;  // d <= 1024
  float x[kMaxPer];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int j = lane + 32 * i;
    x[i] = (j < d) ? hrow[j] : 0.f;
    s += x[i];
  }
  const float mean = warp_sum(s) / (float)d;
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int j = lane + 32 * i;
    float c = (j < d) ? x[i] - mean : 0.f;
    v += c * c;
  }
  const float rstd = 1.f / sqrtf(warp_sum(v) / (float)d + 1e-5f);
  // g(h): raw h, fp32 (asrn/estable.py:393-394)
  float gl = 0.f;
  float hn[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int j = lane + 32 * i;
    if (j < d) {
      gl += x[i] * a.g_w[j];
      hn[i] = (x[i] - mean) * rstd * a.ln_w[j] + a.ln_b[j];
    } else {
      hn[i] = 0.f;
    }
  }
  gl = warp_sum(gl);
  // clock projection u = LN(h) . w_reloj + b_reloj in true fp32 (asrn/estable.py:171-185)
  float u0 = 0.f, u1 = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    int j = lane + 32 * i;
    if (j < d) {
      u0 += hn[i] * a.w_reloj[j];
      u1 += hn[i] * a.w_reloj[d + j];
    }
  }
  u0 = warp_sum(u0) + a.b_reloj[0];
  u1 = warp_sum(u1) + a.b_reloj[1];
  // Qc, Kc = LN(h)_act . [cq; ck]^T (act: bf16 inputs and output under autocast)
  const typename A::T* W = reinterpret_cast<const typename A::T*>(a.wctx);
  for (int o = 0; o < 2 * cf; ++o) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      int j = lane + 32 * i;
      if (j < d) acc += act<Half>(hn[i]) * A::load(W + (int64_t)o * d + j);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      typename A::T* dst = reinterpret_cast<typename A::T*>(o < cf ? a.Qc : a.Kc);
      A::store(dst + tok * cf + (o < cf ? o : o - cf), acc);
    }
  }
  // signature: token id as fp32, or E . r_firma (fp32) when no ids are given
  float sig;
  if (a.tokens) {
    sig = (float)a.tokens[tok];
  } else {
    float e = 0.f;
    const float* erow = a.E + tok * d;
    for (int j = lane; j < d; j += 32) e += erow[j] * a.r_firma[j];
    sig = warp_sum(e);
  }
  if (lane == 0) {
    float beta = fminf(softplus_t(u0), a.beta_max);
    float la = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
    a.beta[tok] = (double)beta;
    a.log_alfa[tok] = la;
    a.glogit[tok] = gl + a.g_b[0];
    a.sig[tok] = sig;
  }
}

// Inclusive fp64 prefix sum along L (the clock B_t = cumsum(beta), asrn/estable.py:418). Block (c, b) owns chunk c
// of row b (kClockChunk slots): it first sums every beta before its chunk itself (a block-wide fp64 reduction; the
// reads of all blocks add up to about L^2 / (2 kClockChunk) values per row, a few tens of MB at L = 262,144), then
// scans its chunk (4 slots per thread) on top of that sum. No block waits for another and no workspace is needed; a
// long row is spread over L / kClockChunk blocks instead of one block walking the whole row.
constexpr int kClockItems = 4;
constexpr int kClockChunk = 1024 * kClockItems;

__global__ void __launch_bounds__(1024) k_clock(const double* __restrict__ beta, double* __restrict__ Bt, int64_t L) {
  const int64_t b = blockIdx.y, c0 = (int64_t)blockIdx.x * kClockChunk;
  const double* src = beta + b * L;
  double* dst = Bt + b * L;
  __shared__ double warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // the sum of the row before this chunk
  double pre = 0.0;
  for (int64_t i = tid; i < c0; i += 1024) pre += src[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
  if (lane == 0) warp_tot[wid] = pre;
  __syncthreads();
  double carry = 0.0;
  for (int w = 0; w < 32; ++w) carry += warp_tot[w];
  __syncthreads();
  // the chunk: per-thread runs, a warp scan of the run totals, a block scan of the warp totals
  double v[kClockItems];
  double run = 0.0;
#pragma unroll
  for (int k = 0; k < kClockItems; ++k) {
    const int64_t i = c0 + (int64_t)tid * kClockItems + k;
    run += (i < L) ? src[i] : 0.0;
    v[k] = run;
  }
  double t = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, t, o);
    if (lane >= o) t += y;
  }
  if (lane == 31) warp_tot[wid] = t;
  __syncthreads();
  if (wid == 0) {
    double w = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;
  }
  __syncthreads();
  const double excl = carry + (wid > 0 ? warp_tot[wid - 1] : 0.0) + (t - run);
#pragma unroll
  for (int k = 0; k < kClockItems; ++k) {
    const int64_t i = c0 + (int64_t)tid * kClockItems + k;
    if (i < L) dst[i] = excl + v[k];
  }
}

bool context_tc_supported(const ContextArgs& a);
int launch_context_tc(const ContextArgs& a, int* status, cudaStream_t s);

int launch_context(const ContextArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  if (half && tensor_cores_enabled() && context_tc_supported(a)) return launch_context_tc(a, a.status, s);
  const int warps = 8;
  dim3 grid((unsigned)((M + warps - 1) / warps));
  if (half)
    k_context<true><<<grid, warps * 32, 0, s>>>(a);
  else
    k_context<false><<<grid, warps * 32, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_clock(const double* beta, double* Bt, int64_t B, int64_t L, cudaStream_t s) {
  if (B == 0 || L == 0) return ASRN_OK;
  for (int64_t b0 = 0; b0 < B; b0 += 65535) {          // grid.y holds at most 65535 rows
    const dim3 grid((unsigned)((L + kClockChunk - 1) / kClockChunk), (unsigned)(B - b0 < 65535 ? B - b0 : 65535));
    k_clock<<<grid, 1024, 0, s>>>(beta + b0 * L, Bt + b0 * L, L);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
