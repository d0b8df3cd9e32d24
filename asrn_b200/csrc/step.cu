// Per-token kernels of the generation step for the stages whose whole-sequence kernels are tiled for long inputs
// (128-token tensor-core tiles, weights streamed through one tile): with one new token per sequence, B rows, those
// kernels run a handful of CTAs through the full weight matrices. These spread the weights over many CTAs instead.
//
// k_gen_front: one block per sequence computes, for its new token, the context stage (LN(h), Qc, Kc, the clock
//   projection -> beta / log_alfa, g(h), the signature) and the sign-hash projection (both MLP layers, the bucket ids),
//   with the rounding chains of k_context and k_hash_simt (asrn/estable.py:153-194, asrn/nucleo.py:639-664).
// The gate of the new tokens (k_gen_gate_tc) is in gate.cu, beside the gate's other kernels.
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {

constexpr int kFrontThreads = 256;

// sum_j x[j] * w[j] over a row of d, x in shared memory (fp32), w in global memory; 16-byte weight loads when the row
// is aligned. Result in every lane.
template <typename W>
__device__ __forceinline__ float dot_row(const float* x, const W* w, int d, int lane) {
  constexpr int VW = 16 / sizeof(W);
  float acc = 0.f;
  int j0 = 0;
  if (d % VW == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    const int nv = d / VW;
    for (int v = lane; v < nv; v += 32) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(w) + v);
      const float* xv = x + v * VW;
      if constexpr (sizeof(W) == 2) {
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(p[e]);
          acc = fmaf(xv[2 * e], f.x, acc);
          acc = fmaf(xv[2 * e + 1], f.y, acc);
        }
      } else {
        const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc = fmaf(xv[e], f[e], acc);
      }
    }
    j0 = d;
  }
  for (int j = j0 + lane; j < d; j += 32) {
    float wv;
    if constexpr (sizeof(W) == 2) wv = __bfloat162float(w[j]);
    else wv = w[j];
    acc = fmaf(x[j], wv, acc);
  }
  return warp_sum(acc);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

}  // namespace

template <bool Half>
__global__ void __launch_bounds__(kFrontThreads) k_gen_front(GenFrontArgs a) {
  using A = Act<Half>;
  using AT = typename A::T;
  extern __shared__ float sm[];
  const int d = a.d, cf = a.cf, m = a.m, P = a.P, nb = a.nb, T = a.T;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = kFrontThreads / 32;
  float* s_h = sm;                 // raw h row
  float* s_hn = s_h + d;           // LN(h), fp32
  float* s_hna = s_hn + d;         // act(LN(h))
  float* s_e = s_hna + d;          // act(E_t)
  float* s_p = s_e + d;            // act(E_{t-1})
  const int nq = 2 * cf + 3 + 3 * m;
  float* s_dot = s_p + d;          // nq dot products
  float* s_hid = s_dot + nq;       // 2m hidden (after GELU)
  float* s_phi = s_hid + 2 * m;    // P
  float* s_red = s_phi + P;        // 32

  const float* hrow = a.h + b * d;
  float s = 0.f;
  for (int j = tid; j < d; j += kFrontThreads) {
    const float x = hrow[j];
    s_h[j] = x;
    s += x;
    s_e[j] = act<Half>(a.e_t[b * d + j]);
    s_p[j] = act<Half>(a.e_prev[b * d + j]);
  }
  const float mean = block_sum(s, s_red) / (float)d;
  float v = 0.f;
  for (int j = tid; j < d; j += kFrontThreads) {
    const float c = s_h[j] - mean;
    v += c * c;
  }
  const float rstd = 1.f / sqrtf(block_sum(v, s_red) / (float)d + 1e-5f);
  for (int j = tid; j < d; j += kFrontThreads) {
    const float hn = (s_h[j] - mean) * rstd * a.ln_w[j] + a.ln_b[j];
    s_hn[j] = hn;
    s_hna[j] = act<Half>(hn);
  }
  __syncthreads();

  // dot products: [0, 2cf) Qc / Kc; 2cf, 2cf + 1 the clock projection; 2cf + 2 g(h); then the 3m hidden sums
  // hp = act(E_t) . pal0, ca = act(E_t) . ctx0[:, :d], cb = act(E_{t-1}) . ctx0[:, d:]
  const AT* wctx = reinterpret_cast<const AT*>(a.wctx);
  const AT* w1 = reinterpret_cast<const AT*>(a.w1);
  for (int q = wid; q < nq; q += nw) {
    float r;
    if (q < 2 * cf) r = dot_row(s_hna, wctx + (int64_t)q * d, d, lane);
    else if (q < 2 * cf + 2) r = dot_row(s_hn, a.w_reloj + (int64_t)(q - 2 * cf) * d, d, lane);
    else if (q == 2 * cf + 2) r = dot_row(s_h, a.g_w, d, lane);
    else {
      const int i = q - (2 * cf + 3);
      r = dot_row(i < 2 * m ? s_e : s_p, w1 + (int64_t)i * d, d, lane);
    }
    if (lane == 0) s_dot[q] = r;
  }
  __syncthreads();

  if (tid < 2 * cf) {
    AT* dst = reinterpret_cast<AT*>(tid < cf ? a.Qc : a.Kc);
    A::store(dst + b * cf + (tid < cf ? tid : tid - cf), s_dot[tid]);
  } else if (tid == 2 * cf) {
    const float u0 = s_dot[2 * cf] + a.b_reloj[0];
    const float u1 = s_dot[2 * cf + 1] + a.b_reloj[1];
    a.beta[b] = (double)fminf(softplus_t(u0), a.beta_max);
    a.log_alfa[b] = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
    a.glogit[b] = s_dot[2 * cf + 2] + a.g_b[0];
    a.sig[b] = (float)a.tokens[b];
  }
  const float* y = s_dot + 2 * cf + 3;
  for (int i = tid; i < m; i += kFrontThreads) {
    s_hid[i] = act<Half>(gelu_t(act<Half>(y[i] + a.b1[i])));
    s_hid[m + i] = act<Half>(gelu_t(act<Half>((y[m + i] + y[2 * m + i]) + a.b1[m + i])));
  }
  __syncthreads();
  const AT* w2 = reinterpret_cast<const AT*>(a.w2);
  AT* phi = reinterpret_cast<AT*>(a.phi);
  for (int o = wid; o < P; o += nw) {
    const float* src = (o / nb < a.Tw) ? s_hid : s_hid + m;
    float acc = 0.f;
    for (int i = lane; i < m; i += 32) acc = fmaf(src[i], A::load(w2 + (int64_t)o * m + i), acc);
    acc = warp_sum(acc);
    if (lane == 0) {
      const float val = act<Half>(acc + a.b2[o]);
      s_phi[o] = val;
      A::store(phi + b * P + o, val);
    }
  }
  __syncthreads();
  if (tid < T) {
    uint32_t id = 0;
    for (int j = 0; j < nb; ++j) id |= (s_phi[tid * nb + j] > 0.f ? 1u : 0u) << j;
    a.ids[b * T + tid] = (uint16_t)id;
  }
}

size_t gen_front_smem(const GenFrontArgs& a) {
  return sizeof(float) * (5 * (size_t)a.d + (2 * a.cf + 3 + 3 * a.m) + 2 * a.m + a.P + 32);
}

int launch_gen_front(const GenFrontArgs& a, bool half, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  const size_t smem = gen_front_smem(a);
  if (smem > 200 * 1024) return ASRN_ERR_UNSUPPORTED;
  if (half) {
    cudaFuncSetAttribute(k_gen_front<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_gen_front<true><<<(unsigned)a.B, kFrontThreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(k_gen_front<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_gen_front<false><<<(unsigned)a.B, kFrontThreads, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
