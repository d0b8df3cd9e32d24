// Gate and output projection. Reference: CapaASRNEstable._combinar (asrn/estable.py:376-403), _senales
// (asrn/estable.py:294-300) and _respuesta_racha (asrn/nucleo.py:865-878):
//   pt = tables with candidates; mejor = max over those tables of their best score (else 0), clamped to +-mejor_max
//   logit = g(h) + g_conf([pt/T, mejor, pico/max(1,pt), pt_ctx/Tc]) + w_vistos . vistos + u_hawkes . log1p(hawkes)
//           + response(racha)                                     (all fp32; g_conf in bf16 under autocast)
//   h' = h + sigmoid(logit) * o(salida / max(1, pt))
// Here salida = W_v acc (acc = sum of att * Ea rows from the scoring kernel), so o(salida) = (W_o W_v) acc and the
// projection is one GEMM against the prepared W_ov.
#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kGateTM = 64, kGateTN = 64, kGateKC = 32;

// Gate of one token (sigmoid(logit), rounded to the compute type) and max(1, pt).
template <bool Half>
__device__ __forceinline__ void gate_of_token(const GateArgs& a, int64_t g, float* sigma, float* ptc) {
  const int T = a.T;
  float pt = 0.f, mejor = kProhibido, pico = 0.f, pctx = 0.f;
  for (int tau = 0; tau < T; ++tau) {
    const float hay = (float)a.sen_hay[g * T + tau];
    pt = __fadd_rn(pt, hay);
    if (hay > 0.f) mejor = fmaxf(mejor, a.sen_mx[g * T + tau]);
    pico = __fadd_rn(pico, __fmul_rn(a.sen_pk[g * T + tau], hay));
    if (tau >= T - a.Tc) pctx = __fadd_rn(pctx, hay);
  }
  mejor = fmaxf(mejor, kProhibido);
  mejor = (pt > 0.f) ? mejor : 0.f;
  mejor = fminf(fmaxf(mejor, -a.mejor_max), a.mejor_max);
  const float pt1 = fmaxf(pt, 1.f);
  float s[4] = {__fdiv_rn(pt, (float)T), mejor, __fdiv_rn(pico, pt1), __fdiv_rn(pctx, (float)a.Tc)};
  float gc = 0.f;
  for (int i = 0; i < 4; ++i) gc = fmaf(act<Half>(s[i]), a.gconf[i], gc);
  gc = act<Half>(__fadd_rn(gc, a.gconf[4]));
  float logit = __fadd_rn(a.glogit[g], gc);
  float sv = 0.f;
  for (int j = 0; j < a.n; ++j) sv = __fadd_rn(sv, __fmul_rn((float)a.vistos[g * a.n + j], a.w_vistos[j]));
  logit = __fadd_rn(logit, sv);
  float sh = 0.f;
  for (int j = 0; j < a.n; ++j) sh = __fadd_rn(sh, __fmul_rn(log1pf(a.hawkes[g * a.n + j]), a.u_hawkes[j]));
  logit = __fadd_rn(logit, sh);
  // response to the streak: linear interpolation of u_racha on x = log1p(racha) / paso, flat past the last node
  float x = __fdiv_rn(log1pf(a.racha[g]), a.racha_paso);
  x = fminf(x, (float)(a.nodes - 1));
  const float xf = (x != x) ? 0.f : x;
  int i = (int)floorf(xf);
  i = min(max(i, 0), a.nodes - 2);
  const float resp = __fadd_rn(a.u_racha[i], __fmul_rn(__fsub_rn(x, (float)i), a.d_racha[i + 1]));
  logit = __fadd_rn(logit, resp);
  if (a.tope > 0.f) logit = __fmul_rn(a.tope, tanhf(__fdiv_rn(logit, a.tope)));
  *sigma = act<Half>(1.f / (1.f + expf(-logit)));
  *ptc = pt1;
}

template <bool Half>
__global__ void __launch_bounds__(256) k_gate_simt(GateArgs a) {
  using A = Act<Half>;
  __shared__ float s_sigma[kGateTM], s_pt[kGateTM];
  __shared__ __align__(16) float As[kGateKC][kGateTM];
  __shared__ __align__(16) float Bs[kGateKC][kGateTN];
  const int64_t M = a.B * a.L;
  const int d = a.d;
  const int64_t t0 = (int64_t)blockIdx.y * kGateTM;
  const int n0 = blockIdx.x * kGateTN;
  const int tid = threadIdx.x;
  for (int r = tid; r < kGateTM; r += blockDim.x) {
    const int64_t g = t0 + r;
    float sg = 0.f, pt = 1.f;
    if (g < M) gate_of_token<Half>(a, g, &sg, &pt);
    s_sigma[r] = sg;
    s_pt[r] = pt;
  }
  __syncthreads();
  const int tr = tid >> 4, tc = tid & 15;
  float acc[4][4] = {};
  const typename A::T* W = reinterpret_cast<const typename A::T*>(a.wov);
  for (int k0 = 0; k0 < d; k0 += kGateKC) {
    for (int e = tid; e < kGateTM * kGateKC; e += blockDim.x) {
      const int r = e / kGateKC, kk = e % kGateKC;
      const int64_t g = t0 + r;
      const int k = k0 + kk;
      As[kk][r] = (g < M && k < d) ? act<Half>(__fdiv_rn(a.acc[g * d + k], s_pt[r])) : 0.f;
    }
    for (int e = tid; e < kGateTN * kGateKC; e += blockDim.x) {
      const int c = e / kGateKC, kk = e % kGateKC;
      const int k = k0 + kk;
      Bs[kk][c] = (n0 + c < d && k < d) ? A::load(W + (int64_t)(n0 + c) * d + k) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGateKC; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&As[kk][tr * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tc * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w}, br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tr * 4 + i;
    const int64_t g = t0 + r;
    if (g >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tc * 4 + j;
      if (c >= d) continue;
      const float o = act<Half>(acc[i][j]);
      const float add = act<Half>(__fmul_rn(s_sigma[r], o));
      a.out[g * d + c] = __fadd_rn(a.h[g * d + c], add);
    }
  }
}

int launch_gate(const GateArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  dim3 grid((unsigned)((a.d + kGateTN - 1) / kGateTN), (unsigned)((M + kGateTM - 1) / kGateTM));
  if (half)
    k_gate_simt<true><<<grid, 256, 0, s>>>(a);
  else
    k_gate_simt<false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
