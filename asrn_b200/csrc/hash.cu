// Sign-hash projection: E -> phi (T tables x nb bits) and the bucket id of every (token, table).
// Reference: CapaASRN._phi_y_valores / _phi / _ids (asrn/nucleo.py:639-664):
//   hp = E . pal0^T + b ; phi_word = pal2(GELU(hp))                       (tables 0 .. T-Tc-1)
//   c0 = [E_t, E_{t-1}] . ctx0^T + b ; phi_ctx = ctx2(GELU(c0))            (tables T-Tc .. T-1, E_{-1} = 0)
//   id_tau = sum_j 2^j [phi[tau * nb + j] > 0]
// The value projection v(E_{t+1}) of the reference is not computed here: the scoring kernel gathers rows of Ea
// (E in the compute type) and the gate applies W_o W_v to their weighted sum.
// The context projection is split as c0(t) = E_t . ctx0[:, :d]^T + E_{t-1} . ctx0[:, d:]^T + b, both halves
// accumulated in fp32 before the (bf16) rounding, so the rounding chain matches the reference's single product.
#include <cuda.h>

#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kHashTM = 32;   // tokens per block
constexpr int kHashKC = 32;   // k chunk

template <bool Half>
__global__ void __launch_bounds__(256) k_hash_simt(HashArgs a) {
  using A = Act<Half>;
  extern __shared__ float smem[];
  const int m = a.m, d = a.d, P = a.P, nb = a.nb, T = a.T, Tw = a.Tw;
  const int N = 3 * m;
  const int64_t M = a.B * a.L;
  const int64_t g0 = (int64_t)blockIdx.x * kHashTM;
  float* As = smem;                                   // [KC][TM + 1]
  float* Bs = As + kHashKC * (kHashTM + 1);           // [KC][N]  (reused as Y[TM][N])
  float* G = Bs + kHashKC * N;                        // per warp: [2m] gelu outputs + [P] phi row
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int rg = tid >> 5;      // rows rg*4 .. rg*4+3
  const int cl = tid & 31;      // cols cl + 32 j
  const int ncj = (N + 31) / 32;
  float acc[4][12];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < 12; ++j) acc[r][j] = 0.f;

  const typename A::T* W1 = reinterpret_cast<const typename A::T*>(a.w1);
  typename A::T* Ea = reinterpret_cast<typename A::T*>(a.Ea);
  for (int k0 = 0; k0 < d; k0 += kHashKC) {
    for (int e = tid; e < (kHashTM + 1) * kHashKC; e += blockDim.x) {
      const int r = e / kHashKC, kk = e % kHashKC;
      const int64_t gr = g0 - 1 + r;
      const int k = k0 + kk;
      float v = 0.f;
      if (gr >= 0 && gr < M && k < d) {
        const float x = a.E[gr * d + k];
        v = act<Half>(x);
        if (Half && r >= 1) A::store(Ea + gr * d + k, x);
      }
      As[kk * (kHashTM + 1) + r] = v;
    }
    for (int e = tid; e < N * kHashKC; e += blockDim.x) {
      const int c = e / kHashKC, kk = e % kHashKC;
      const int k = k0 + kk;
      Bs[kk * N + c] = (k < d) ? A::load(W1 + (int64_t)c * d + k) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kHashKC; ++kk) {
      float ar[5];
#pragma unroll
      for (int r = 0; r < 5; ++r) ar[r] = As[kk * (kHashTM + 1) + rg * 4 + r];
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        const int c = cl + 32 * j;
        if (j < ncj && c < N) {
          const float bv = Bs[kk * N + c];
          const int sh = (c < 2 * m) ? 1 : 0;    // hp / ca use the token's row, cb the previous row
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[r][j] += ar[r + sh] * bv;
        }
      }
    }
    __syncthreads();
  }
  float* Y = Bs;  // [TM][N]
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < 12; ++j) {
      const int c = cl + 32 * j;
      if (j < ncj && c < N) Y[(rg * 4 + r) * N + c] = acc[r][j];
    }
  __syncthreads();

  float* g1 = G + wid * (2 * m + P);
  float* g2 = g1 + m;
  float* prow = g2 + m;
  const typename A::T* W2 = reinterpret_cast<const typename A::T*>(a.w2);
  typename A::T* phi = reinterpret_cast<typename A::T*>(a.phi);
  for (int r = wid; r < kHashTM; r += 8) {
    const int64_t g = g0 + r;
    if (g >= M) break;
    const int64_t t = g % a.L, b = g / a.L;
    const float* y = Y + r * N;
    for (int i = lane; i < m; i += 32) {
      const float hp = act<Half>(y[i] + a.b1[i]);
      g1[i] = act<Half>(gelu_t(hp));
      const float prev = (t > 0) ? y[2 * m + i] : 0.f;
      const float c0 = act<Half>((y[m + i] + prev) + a.b1[m + i]);
      g2[i] = act<Half>(gelu_t(c0));
    }
    __syncwarp();
    for (int o = lane; o < P; o += 32) {
      const float* src = (o / nb < Tw) ? g1 : g2;
      const typename A::T* wr = W2 + (int64_t)o * m;
      float s = 0.f;
      for (int i = 0; i < m; ++i) s += src[i] * A::load(wr + i);
      const float v = act<Half>(s + a.b2[o]);
      prow[o] = v;
      A::store(phi + g * P + o, v);
    }
    __syncwarp();
    if (lane < T) {
      uint32_t id = 0;
      for (int j = 0; j < nb; ++j) id |= (prow[lane * nb + j] > 0.f ? 1u : 0u) << j;
      a.ids_rows[((int64_t)b * T + lane) * a.L + t] = (uint16_t)id;
    }
    __syncwarp();
  }
}

__global__ void k_ids_from_phi(int64_t B, int64_t L, int T, int nb, const float* __restrict__ phi,
                               uint16_t* __restrict__ ids_rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (b, t, tau)
  if (i >= B * L * T) return;
  const int tau = (int)(i % T);
  const int64_t g = i / T;
  const int64_t b = g / L, t = g % L;
  const float* p = phi + g * (int64_t)T * nb + (int64_t)tau * nb;
  uint32_t id = 0;
  for (int j = 0; j < nb; ++j) id |= (p[j] > 0.f ? 1u : 0u) << j;
  ids_rows[(b * T + tau) * L + t] = (uint16_t)id;
}

bool hash_tc_supported(const HashArgs& a);
int launch_hash_tc(const HashArgs& a, const CUtensorMap& w1, const CUtensorMap& w2, cudaStream_t s);

int launch_hash(const HashArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  if (half && tensor_cores_enabled() && hash_tc_supported(a)) {
    CUtensorMap w1, w2;
    const int Np = (a.P + 15) / 16 * 16;
    if (!make_tmap_bf16(&w1, a.w1, (uint64_t)a.d, (uint64_t)(3 * a.m), (uint64_t)a.d * 2, 64, (uint32_t)(3 * a.m)) ||
        !make_tmap_bf16(&w2, a.w2bd, (uint64_t)(2 * a.m), (uint64_t)Np, (uint64_t)(2 * a.m) * 2, 64, (uint32_t)Np))
      return ASRN_ERR_CUDA;
    return launch_hash_tc(a, w1, w2, s);
  }
  if (3 * a.m > 384) return ASRN_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * ((size_t)kHashKC * (kHashTM + 1) + (size_t)kHashKC * 3 * a.m +
                                       8 * (size_t)(2 * a.m + a.P));
  dim3 grid((unsigned)((M + kHashTM - 1) / kHashTM));
  if (half) {
    cudaFuncSetAttribute(k_hash_simt<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_hash_simt<true><<<grid, 256, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(k_hash_simt<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_hash_simt<false><<<grid, 256, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_ids_from_phi(int64_t B, int64_t L, int T, int nb, const float* phi, uint16_t* ids_rows, cudaStream_t s) {
  const int64_t n = B * L * T;
  if (n == 0) return ASRN_OK;
  k_ids_from_phi<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(B, L, T, nb, phi, ids_rows);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
