// Derived weights of a layer, computed on the device from the reference's parameters:
//   [cq; ck], [pal0; ctx0[:, :d]; ctx0[:, d:]], [pal2; ctx2] in the compute type (bf16 under autocast, which rounds
//   weights and biases of every F.linear), W_ov = W_o @ W_v (fp32 product, then the compute type),
//   tasa = gamma / C (asrn/estable.py:253), kappa = exp(log_kappa) floored by kappa_min (asrn/estable.py:196-200),
//   u_racha = cumsum(d_racha) (asrn/nucleo.py:865-868).
#include "common.cuh"
#include "layout.h"

namespace asrn {

template <bool Half>
__global__ void k_copy_rows(const float* __restrict__ src, int64_t src_stride, int64_t col0, int64_t rows,
                            int64_t cols, void* dst_v, int64_t dst_row0) {
  using A = Act<Half>;
  typename A::T* dst = reinterpret_cast<typename A::T*>(dst_v);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  A::store(dst + (dst_row0 + r) * cols + c, src[r * src_stride + col0 + c]);
}

__global__ void k_round_vec(const float* __restrict__ src, float* __restrict__ dst, int n, int half) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = half ? round_bf16(src[i]) : src[i];
}

// W_ov[i][j] = sum_k W_o[i][k] W_v[k][j], fp32, 32x32 tiles.
template <bool Half>
__global__ void k_wov(const float* __restrict__ Wo, const float* __restrict__ Wv, int d, void* dst_v) {
  using A = Act<Half>;
  __shared__ float sa[32][33], sb[32][33];
  const int i = blockIdx.y * 32 + threadIdx.y, j = blockIdx.x * 32 + threadIdx.x;
  float acc = 0.f;
  for (int k0 = 0; k0 < d; k0 += 32) {
    const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    sa[threadIdx.y][threadIdx.x] = (i < d && ka < d) ? Wo[(int64_t)i * d + ka] : 0.f;
    sb[threadIdx.y][threadIdx.x] = (kb < d && j < d) ? Wv[(int64_t)kb * d + j] : 0.f;
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < 32; ++k) acc = fmaf(sa[threadIdx.y][k], sb[k][threadIdx.x], acc);
    __syncthreads();
  }
  if (i < d && j < d) A::store(reinterpret_cast<typename A::T*>(dst_v) + (int64_t)i * d + j, acc);
}

__global__ void k_scalars(asrn_layer_config c, const float* gamma, const float* log_kappa, const float* log_kappa_r,
                          const float* d_racha, const float* gconf_w, const float* gconf_b, float* tasa,
                          float* kappa, float* u_racha, float* gconf) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int t = 0; t < c.n_tablas; ++t) tasa[t] = __fdiv_rn(gamma[t], (float)c.chunk);
  for (int j = 0; j < c.vistos; ++j) {
    float k = expf(log_kappa[j]);
    if (c.kappa_min > 0.f) k = fmaxf(k, c.kappa_min);
    kappa[j] = k;
  }
  float kr = expf(log_kappa_r[0]);
  if (c.kappa_min > 0.f) kr = fmaxf(kr, c.kappa_min);
  kappa[c.vistos] = kr;
  float s = 0.f;
  for (int j = 0; j < c.nodos_racha; ++j) {
    s = __fadd_rn(s, d_racha[j]);
    u_racha[j] = s;
  }
  for (int j = 0; j < 4; ++j) gconf[j] = c.half ? round_bf16(gconf_w[j]) : gconf_w[j];
  gconf[4] = c.half ? round_bf16(gconf_b[0]) : gconf_b[0];
}

// Block-diagonal second hash layer in bf16: row o < Pw holds pal2[o] in K [0, m); row Pw <= o < P holds
// ctx2[o - Pw] in K [m, 2m); everything else is 0 (products with 0 add exact zeros to the fp32 accumulator).
__global__ void k_w2bd(const float* __restrict__ pal2, const float* __restrict__ ctx2, int Pw, int P, int Np, int m,
                       __nv_bfloat16* __restrict__ dst) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= Np * 2 * m) return;
  const int o = i / (2 * m), k = i % (2 * m);
  float v = 0.f;
  if (o < Pw && k < m) v = pal2[o * m + k];
  else if (o >= Pw && o < P && k >= m) v = ctx2[(o - Pw) * m + (k - m)];
  dst[i] = __float2bfloat16_rn(v);
}

template <bool Half>
static void copy_rows(const float* src, int64_t stride, int64_t col0, int64_t rows, int64_t cols, void* dst,
                      int64_t row0, cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n == 0) return;
  k_copy_rows<Half><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, stride, col0, rows, cols, dst, row0);
}

template <bool Half>
static void prepare_t(const asrn_layer_config& c, const asrn_layer_weights& w, char* base, cudaStream_t s) {
  const PreparedLayout L = prepared_layout(c);
  const int64_t d = c.d, m = c.hidden, cf = c.confirmar, nb = c.n_bits;
  const int64_t Pw = (int64_t)(c.n_tablas - c.tablas_contexto) * nb, Pc = (int64_t)c.tablas_contexto * nb;
  copy_rows<Half>(w.cq, d, 0, cf, d, base + L.wctx, 0, s);
  copy_rows<Half>(w.ck, d, 0, cf, d, base + L.wctx, cf, s);
  copy_rows<Half>(w.pal0_w, d, 0, m, d, base + L.w1, 0, s);
  copy_rows<Half>(w.ctx0_w, 2 * d, 0, m, d, base + L.w1, m, s);
  copy_rows<Half>(w.ctx0_w, 2 * d, d, m, d, base + L.w1, 2 * m, s);
  copy_rows<Half>(w.pal2_w, m, 0, Pw, m, base + L.w2, 0, s);
  copy_rows<Half>(w.ctx2_w, m, 0, Pc, m, base + L.w2, Pw, s);
  float* b1 = reinterpret_cast<float*>(base + L.b1);
  float* b2 = reinterpret_cast<float*>(base + L.b2);
  k_round_vec<<<(unsigned)((m + 255) / 256), 256, 0, s>>>(w.pal0_b, b1, (int)m, Half);
  k_round_vec<<<(unsigned)((m + 255) / 256), 256, 0, s>>>(w.ctx0_b, b1 + m, (int)m, Half);
  k_round_vec<<<(unsigned)((Pw + 255) / 256), 256, 0, s>>>(w.pal2_b, b2, (int)Pw, Half);
  k_round_vec<<<(unsigned)((Pc + 255) / 256), 256, 0, s>>>(w.ctx2_b, b2 + Pw, (int)Pc, Half);
  const int P = (int)(Pw + Pc), Np = (P + 15) / 16 * 16;
  k_w2bd<<<(unsigned)((Np * 2 * m + 255) / 256), 256, 0, s>>>(w.pal2_w, w.ctx2_w, (int)Pw, P, Np, (int)m,
                                                             reinterpret_cast<__nv_bfloat16*>(base + L.w2bd));
  cudaMemsetAsync(base + L.status, 0, 4, s);
  dim3 g((unsigned)((d + 31) / 32), (unsigned)((d + 31) / 32));
  k_wov<Half><<<g, dim3(32, 32), 0, s>>>(w.o_w, w.v_w, (int)d, base + L.wov);
  k_scalars<<<1, 32, 0, s>>>(c, w.gamma, w.log_kappa, w.log_kappa_racha, w.d_racha, w.g_conf_w, w.g_conf_b,
                             reinterpret_cast<float*>(base + L.tasa), reinterpret_cast<float*>(base + L.kappa),
                             reinterpret_cast<float*>(base + L.u_racha), reinterpret_cast<float*>(base + L.gconf));
}

int launch_prepare(const asrn_layer_config& c, const asrn_layer_weights& w, void* prepared, cudaStream_t s) {
  if (c.half)
    prepare_t<true>(c, w, reinterpret_cast<char*>(prepared), s);
  else
    prepare_t<false>(c, w, reinterpret_cast<char*>(prepared), s);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
