// Element-wise parts of one generation step of the model's local blocks (asrn/nucleo.py:969-1014, the O(1) writer's
// conv buffer asrn/nucleo.py:1816-1822), one block per sequence row, fused around the block's three GEMMs:
//   k_local_in   h = h_prev (+ y_prev, the previous block's MLP output), LN1(h) in fp32, rounded to the compute
//                type and pushed into the row's conv window (B, k, d) (the k - 1 previous rows shift down in place);
//                with no window (k == 0) it is the final LN before the head
//   k_local_mid  h1 = h + act(gelu(z)) (z: the conv output), LN2(h1) rounded to the compute type
//   k_local_gelu f = act(gelu(f)) in place (the MLP's hidden layer)
// The compute type is bf16 under autocast (half = 1) or fp32; residual sums are fp32 (torch's promotion of
// fp32 + bf16). LayerNorm: biased variance, 1 / sqrt(var + eps), as torch.nn.functional.layer_norm.
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {
constexpr int kLocalThreads = 256;

__device__ __forceinline__ float block_sum_local(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < kLocalThreads / 32; ++i) s += red[i];
  return s;
}

template <bool Half>
__device__ __forceinline__ float load_act(const void* p, int64_t i) {
  return Half ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}
template <bool Half>
__device__ __forceinline__ void store_act(void* p, int64_t i, float v) {
  if (Half) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// LayerNorm of the row held in s_x (d values) -> out (compute type) at out + row offset
template <bool Half>
__device__ __forceinline__ void row_layer_norm(const float* s_x, int d, const float* w, const float* b, float eps,
                                               float* red, float* out_f) {
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += kLocalThreads) s += s_x[j];
  const float mean = block_sum_local(s, red) / (float)d;
  float v = 0.f;
  for (int j = threadIdx.x; j < d; j += kLocalThreads) {
    const float c = s_x[j] - mean;
    v += c * c;
  }
  const float rstd = 1.f / sqrtf(block_sum_local(v, red) / (float)d + eps);
  for (int j = threadIdx.x; j < d; j += kLocalThreads) out_f[j] = act<Half>((s_x[j] - mean) * rstd * w[j] + b[j]);
}
}  // namespace

template <bool Half>
__global__ void __launch_bounds__(kLocalThreads) k_local_in(int d, int k, const float* h_prev, const void* y_prev,
                                                            float* h_out, const float* ln_w, const float* ln_b,
                                                            float eps, void* win) {
  extern __shared__ float s_loc[];
  float* s_x = s_loc;
  float* s_u = s_loc + d;
  float* red = s_loc + 2 * d;
  const int64_t b = blockIdx.x;
  for (int j = threadIdx.x; j < d; j += kLocalThreads) {
    float x = h_prev[b * d + j];
    if (y_prev) x = __fadd_rn(x, load_act<Half>(y_prev, b * d + j));
    s_x[j] = x;
    if (h_out) h_out[b * d + j] = x;
  }
  __syncthreads();
  row_layer_norm<Half>(s_x, d, ln_w, ln_b, eps, red, s_u);
  // window (B, k, d): rows 0 .. k-2 take rows 1 .. k-1, row k-1 the new LN output (each thread owns its columns)
  for (int j = threadIdx.x; j < d; j += kLocalThreads) {
    const int64_t base = b * (int64_t)k * d + j;
    for (int r = 0; r + 1 < k; ++r) store_act<Half>(win, base + (int64_t)r * d, load_act<Half>(win, base + (int64_t)(r + 1) * d));
    store_act<Half>(win, base + (int64_t)(k - 1) * d, s_u[j]);
  }
}

template <bool Half>
__global__ void __launch_bounds__(kLocalThreads) k_local_mid(int d, const float* h, const void* z, float* h1,
                                                             const float* ln_w, const float* ln_b, float eps,
                                                             void* v_out) {
  extern __shared__ float s_loc[];
  float* s_x = s_loc;
  float* s_u = s_loc + d;
  float* red = s_loc + 2 * d;
  const int64_t b = blockIdx.x;
  for (int j = threadIdx.x; j < d; j += kLocalThreads) {
    const float g = act<Half>(gelu_t(load_act<Half>(z, b * d + j)));
    const float x = __fadd_rn(h[b * d + j], g);
    s_x[j] = x;
    h1[b * d + j] = x;
  }
  __syncthreads();
  row_layer_norm<Half>(s_x, d, ln_w, ln_b, eps, red, s_u);
  for (int j = threadIdx.x; j < d; j += kLocalThreads) store_act<Half>(v_out, b * d + j, s_u[j]);
}

template <bool Half>
__global__ void k_local_gelu(int64_t n, void* f) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) store_act<Half>(f, i, act<Half>(gelu_t(load_act<Half>(f, i))));
}

int launch_local_in(int64_t B, int d, int k, const float* h_prev, const void* y_prev, float* h_out, const float* ln_w,
                    const float* ln_b, float eps, void* win, bool half, cudaStream_t s) {
  if (B == 0) return ASRN_OK;
  const size_t smem = (2 * (size_t)d + 32) * sizeof(float);
  if (half) k_local_in<true><<<(unsigned)B, kLocalThreads, smem, s>>>(d, k, h_prev, y_prev, h_out, ln_w, ln_b, eps, win);
  else k_local_in<false><<<(unsigned)B, kLocalThreads, smem, s>>>(d, k, h_prev, y_prev, h_out, ln_w, ln_b, eps, win);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_local_mid(int64_t B, int d, const float* h, const void* z, float* h1, const float* ln_w, const float* ln_b,
                     float eps, void* v_out, bool half, cudaStream_t s) {
  if (B == 0) return ASRN_OK;
  const size_t smem = (2 * (size_t)d + 32) * sizeof(float);
  if (half) k_local_mid<true><<<(unsigned)B, kLocalThreads, smem, s>>>(d, h, z, h1, ln_w, ln_b, eps, v_out);
  else k_local_mid<false><<<(unsigned)B, kLocalThreads, smem, s>>>(d, h, z, h1, ln_w, ln_b, eps, v_out);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_local_gelu(int64_t n, void* f, bool half, cudaStream_t s) {
  if (n == 0) return ASRN_OK;
  if (half) k_local_gelu<true><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, f);
  else k_local_gelu<false><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, f);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
