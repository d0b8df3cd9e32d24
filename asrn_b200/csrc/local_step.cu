// Element-wise parts of one generation step of the model's local blocks (asrn/nucleo.py:969-1014, the O(1) writer's
// conv buffer asrn/nucleo.py:1816-1822), one block per sequence row, fused around the block's three GEMMs:
//   k_local_in   h = h_prev (+ y_prev, the previous block's MLP output), LN1(h) in fp32, rounded to the compute
//                type and pushed into the row's conv window (B, k, d) (the k - 1 previous rows shift down in place);
//                with a one-row window (k == 1) it is the final LN before the head
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

}  // namespace

// Each thread owns the columns j = threadIdx.x + 256 i (d <= 256 * kLocalCols): all of its loads (h, y, the LN
// parameters, the window rows) are issued before the row statistics, so the kernel waits on memory once.
constexpr int kLocalCols = 4;
constexpr int kMaxTaps = 16;

template <bool Half>
__global__ void __launch_bounds__(kLocalThreads) k_local_in(int d, int k, const float* h_prev, const void* y_prev,
                                                            float* h_out, const float* ln_w, const float* ln_b,
                                                            float eps, void* win) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  float x[kLocalCols], w[kLocalCols], bb[kLocalCols];
  float v[kLocalCols][kMaxTaps];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i) {
    const int j = threadIdx.x + kLocalThreads * i;
    x[i] = 0.f;
    if (j < d) {
      x[i] = h_prev[b * d + j];
      if (y_prev) x[i] = __fadd_rn(x[i], load_act<Half>(y_prev, b * d + j));
      w[i] = ln_w[j];
      bb[i] = ln_b[j];
      const int64_t base = b * (int64_t)k * d + j;
#pragma unroll
      for (int r = 0; r < kMaxTaps; ++r)
        if (r + 1 < k) v[i][r] = load_act<Half>(win, base + (int64_t)(r + 1) * d);
      s += x[i];
    }
  }
  const float mean = block_sum_local(s, red) / (float)d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i)
    if (threadIdx.x + kLocalThreads * i < d) q += (x[i] - mean) * (x[i] - mean);
  const float rstd = 1.f / sqrtf(block_sum_local(q, red) / (float)d + eps);
  // window (B, k, d): rows 0 .. k-2 take rows 1 .. k-1, row k-1 the new LN output (each thread owns its columns)
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i) {
    const int j = threadIdx.x + kLocalThreads * i;
    if (j >= d) continue;
    if (h_out) h_out[b * d + j] = x[i];
    const int64_t base = b * (int64_t)k * d + j;
#pragma unroll
    for (int r = 0; r < kMaxTaps; ++r)
      if (r + 1 < k) store_act<Half>(win, base + (int64_t)r * d, v[i][r]);
    store_act<Half>(win, base + (int64_t)(k - 1) * d, act<Half>((x[i] - mean) * rstd * w[i] + bb[i]));
  }
}

template <bool Half>
__global__ void __launch_bounds__(kLocalThreads) k_local_mid(int d, const float* h, const void* z, float* h1,
                                                             const float* ln_w, const float* ln_b, float eps,
                                                             void* v_out) {
  __shared__ float red[32];
  const int64_t b = blockIdx.x;
  float x[kLocalCols], w[kLocalCols], bb[kLocalCols];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i) {
    const int j = threadIdx.x + kLocalThreads * i;
    x[i] = 0.f;
    if (j < d) {
      const float g = act<Half>(gelu_t(load_act<Half>(z, b * d + j)));
      x[i] = __fadd_rn(h[b * d + j], g);
      w[i] = ln_w[j];
      bb[i] = ln_b[j];
      s += x[i];
    }
  }
  const float mean = block_sum_local(s, red) / (float)d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i)
    if (threadIdx.x + kLocalThreads * i < d) q += (x[i] - mean) * (x[i] - mean);
  const float rstd = 1.f / sqrtf(block_sum_local(q, red) / (float)d + eps);
#pragma unroll
  for (int i = 0; i < kLocalCols; ++i) {
    const int j = threadIdx.x + kLocalThreads * i;
    if (j >= d) continue;
    h1[b * d + j] = x[i];
    store_act<Half>(v_out, b * d + j, act<Half>((x[i] - mean) * rstd * w[i] + bb[i]));
  }
}

template <bool Half>
__global__ void k_local_gelu(int64_t n, void* f) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) store_act<Half>(f, i, act<Half>(gelu_t(load_act<Half>(f, i))));
}

int launch_local_in(int64_t B, int d, int k, const float* h_prev, const void* y_prev, float* h_out, const float* ln_w,
                    const float* ln_b, float eps, void* win, bool half, cudaStream_t s) {
  if (B == 0) return ASRN_OK;
  if (d > kLocalThreads * kLocalCols || k > kMaxTaps) return ASRN_ERR_UNSUPPORTED;
  if (half) k_local_in<true><<<(unsigned)B, kLocalThreads, 0, s>>>(d, k, h_prev, y_prev, h_out, ln_w, ln_b, eps, win);
  else k_local_in<false><<<(unsigned)B, kLocalThreads, 0, s>>>(d, k, h_prev, y_prev, h_out, ln_w, ln_b, eps, win);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_local_mid(int64_t B, int d, const float* h, const void* z, float* h1, const float* ln_w, const float* ln_b,
                     float eps, void* v_out, bool half, cudaStream_t s) {
  if (B == 0) return ASRN_OK;
  if (d > kLocalThreads * kLocalCols) return ASRN_ERR_UNSUPPORTED;
  if (half) k_local_mid<true><<<(unsigned)B, kLocalThreads, 0, s>>>(d, h, z, h1, ln_w, ln_b, eps, v_out);
  else k_local_mid<false><<<(unsigned)B, kLocalThreads, 0, s>>>(d, h, z, h1, ln_w, ln_b, eps, v_out);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_local_gelu(int64_t n, void* f, bool half, cudaStream_t s) {
  if (n == 0) return ASRN_OK;
  if (half) k_local_gelu<true><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, f);
  else k_local_gelu<false><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, f);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
