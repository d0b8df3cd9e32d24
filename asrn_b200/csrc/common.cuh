// Shared device helpers for the ASRN B200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "../../include/asrn_b200.h"

#define ASRN_DEV __device__ __forceinline__

namespace asrn {

constexpr float kProhibido = -1e9f;           // asrn/nucleo.py:86 (score of "not allowed")
constexpr int kMaxTables = 16;
constexpr int kMaxBits = 16;                   // bucket ids fit in uint16
constexpr int kMaxConfirm = 32;
constexpr int kMaxSuffix = 8;
constexpr int kMaxSeen = 8;
constexpr int kMaxHidden = 128;
constexpr int kMaxPhi = 256;

// ---- rounding helpers ----------------------------------------------------------------------------------------------
// Round-to-nearest-even fp32 -> bf16 -> fp32 (what torch's .to(bfloat16) does; NaN stays NaN).
ASRN_DEV float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
// Precision mode: Half = autocast bf16 (round activations where autocast would), else exact fp32.
template <bool Half> ASRN_DEV float act(float x) { return Half ? round_bf16(x) : x; }

// Storage of an activation tensor: bf16 in Half mode, fp32 otherwise.
template <bool Half> struct Act;
template <> struct Act<true> {
  using T = __nv_bfloat16;
  static ASRN_DEV float load(const T* p) { return __bfloat162float(*p); }
  static ASRN_DEV void store(T* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Act<false> {
  using T = float;
  static ASRN_DEV float load(const T* p) { return *p; }
  static ASRN_DEV void store(T* p, float v) { *p = v; }
};

// ---- warp / block reductions ---------------------------------------------------------------------------------------
ASRN_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
ASRN_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
ASRN_DEV double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Vector fp32 reduction into global memory (resolved in L2; sm_90+).
ASRN_DEV void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
ASRN_DEV void red_add_f32(float* addr, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(a) : "memory");
}
// bf16 reductions into global memory (resolved in L2): each element rounds (its value + the addend) to bf16.
ASRN_DEV uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
ASRN_DEV void red_add_bf16x8(__nv_bfloat16* addr, uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3) {
  asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(p0), "r"(p1), "r"(p2),
               "r"(p3)
               : "memory");
}
ASRN_DEV void red_add_bf16x4(__nv_bfloat16* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.noftz.v2.bf16x2 [%0], {%1, %2};" ::"l"(addr), "r"(pack2_bf16(a, b)),
               "r"(pack2_bf16(c, d))
               : "memory");
}
ASRN_DEV void red_add_bf16(__nv_bfloat16* addr, float a) {
  const unsigned short v = __bfloat16_as_ushort(__float2bfloat16_rn(a));
  asm volatile("red.global.add.noftz.bf16 [%0], %1;" ::"l"(addr), "h"(v) : "memory");
}

// ---- torch-compatible scalar math ----------------------------------------------------------------------------------
// torch.nn.functional.softplus with beta = 1, threshold = 20.
ASRN_DEV float softplus_t(float x) { return x > 20.f ? x : log1pf(expf(x)); }
// torch.nn.functional.logsigmoid: min(x, 0) - log1p(exp(-|x|)).
ASRN_DEV float logsigmoid_t(float x) { return fminf(x, 0.f) - log1pf(expf(-fabsf(x))); }
// Exact (erf) GELU, nn.GELU() default.
ASRN_DEV float gelu_t(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

// Affine map composition for S_i = a_i S_{i-1} + b_i: first (a1, b1), then (a2, b2).
struct Affine {
  float a, b;
};
ASRN_DEV Affine compose(Affine first, Affine second) {
  return Affine{first.a * second.a, second.a * first.b + second.b};
}

// Order-preserving map of an fp64 key to uint64 (NaN last, -0.0 == +0.0), for sorting n-gram keys.
ASRN_DEV uint64_t sortable_key(double k) {
  if (k != k) return 0xFFFFFFFFFFFFFFFFull;
  if (k == 0.0) k = 0.0;
  uint64_t u = (uint64_t)__double_as_longlong(k);
  return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

}  // namespace asrn
