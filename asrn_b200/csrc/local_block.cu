// The model's local block (BloqueLocal, asrn/nucleo.py:969-1014, mezcla='conv') over whole sequences under bfloat16
// autocast:
//   z = LN1(h); c = gelu(conv_k(pad(z))) ; h1 = h + c ; h' = h1 + W2 gelu(W1 LN2(h1) + b1) + b2
// PyTorch runs it as about fifteen kernels (two fp32 LayerNorms, the transposes and pad copy around cuDNN's conv and its
// layout conversions, the bias add, GELUs, casts, residual adds); here it is five launches:
//   k_local_ln         LN1(h) -> z (bf16), a warp per token
//   k_local_gemm<0>    the causal conv as one GEMM: out(b, p) = sum_j z(b, p - (k-1) + j) . W_j^T, the k taps as k
//                      K-blocks whose A tiles are the same z rows shifted by j (a 3-D tensor map over (d, L, B): rows
//                      before the sequence read zeros, the conv's left padding); epilogue bf16(bf16(acc) + b) (cuDNN's
//                      output then the separate bias add), GELU, h1 = h + that
//   k_local_ln         LN2(h1) -> u (bf16)
//   k_local_gemm<1>    f = gelu(bf16(u . W1^T + b1)) (bf16)
//   k_local_gemm<2>    h' = h1 + bf16(f . W2^T + b2)
// Each GEMM is the persistent tcgen05 pipeline of the gate (one block per SM over 128-token x NT-column tiles, a TMA
// producer warp for both operands through four stages of 16 + NT / 8 KB, an MMA warp filling one of two TMEM
// accumulators, a TMA warp staging the fp32 residual rows through two 16 KB slots, eight epilogue warps draining the
// other accumulator). Per token and block the HBM
// traffic is about 31 KB (the fp32 residual stream read four times and written twice, the bf16 intermediates once each
// way), against about 90 KB for the PyTorch sequence.
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

struct LocalGemmArgs {
  int64_t B, L;
  int K;                 // reduction length of one tap (a multiple of 64)
  int taps;              // conv: k; linear: 1
  int N;                 // output columns (a multiple of the column tile)
  const float* bias;     // (N), rounded to bf16 as autocast does
  float* out32;          // modes 0 and 2: (B, L, N) fp32
  __nv_bfloat16* out16;  // mode 1: (B, L, N) bf16
  int* status;           // device status word for the bounded waits (may be null)
};

namespace {
constexpr int kLTM = 128, kLBK = 64;
constexpr int kLStageA = kLTM * 128;
constexpr int kLStages = 4;
constexpr int kLEpiWarps = 8;
constexpr int kLHSlots = 2;
constexpr int kLHTile = kLTM * 128;
constexpr int kLThreads = (3 + kLEpiWarps) * 32;
constexpr int kLnThreads = 256;

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(umma::smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(umma::smem_u32(bar))
      : "memory");
}

// torch's GELU (approximate='none') on a bf16 value, computed in fp32
__device__ __forceinline__ float gelu_f(float x) { return x * 0.5f * (1.0f + erff(x * 0.70710678118654752f)); }
}  // namespace

// LayerNorm of fp32 rows into bf16 (a warp per row; d a multiple of 128, at most 1024): mean, then the population
// variance of the centred values, rstd = rsqrt(var + eps), y = (x - mean) * rstd * w + b.
__global__ void __launch_bounds__(kLnThreads) k_local_ln(int64_t rows, int d, const float* __restrict__ x,
                                                         const float* __restrict__ w, const float* __restrict__ b,
                                                         float eps, __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kLnThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = d / 128;                       // float4 per lane
  const float4* xr = reinterpret_cast<const float4*>(x + row * d);
  float4 v[8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < nv) {
      v[i] = xr[i * 32 + lane];
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < nv) {
      const float a0 = v[i].x - mean, a1 = v[i].y - mean, a2 = v[i].z - mean, a3 = v[i].w - mean;
      q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / (float)d + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  uint2* o2 = reinterpret_cast<uint2*>(out + row * d);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < nv) {
      const float4 g = w4[i * 32 + lane], c = b4[i * 32 + lane];
      uint2 pk;
      pk.x = umma::pack_bf16x2((v[i].x - mean) * rstd * g.x + c.x, (v[i].y - mean) * rstd * g.y + c.y);
      pk.y = umma::pack_bf16x2((v[i].z - mean) * rstd * g.z + c.z, (v[i].w - mean) * rstd * g.w + c.w);
      o2[i * 32 + lane] = pk;
    }
}

// Persistent GEMM over (sequence, 128-position) x NT-column tiles, n-tile fastest. A: 3-D map over (K, L, B) bf16,
// box 64 x 128 x 1 (tap j reads rows p0 - (taps - 1) + j); W: 2-D map over (taps * K, N) bf16, box 64 x NT; H: 3-D map
// over the fp32 residual (N, L, B), box 32 x 128 x 1 (128-byte swizzle), used by modes 0 and 2.
template <int NT, int Mode>
__global__ void __launch_bounds__(kLThreads, 1)
k_local_gemm(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
             const __grid_constant__ CUtensorMap tmap_h, LocalGemmArgs a, int ntn, int ptiles, int ntiles) {
  using namespace umma;
  constexpr bool kRes = Mode != 1;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  constexpr int kStageB = NT * 128;
  uint8_t* sA = sm;
  uint8_t* sB = sm + kLStages * kLStageA;
  uint8_t* sH = sB + kLStages * kStageB;                                     // [kLHSlots][128 rows][128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(sH + (kRes ? kLHSlots * kLHTile : 0));
  uint64_t* empty = full + kLStages;
  uint64_t* tfull = empty + kLStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* hfull = tempty + 2;
  uint64_t* hempty = hfull + kLHSlots;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(hempty + kLHSlots);

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nkc = a.K / kLBK;
  const int nk = a.taps * nkc;
  if (tid == 0) {
    for (int i = 0; i < kLStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull + i, 1);
      mbar_init(tempty + i, kLEpiWarps);
    }
    for (int i = 0; i < kLHSlots; ++i) {
      mbar_init(hfull + i, 1);
      mbar_init(hempty + i, 4);
    }
    fence_mbar_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_w);
    if (kRes) prefetch_tensormap(&tmap_h);
  }
  if (wid == 1) {
    tmem_alloc(tmem_base_s, 2 * NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  constexpr uint32_t kTx = (uint32_t)(kLStageA + kStageB);

  if (wid == 0) {
    if (lane == 0) {                      // operand producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int mt = tile / ntn, n0 = (tile % ntn) * NT;
        const int b = mt / ptiles, p0 = (mt % ptiles) * kLTM;
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % kLStages;
          if (it >= kLStages && !(ok = mbar_wait(empty + s, ((it / kLStages) - 1) & 1, a.status))) break;
          const int j = k / nkc, kc = k % nkc;
          mbar_expect_tx(full + s, kTx);
          tma_load_3d(sA + s * kLStageA, &tmap_a, kc * kLBK, p0 - (a.taps - 1) + j, b, full + s);
          tma_load_2d(sB + s * kStageB, &tmap_w, j * a.K + kc * kLBK, n0, full + s);
        }
      }
    }
  } else if (wid == 1) {
    if (lane == 0) {                      // MMA issuer
      const uint32_t idesc = idesc_bf16(kLTM, NT);
      int it = 0, jt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++jt) {
        const int b = jt & 1;
        if (jt >= 2 && !(ok = mbar_wait(tempty + b, ((jt >> 1) - 1) & 1, a.status))) break;
        tc_fence_after();
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % kLStages;
          if (!(ok = mbar_wait(full + s, (it / kLStages) & 1, a.status))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kLStageA), b0 = smem_u32(sB + s * kStageB);
#pragma unroll
          for (int q = 0; q < kLBK / 16; ++q)
            mma_bf16(tmem + (uint32_t)(b * NT), desc_sw128(a0 + q * 32), desc_sw128(b0 + q * 32), idesc,
                     (k > 0 || q > 0) ? 1u : 0u);
          mma_commit(empty + s);
        }
        mma_commit(tfull + b);
      }
    }
  } else if (wid == 2) {
    if (kRes && lane == 0) {              // residual rows: chunk cc (tile, 32 columns) into slot cc % kLHSlots
      int cc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int mt = tile / ntn, n0 = (tile % ntn) * NT;
        const int b = mt / ptiles, p0 = (mt % ptiles) * kLTM;
        for (int ch = 0; ch * 32 < NT; ++ch, ++cc) {
          const int sl = cc % kLHSlots;
          if (cc >= kLHSlots && !(ok = mbar_wait(hempty + sl, ((cc / kLHSlots) - 1) & 1, a.status))) break;
          mbar_expect_tx(hfull + sl, (uint32_t)kLHTile);
          tma_load_3d(sH + sl * kLHTile, &tmap_h, n0 + ch * 32, p0, b, hfull + sl);
        }
      }
    }
  } else {                                // epilogue
    const int q4 = wid & 3, half = (wid - 3) >> 2;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const int r = q4 * 32 + lane;
    const int nch = NT / 32;
    int jt = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++jt) {
      const int acc = jt & 1;
      const int mt = tile / ntn, n0 = (tile % ntn) * NT;
      const int64_t b = mt / ptiles;
      const int64_t p = (int64_t)(mt % ptiles) * kLTM + r;
      const bool row_ok = p < a.L;
      const int64_t g = b * a.L + p;
      if (!mbar_wait(tfull + acc, (jt >> 1) & 1, a.status)) break;
      tc_fence_after();
      bool ok = true;
#pragma unroll 1
      for (int ch = half; ch < nch; ch += 2) {
        const int c0 = n0 + ch * 32;
        float v[32];
        tmem_ld32(trow + (uint32_t)(acc * NT + ch * 32), v);
        // the bias as autocast passes it (bf16), then the mode's rounding chain
        float bias[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(a.bias + c0) + i);
          bias[4 * i] = b4.x; bias[4 * i + 1] = b4.y; bias[4 * i + 2] = b4.z; bias[4 * i + 3] = b4.w;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float bb = round_bf16(bias[i]);
          if (Mode == 0) v[i] = round_bf16(gelu_f(round_bf16(__fadd_rn(round_bf16(v[i]), bb))));
          else if (Mode == 1) v[i] = gelu_f(round_bf16(__fadd_rn(v[i], bb)));
          else v[i] = round_bf16(__fadd_rn(v[i], bb));
        }
        if (kRes) {
          const int cc = jt * nch + ch, sl = cc % kLHSlots;
          if (!(ok = mbar_wait(hfull + sl, (cc / kLHSlots) & 1, a.status))) break;
          const uint8_t* hs = sH + sl * kLHTile + r * 128;
          if (row_ok) {
            float4* orow = reinterpret_cast<float4*>(a.out32 + g * a.N + c0);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 hv = *reinterpret_cast<const float4*>(hs + ((i ^ (r & 7)) << 4));
              orow[i] = make_float4(__fadd_rn(hv.x, v[4 * i]), __fadd_rn(hv.y, v[4 * i + 1]),
                                    __fadd_rn(hv.z, v[4 * i + 2]), __fadd_rn(hv.w, v[4 * i + 3]));
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(hempty + sl);
        } else if (row_ok) {
          uint4* orow = reinterpret_cast<uint4*>(a.out16 + g * a.N + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            orow[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                 pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
        }
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * NT);
  }
}

namespace {

template <int NT, int Mode>
size_t local_gemm_smem() {
  return 1024 + (size_t)kLStages * (kLStageA + (size_t)NT * 128) + (Mode != 1 ? (size_t)kLHSlots * kLHTile : 0) +
         (2 * kLStages + 4 + 2 * kLHSlots) * 8 + 16;
}

int sm_count_local() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

template <int NT, int Mode>
int launch_local_gemm(const LocalGemmArgs& a, const void* A, const void* W, const float* H, cudaStream_t s) {
  CUtensorMap ma, mw, mh;
  if (!make_tmap_bf16_3d(&ma, A, (uint64_t)a.K, (uint64_t)a.L, (uint64_t)a.B, 64, 128) ||
      !make_tmap_bf16(&mw, W, (uint64_t)a.taps * a.K, (uint64_t)a.N, (uint64_t)a.taps * a.K * 2, 64, (uint32_t)NT))
    return ASRN_ERR_CUDA;
  if (Mode != 1 && !make_tmap_f32_3d_sw128(&mh, H, (uint64_t)a.N, (uint64_t)a.L, (uint64_t)a.B, 32, 128))
    return ASRN_ERR_CUDA;
  if (Mode == 1) mh = mw;                                  // unused
  const size_t smem = local_gemm_smem<NT, Mode>();
  cudaFuncSetAttribute(k_local_gemm<NT, Mode>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t ptiles = (a.L + kLTM - 1) / kLTM;
  const int64_t ntn = a.N / NT;
  const int64_t ntiles = a.B * ptiles * ntn;
  if (ntiles >= ((int64_t)1 << 31) || ptiles >= ((int64_t)1 << 30)) return ASRN_ERR_UNSUPPORTED;
  const int grid = (int)std::min<int64_t>(ntiles, sm_count_local());
  k_local_gemm<NT, Mode><<<grid, kLThreads, smem, s>>>(ma, mw, mh, a, (int)ntn, (int)ptiles, (int)ntiles);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

template <int Mode>
int launch_local_gemm_n(const LocalGemmArgs& a, const void* A, const void* W, const float* H, cudaStream_t s) {
  if (a.N % 256 == 0) return launch_local_gemm<256, Mode>(a, A, W, H, s);
  if (a.N % 128 == 0) return launch_local_gemm<128, Mode>(a, A, W, H, s);
  return ASRN_ERR_UNSUPPORTED;
}

struct LocalWs {
  size_t zu, g, h1, total;
};

LocalWs local_ws(int64_t B, int64_t L, int64_t d, int64_t ff) {
  LocalWs w{};
  const size_t M = (size_t)B * L;
  size_t o = 0;
  w.zu = o; o = align_up(o + M * d * 2);
  w.g = o; o = align_up(o + M * ff * 2);
  w.h1 = o; o = align_up(o + M * d * 4);
  w.total = o;
  return w;
}

}  // namespace
}  // namespace asrn

extern "C" {

size_t asrn_local_block_workspace_bytes(int64_t B, int64_t L, int32_t d, int32_t ff) {
  if (B < 0 || L < 0 || d <= 0 || ff <= 0) return 0;
  return asrn::local_ws(B, L, d, ff).total;
}

int asrn_local_block(int64_t B, int64_t L, int32_t d, int32_t k, int32_t ff, const float* h, float* h_out,
                     const float* ln1_w, const float* ln1_b, float eps1, const void* w_conv, const float* b_conv,
                     const float* ln2_w, const float* ln2_b, float eps2, const void* w1, const float* b1,
                     const void* w2, const float* b2, void* workspace, size_t workspace_bytes, int* status,
                     void* stream) {
  using namespace asrn;
  if (B < 0 || L < 0 || k < 1 || k > 16 || d <= 0 || ff <= 0) return ASRN_ERR_ARG;
  if (d % 128 || d > 1024 || ff % 128) return ASRN_ERR_UNSUPPORTED;
  if (B * L == 0) return ASRN_OK;
  if (!h || !h_out || !ln1_w || !ln1_b || !w_conv || !b_conv || !ln2_w || !ln2_b || !w1 || !b1 || !w2 || !b2)
    return ASRN_ERR_ARG;
  if (L >= ((int64_t)1 << 31) || B >= ((int64_t)1 << 31)) return ASRN_ERR_UNSUPPORTED;
  const LocalWs ws = local_ws(B, L, d, ff);
  if (!workspace || workspace_bytes < ws.total) return ASRN_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* base = reinterpret_cast<char*>(workspace);
  __nv_bfloat16* zu = reinterpret_cast<__nv_bfloat16*>(base + ws.zu);
  __nv_bfloat16* g = reinterpret_cast<__nv_bfloat16*>(base + ws.g);
  float* h1 = reinterpret_cast<float*>(base + ws.h1);
  const int64_t M = B * L;
  const unsigned ln_grid = (unsigned)((M + kLnThreads / 32 - 1) / (kLnThreads / 32));
  int st;
  k_local_ln<<<ln_grid, kLnThreads, 0, s>>>(M, d, h, ln1_w, ln1_b, eps1, zu);
  if (cudaGetLastError() != cudaSuccess) return ASRN_ERR_CUDA;
  LocalGemmArgs a{};
  a.B = B; a.L = L; a.status = status;
  a.K = d; a.taps = k; a.N = d; a.bias = b_conv; a.out32 = h1;
  if ((st = launch_local_gemm_n<0>(a, zu, w_conv, h, s))) return st;
  k_local_ln<<<ln_grid, kLnThreads, 0, s>>>(M, d, h1, ln2_w, ln2_b, eps2, zu);
  if (cudaGetLastError() != cudaSuccess) return ASRN_ERR_CUDA;
  a.K = d; a.taps = 1; a.N = ff; a.bias = b1; a.out32 = nullptr; a.out16 = g;
  if ((st = launch_local_gemm_n<1>(a, zu, w1, nullptr, s))) return st;
  a.K = ff; a.taps = 1; a.N = d; a.bias = b2; a.out32 = h_out; a.out16 = nullptr;
  return launch_local_gemm_n<2>(a, g, w2, h1, s);
}

}  // extern "C"
