// Gate and output projection. Reference: CapaASRNEstable._combinar (asrn/estable.py:376-403), _senales
// (asrn/estable.py:294-300) and _respuesta_racha (asrn/nucleo.py:865-878):
//   pt = tables with candidates; mejor = max over those tables of their best score (else 0), clamped to +-mejor_max
//   logit = g(h) + g_conf([pt/T, mejor, pico/max(1,pt), pt_ctx/Tc]) + w_vistos . vistos + u_hawkes . log1p(hawkes)
//           + response(racha)                                     (all fp32; g_conf in bf16 under autocast)
//   h' = h + sigmoid(logit) * o(salida / max(1, pt))
// Here salida = W_v acc (acc = sum of att * Ea rows from the scoring kernel; a bf16 accumulator under autocast), so
// o(salida / pt) = (W_o W_v) acc / pt and the projection is one GEMM against the prepared W_ov.
#include "common.cuh"
#include "gate.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

constexpr int kGateTM = 64, kGateTN = 64, kGateKC = 32;

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
      const float av = (g < M && k < d) ? (a.acc16 ? __bfloat162float(a.acc16[g * d + k]) : a.acc[g * d + k]) : 0.f;
      As[kk][r] = (g < M && k < d) ? act<Half>(__fdiv_rn(av, s_pt[r])) : 0.f;
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

// ---- tensor-core version (bf16 autocast mode) -------------------------------------------------------------------
// k_gate_scalars: one thread per token computes the gate sigmoid(logit) (rounded to bf16) and 1 / max(1, pt).
// k_gate_tc: h' = h + bf16(sigma * bf16((acc . W_ov^T) / max(1, pt))) with acc the scoring's bf16 accumulator read as
//   the A operand (the reference rounds acc / pt to bf16 before o; here the division follows the GEMM: the same value
//   up to bf16 rounding). Tile 128 tokens (TMEM lanes) x NT columns (TMEM columns), K = d in chunks of 64; both
//   operands by TMA (128-byte swizzle), one producer thread and one MMA thread (tcgen05.commit frees each stage), the
//   fp32 accumulators in TMEM; in the epilogue each thread owns one tile row (its TMEM lane) and reads h / writes h'
//   for 32 consecutive columns at a time with 16-byte accesses.
template <bool Half>
__global__ void __launch_bounds__(256) k_gate_scalars(GateArgs a) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= a.B * a.L) return;
  float sg, pt;
  gate_of_token<Half>(a, g, &sg, &pt);
  a.sigma[g] = sg;
  // pt is a count of tables (1 .. T): the division becomes a product with 1 / pt (exact for powers of two, else
  // within one fp32 ulp of the quotient before the bf16 rounding)
  a.rpt[g] = __frcp_rn(pt);
}

namespace {
constexpr int kGTM = 128, kGBK = 64;
constexpr int kGStageA = kGTM * 128;
constexpr int kGStages = 3;
constexpr int kGEpiWarps = 8;
constexpr int kGHSlots = 4;                         // h tiles (128 rows x 32 fp32, 16 KB) staged for the epilogue
constexpr int kGHTile = kGTM * 128;
// warp 0: operand TMA producer, warp 1: MMA issuer, warp 2: h TMA producer, warps 3-10: epilogue
constexpr int kGThreads = (3 + kGEpiWarps) * 32;
}  // namespace

// Persistent: one block per SM walks the (128-token, NT-column) tiles of the output, n-tile fastest (the blocks of one
// token tile run side by side and share its operand rows in L2). Warp 0 streams the K chunks of both operands through
// kGStages shared-memory stages, warp 1 issues the MMAs into one of two TMEM accumulators (2 NT columns), warp 2
// streams the tile's h as 128 x 32 fp32 boxes (128-byte swizzle) through kGHSlots slots, and the 8 epilogue warps
// drain the other accumulator meanwhile: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its tile rows) for the 32-column
// chunks of its half (even or odd chunks), adds the staged h and writes h'.
template <int NT>
__global__ void __launch_bounds__(kGThreads, 1)
k_gate_tc(const __grid_constant__ CUtensorMap tmap_c, const __grid_constant__ CUtensorMap tmap_wov,
          const __grid_constant__ CUtensorMap tmap_h, GateArgs a, int ntn, int ntiles) {
  using namespace umma;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  constexpr int kStageB = NT * 128;
  uint8_t* sA = sm;
  uint8_t* sB = sm + kGStages * kGStageA;
  uint8_t* sH = sB + kGStages * kStageB;                                     // [kGHSlots][128 rows][128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(sH + kGHSlots * kGHTile);     // [kGStages]
  uint64_t* empty = full + kGStages;                                         // [kGStages]
  uint64_t* tfull = empty + kGStages;                                        // [2] accumulator ready
  uint64_t* tempty = tfull + 2;                                              // [2] accumulator drained
  uint64_t* hfull = tempty + 2;                                              // [kGHSlots]
  uint64_t* hempty = hfull + kGHSlots;                                       // [kGHSlots]
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(hempty + kGHSlots);

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int d = a.d;
  const int nk = d / kGBK;
  const int64_t M = a.B * a.L;
  if (tid == 0) {
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull + i, 1);
      mbar_init(tempty + i, kGEpiWarps);
    }
    for (int i = 0; i < kGHSlots; ++i) {
      mbar_init(hfull + i, 1);
      mbar_init(hempty + i, 4);                // the four warps (row quadrants) of one half read a chunk
    }
    fence_mbar_init();
    prefetch_tensormap(&tmap_c);
    prefetch_tensormap(&tmap_wov);
    prefetch_tensormap(&tmap_h);
  }
  if (wid == 1) {
    tmem_alloc(tmem_base_s, 2 * NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  constexpr uint32_t kTx = (uint32_t)(kGStageA + kStageB);

  if (wid == 0) {
    if (lane == 0) {                      // producer
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile / ntn) * kGTM, n0 = (tile % ntn) * NT;
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % kGStages;
          if (it >= kGStages && !(ok = mbar_wait(empty + s, ((it / kGStages) - 1) & 1, a.status))) break;
          mbar_expect_tx(full + s, kTx);
          tma_load_2d(sA + s * kGStageA, &tmap_c, k * kGBK, m0, full + s);
          tma_load_2d(sB + s * kStageB, &tmap_wov, k * kGBK, n0, full + s);
        }
      }
    }
  } else if (wid == 1) {
    if (lane == 0) {                      // MMA issuer
      const uint32_t idesc = idesc_bf16(kGTM, NT);
      int it = 0, j = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !(ok = mbar_wait(tempty + b, ((j >> 1) - 1) & 1, a.status))) break;
        tc_fence_after();
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % kGStages;
          if (!(ok = mbar_wait(full + s, (it / kGStages) & 1, a.status))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kGStageA), b0 = smem_u32(sB + s * kStageB);
#pragma unroll
          for (int q = 0; q < kGBK / 16; ++q)
            mma_bf16(tmem + (uint32_t)(b * NT), desc_sw128(a0 + q * 32), desc_sw128(b0 + q * 32), idesc,
                     (k > 0 || q > 0) ? 1u : 0u);
          mma_commit(empty + s);
        }
        mma_commit(tfull + b);
      }
    }
  } else if (wid == 2) {
    if (lane == 0) {                      // h producer: chunk cc (tile j, column chunk ch) into slot cc % kGHSlots
      int cc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile / ntn) * kGTM, n0 = (tile % ntn) * NT;
        for (int ch = 0; ch * 32 < NT; ++ch, ++cc) {
          const int sl = cc % kGHSlots;
          if (cc >= kGHSlots && !(ok = mbar_wait(hempty + sl, ((cc / kGHSlots) - 1) & 1, a.status))) break;
          mbar_expect_tx(hfull + sl, (uint32_t)kGHTile);
          tma_load_2d(sH + sl * kGHTile, &tmap_h, n0 + ch * 32, m0, hfull + sl);
        }
      }
    }
  } else {                                // epilogue
    const int q4 = wid & 3, half = (wid - 3) >> 2;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const int r = q4 * 32 + lane;         // tile row of this thread
    const int nch = NT / 32;
    int j = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++j) {
      const int b = j & 1;
      const int64_t m0 = (int64_t)(tile / ntn) * kGTM;
      const int n0 = (tile % ntn) * NT;
      const int64_t g = m0 + r;
      const bool row_ok = g < M;
      const float sg = row_ok ? a.sigma[g] : 0.f;
      const float rp = row_ok ? a.rpt[g] : 0.f;
      float4* orow = reinterpret_cast<float4*>(a.out + g * d + n0);
      if (!mbar_wait(tfull + b, (j >> 1) & 1, a.status)) break;
      tc_fence_after();
      bool ok = true;
#pragma unroll 1
      for (int ch = half; ch < nch; ch += 2) {
        const int cc = j * nch + ch, sl = cc % kGHSlots;
        float v[32];
        tmem_ld32(trow + (uint32_t)(b * NT + ch * 32), v);
        if (!(ok = mbar_wait(hfull + sl, (cc / kGHSlots) & 1, a.status))) break;
        const uint8_t* hs = sH + sl * kGHTile + r * 128;
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 hv = *reinterpret_cast<const float4*>(hs + ((i ^ (r & 7)) << 4));
            float4 o;
            o.x = __fadd_rn(hv.x, round_bf16(__fmul_rn(sg, round_bf16(__fmul_rn(v[4 * i], rp)))));
            o.y = __fadd_rn(hv.y, round_bf16(__fmul_rn(sg, round_bf16(__fmul_rn(v[4 * i + 1], rp)))));
            o.z = __fadd_rn(hv.z, round_bf16(__fmul_rn(sg, round_bf16(__fmul_rn(v[4 * i + 2], rp)))));
            o.w = __fadd_rn(hv.w, round_bf16(__fmul_rn(sg, round_bf16(__fmul_rn(v[4 * i + 3], rp)))));
            orow[ch * 8 + i] = o;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(hempty + sl);
      }
      if (!ok) break;
      // this warp has read its part of accumulator b
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + b);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * NT);
  }
}

template <int NT>
static size_t gate_tc_smem() {
  return 1024 + (size_t)kGStages * (kGStageA + (size_t)NT * 128) + (size_t)kGHSlots * kGHTile +
         (2 * kGStages + 4 + 2 * kGHSlots) * 8 + 16;
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

int gate_tc_tile(int d) {
  if (d % 256 == 0) return 256;
  if (d % 128 == 0) return 128;
  if (d % 64 == 0) return 64;
  return 0;
}

template <int NT>
static int launch_gate_tc_t(const GateArgs& a, const CUtensorMap& mc, const CUtensorMap& mw, const CUtensorMap& mh,
                            cudaStream_t s) {
  const size_t smem = gate_tc_smem<NT>();
  cudaFuncSetAttribute(k_gate_tc<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t M = a.B * a.L;
  const int64_t ntiles = ((M + kGTM - 1) / kGTM) * (a.d / NT);
  if (ntiles >= ((int64_t)1 << 31)) return ASRN_ERR_UNSUPPORTED;
  const int grid = (int)std::min<int64_t>(ntiles, sm_count());
  k_gate_tc<NT><<<grid, kGThreads, smem, s>>>(mc, mw, mh, a, a.d / NT, (int)ntiles);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_gate_tc(const GateArgs& a, int nt, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  k_gate_scalars<true><<<(unsigned)((M + 255) / 256), 256, 0, s>>>(a);
  if (cudaGetLastError() != cudaSuccess) return ASRN_ERR_CUDA;
  CUtensorMap mc, mw, mh;
  if (!make_tmap_bf16(&mc, a.acc16, (uint64_t)a.d, (uint64_t)M, (uint64_t)a.d * 2, 64, 128) ||
      !make_tmap_bf16(&mw, a.wov, (uint64_t)a.d, (uint64_t)a.d, (uint64_t)a.d * 2, 64, (uint32_t)nt) ||
      !make_tmap_f32_sw128(&mh, a.h, (uint64_t)a.d, (uint64_t)M, (uint64_t)a.d * 4, 32, 128))
    return ASRN_ERR_CUDA;
  switch (nt) {
    case 256: return launch_gate_tc_t<256>(a, mc, mw, mh, s);
    case 128: return launch_gate_tc_t<128>(a, mc, mw, mh, s);
    case 64: return launch_gate_tc_t<64>(a, mc, mw, mh, s);
    default: return ASRN_ERR_UNSUPPORTED;
  }
}

size_t gate_workspace(int64_t M, int d, bool half) {
  if (!half || gate_tc_tile(d) == 0) return 0;
  return align_up((size_t)M * 8);                 // sigma and 1 / max(1, pt) per token
}

int launch_gate(const GateArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  const int nt = gate_tc_tile(a.d);
  if (half && !a.acc16) return ASRN_ERR_ARG;
  if (!half && !a.acc) return ASRN_ERR_ARG;
  if (half && tensor_cores_enabled() && nt > 0) {
    if (!a.sigma || !a.rpt) return ASRN_ERR_WORKSPACE;
    return launch_gate_tc(a, nt, s);
  }
  dim3 grid((unsigned)((a.d + kGateTN - 1) / kGateTN), (unsigned)((M + kGateTM - 1) / kGateTM));
  if (half)
    k_gate_simt<true><<<grid, 256, 0, s>>>(a);
  else
    k_gate_simt<false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

// ---- gate of the new tokens of a generation step (B rows) ----------------------------------------------------------
// k_gen_gate_tc (bf16 autocast): one block per 32 output columns, so W_ov is spread over d / 32 CTAs; the gate scalars
// of every row (gate_of_token), then h' = h + bf16(sigma * bf16(c . W_ov^T)) with c = bf16(acc / max(1, pt)) on
// mma.sync. fp32 mode uses k_gate_simt.

namespace {
constexpr int kGGCols = 32, kGGRows = 64, kGGThreads = 256, kGGUnroll = 8;

__device__ __forceinline__ void mma_16816_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void gg_cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
}  // namespace

// Block: kGGCols output columns for all rows, row tiles of 64; warp w: rows 16 (w % 4) .. + 15, columns
// 16 (w / 4) .. + 15 of the block. Shared memory: the block's W_ov rows (kGGCols x d, by cp.async, in flight while
// the gate scalars and the operand are computed) and the tile's operand c (64 x d), both bf16, rows padded by 8.
__global__ void __launch_bounds__(kGGThreads) k_gen_gate_tc(GateArgs a) {
  extern __shared__ __align__(16) uint8_t smem_gg[];
  const int d = a.d, ld = d + 8;
  const int64_t M = a.B * a.L;
  const int n0 = blockIdx.x * kGGCols;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_gg);
  __nv_bfloat16* s_c = s_w + kGGCols * ld;
  float* s_sigma = reinterpret_cast<float*>(s_c + kGGRows * ld);
  float* s_pt = s_sigma + kGGRows;
  const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(a.wov);
  const int cpr = d / 8;
  for (int e = tid; e < kGGCols * cpr; e += kGGThreads) {
    const int r = e / cpr, c8 = e % cpr;
    __nv_bfloat16* dst = s_w + r * ld + c8 * 8;
    if (n0 + r < d) gg_cp_async16(dst, W + (int64_t)(n0 + r) * d + c8 * 8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int rg = wid & 3, cg = wid >> 2;
  const bool pre = a.cbuf != nullptr && a.sigma != nullptr;   // c and sigma computed by the attention kernel
  for (int64_t r0 = 0; r0 < M; r0 += kGGRows) {
    if (pre) {
      for (int e = tid; e < kGGRows * cpr; e += kGGThreads) {
        const int r = e / cpr, c8 = e % cpr;
        __nv_bfloat16* dst = s_c + r * ld + c8 * 8;
        if (r0 + r < M) gg_cp_async16(dst, a.cbuf + (r0 + r) * d + c8 * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
      if (tid < kGGRows) s_sigma[tid] = (r0 + tid < M) ? a.sigma[r0 + tid] : 0.f;
    } else if (tid < kGGRows) {
      float sg = 0.f, pt = 1.f;
      if (r0 + tid < M) gate_of_token<true>(a, r0 + tid, &sg, &pt);
      s_sigma[tid] = sg;
      s_pt[tid] = pt;
    }
    __syncthreads();
    // c = bf16(acc / pt): kGGUnroll independent 16-byte loads per thread in flight
    const int cq = d / 4, tot = pre ? 0 : kGGRows * cq;
    for (int e0 = tid; e0 < tot; e0 += kGGThreads * kGGUnroll) {
      float4 x[kGGUnroll];
#pragma unroll
      for (int u = 0; u < kGGUnroll; ++u) {
        const int e = e0 + u * kGGThreads;
        const int r = e / cq, c4 = e % cq;
        x[u] = (e < tot && r0 + r < M) ? __ldg(reinterpret_cast<const float4*>(a.acc + (r0 + r) * d + c4 * 4))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kGGUnroll; ++u) {
        const int e = e0 + u * kGGThreads;
        if (e >= tot) continue;
        const int r = e / cq, c4 = e % cq;
        const float p = s_pt[r];
        const __nv_bfloat162 lo = __floats2bfloat162_rn(__fdiv_rn(x[u].x, p), __fdiv_rn(x[u].y, p));
        const __nv_bfloat162 hi = __floats2bfloat162_rn(__fdiv_rn(x[u].z, p), __fdiv_rn(x[u].w, p));
        *reinterpret_cast<__nv_bfloat162*>(s_c + r * ld + c4 * 4) = lo;
        *reinterpret_cast<__nv_bfloat162*>(s_c + r * ld + c4 * 4 + 2) = hi;
      }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    float c[2][4] = {};
    const __nv_bfloat16* ar0 = s_c + (rg * 16 + g) * ld + 2 * t4;
    const __nv_bfloat16* ar1 = ar0 + 8 * ld;
    for (int k0 = 0; k0 < d; k0 += 16) {
      uint32_t af[4];
      af[0] = *reinterpret_cast<const uint32_t*>(ar0 + k0);
      af[1] = *reinterpret_cast<const uint32_t*>(ar1 + k0);
      af[2] = *reinterpret_cast<const uint32_t*>(ar0 + k0 + 8);
      af[3] = *reinterpret_cast<const uint32_t*>(ar1 + k0 + 8);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const __nv_bfloat16* br = s_w + (cg * 16 + nt * 8 + g) * ld + k0 + 2 * t4;
        mma_16816_bf16(c[nt], af, *reinterpret_cast<const uint32_t*>(br),
                       *reinterpret_cast<const uint32_t*>(br + 8));
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = rg * 16 + g + 8 * hf;
        const int64_t row = r0 + r;
        const int col = n0 + cg * 16 + nt * 8 + 2 * t4;
        if (row >= M || col >= d) continue;
        const float2 hv = *reinterpret_cast<const float2*>(a.h + row * d + col);
        const float o0 = round_bf16(c[nt][2 * hf]), o1 = round_bf16(c[nt][2 * hf + 1]);
        float2 ov;
        ov.x = __fadd_rn(hv.x, round_bf16(__fmul_rn(s_sigma[r], o0)));
        ov.y = __fadd_rn(hv.y, round_bf16(__fmul_rn(s_sigma[r], o1)));
        *reinterpret_cast<float2*>(a.out + row * d + col) = ov;
      }
    }
    __syncthreads();
  }
}

int launch_gen_gate(const GateArgs& a, bool half, cudaStream_t s) {
  const int64_t M = a.B * a.L;
  if (M == 0) return ASRN_OK;
  if (half && a.d % kGGCols == 0) {
    const int ld = a.d + 8;
    const size_t smem = (size_t)(kGGCols + kGGRows) * ld * 2 + 2 * kGGRows * sizeof(float);
    if (smem <= 220 * 1024) {
      cudaFuncSetAttribute(k_gen_gate_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      k_gen_gate_tc<<<(unsigned)((a.d + kGGCols - 1) / kGGCols), kGGThreads, smem, s>>>(a);
      return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
    }
  }
  constexpr int kTM = 64, kTN = 64;
  dim3 grid((unsigned)((a.d + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
  if (half) k_gate_simt<true><<<grid, 256, 0, s>>>(a);
  else k_gate_simt<false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
