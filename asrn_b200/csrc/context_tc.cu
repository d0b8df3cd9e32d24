// Context stage on tensor cores (bf16 autocast mode). Same outputs as k_context (asrn/estable.py:153-194):
//   LN(h) in fp32 (two threads per row, Welford statistics merged across the pair)
//   Qc, Kc = bf16(bf16(LN(h)) . [cq; ck]^T)            one M=128 x N=2cf x K=d tcgen05 GEMM, weights by TMA
//   u = LN(h) . w_reloj^T + b_reloj in fp32 (the unrounded normalised row), beta, log_alfa; g(h) = h . g_w + g_b
// A tile is 128 consecutive tokens; the fp32 rows of h are read twice (statistics, then normalise-and-convert).
#include <cuda.h>

#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

using namespace umma;

namespace {
constexpr int kCTM = 128, kCBK = 64;
constexpr int kCStageA = kCTM * 128;
constexpr int kCSlots = 4;                  // h chunks (128 rows x 64 fp32 = two 128 x 32 boxes, 32 KB) in flight
constexpr int kCSlot = 2 * kCTM * 128;
constexpr int kCConsumers = 256;            // warps 0-7: two threads per tile row
constexpr int kCThreads = kCConsumers + 64; // warp 8: h producer, warp 9: MMA issuer
constexpr int kCBarBytes = 256;             // mbarriers and the TMEM address (17 x 8 + 4 bytes used)
}  // namespace

// Persistent: one block per SM walks the 128-token tiles. Warp 8 streams each tile's h twice through kCSlots
// shared-memory slots by TMA (64-column chunks as two 128 x 32 fp32 boxes, 128-byte swizzle): first for the row
// statistics, then for the normalise-and-convert pass. The consumer warps (two threads per row, 32 columns of each
// chunk) merge Welford statistics per 32-value piece, then write bf16(LN(h)) into a two-stage 128-byte-swizzled operand
// ring and accumulate the clock projection in fp32; warp 9 multiplies each stage by the resident [cq; ck] into one of
// two 32-column TMEM accumulators, which warps 0-3 drain (Qc, Kc) while the next tile's statistics run.
__global__ void __launch_bounds__(kCThreads, 1)
k_context_tc(const __grid_constant__ CUtensorMap tmap_wctx, const __grid_constant__ CUtensorMap tmap_h, ContextArgs a,
             int* status, int ntiles) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  const int N = 2 * a.cf;
  const int stageB = N * 128;
  const int d = a.d;
  const int nk = d / kCBK;
  uint8_t* sH = sm;                                    // [kCSlots][2 boxes][128 rows][128 B]
  uint8_t* sA = sH + kCSlots * kCSlot;                 // [2][128 rows][128 B]
  uint8_t* sB = sA + 2 * kCStageA;                     // all d / 64 weight chunks, resident (2cf x 64 each)
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + nk * stageB);   // [kCSlots]
  uint64_t* empty = full + kCSlots;                                  // [kCSlots]
  uint64_t* afull = empty + kCSlots;                                 // [2] operand stage written
  uint64_t* aempty = afull + 2;                                      // [2] operand stage consumed by the MMAs
  uint64_t* tfull = aempty + 2;                                      // [2] accumulator ready
  uint64_t* tempty = tfull + 2;                                      // [2] accumulator drained
  uint64_t* wfull = tempty + 2;                                      // weights resident
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(wfull + 1);
  // per-column parameters, read as float4 from shared memory (16-byte aligned, past the 256 bytes of barriers):
  // ln_w, ln_b, w_reloj[0], w_reloj[1], g_w
  float* s_par = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + kCBarBytes);

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t M = a.B * a.L;
  if (tid == 0) {
    for (int i = 0; i < kCSlots; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kCConsumers / 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(afull + i, kCConsumers / 32);
      mbar_init(aempty + i, 1);
      mbar_init(tfull + i, 1);
      mbar_init(tempty + i, 4);
    }
    mbar_init(wfull, 1);
    fence_mbar_init();
    prefetch_tensormap(&tmap_wctx);
    prefetch_tensormap(&tmap_h);
  }
  if (wid == 9) {
    tmem_alloc(tmem_base_s, 64);
    tmem_relinquish();
  }
  for (int j = tid; j < d; j += kCThreads) {
    s_par[j] = a.ln_w[j];
    s_par[d + j] = a.ln_b[j];
    s_par[2 * d + j] = a.w_reloj[j];
    s_par[3 * d + j] = a.w_reloj[d + j];
    s_par[4 * d + j] = a.g_w[j];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  if (wid == 8) {
    if (lane == 0) {                       // h producer: chunk q of the (tile, pass, k) sequence into slot q % kCSlots
      int q = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = tile * kCTM;
        for (int pass = 0; pass < 2 && ok; ++pass)
          for (int k = 0; k < nk; ++k, ++q) {
            const int sl = q % kCSlots;
            if (q >= kCSlots && !(ok = mbar_wait(empty + sl, ((q / kCSlots) - 1) & 1, status))) break;
            mbar_expect_tx(full + sl, (uint32_t)kCSlot);
            tma_load_2d(sH + sl * kCSlot, &tmap_h, k * kCBK, m0, full + sl);
            tma_load_2d(sH + sl * kCSlot + kCSlot / 2, &tmap_h, k * kCBK + 32, m0, full + sl);
          }
      }
    }
  } else if (wid == 9) {
    if (lane == 0) {                       // MMA issuer
      mbar_expect_tx(wfull, (uint32_t)(nk * stageB));
      for (int kk = 0; kk < nk; ++kk) tma_load_2d(sB + kk * stageB, &tmap_wctx, kk * kCBK, 0, wfull);
      bool ok = mbar_wait(wfull, 0u, status);
      const uint32_t idesc = idesc_bf16(kCTM, N);
      int j = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !(ok = mbar_wait(tempty + b, ((j >> 1) - 1) & 1, status))) break;
        for (int k = 0; k < nk; ++k) {
          const int a2 = j * nk + k, st = a2 & 1;
          if (!(ok = mbar_wait(afull + st, (a2 >> 1) & 1, status))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + st * kCStageA), b0 = smem_u32(sB + k * stageB);
#pragma unroll
          for (int q = 0; q < kCBK / 16; ++q)
            mma_bf16(tmem + (uint32_t)(b * 32), desc_sw128(a0 + q * 32), desc_sw128(b0 + q * 32), idesc,
                     (k > 0 || q > 0) ? 1u : 0u);
          mma_commit(aempty + st);
        }
        mma_commit(tfull + b);
      }
    }
  } else {                                 // consumers
    const float4* p_lnw = reinterpret_cast<const float4*>(s_par);
    const float4* p_lnb = reinterpret_cast<const float4*>(s_par + d);
    const float4* p_w0 = reinterpret_cast<const float4*>(s_par + 2 * d);
    const float4* p_w1 = reinterpret_cast<const float4*>(s_par + 3 * d);
    const float4* p_g = reinterpret_cast<const float4*>(s_par + 4 * d);
    // the two threads of a tile row sit in the two half-warps (lanes l and l + 16): a quarter-warp's 16-byte reads of
    // the staged rows then cover eight different rows (eight distinct swizzled chunks, no bank conflict), where
    // adjacent lanes on the two boxes of one row would read the same banks 16 KB apart
    const int ar = (tid & 15) + 16 * (tid >> 5), ah = (tid >> 4) & 1;
    int q = 0, j = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++j) {
      const int64_t m0 = (int64_t)tile * kCTM;
      const int64_t ag = m0 + ar;
      const bool row_ok = ag < M;
      // ---- statistics: Welford over this thread's half of each chunk, merged with the partner thread; g(h) ------
      float cnt = 0.f, mean = 0.f, m2 = 0.f, gl = 0.f;
      for (int k = 0; k < nk; ++k, ++q) {
        const int sl = q % kCSlots;
        if (!(ok = mbar_wait(full + sl, (q / kCSlots) & 1, status))) break;
        const uint8_t* hs = sH + sl * kCSlot + ah * (kCSlot / 2) + ar * 128;
        float xs[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 x = *reinterpret_cast<const float4*>(hs + ((i ^ (ar & 7)) << 4));
          xs[4 * i] = x.x; xs[4 * i + 1] = x.y; xs[4 * i + 2] = x.z; xs[4 * i + 3] = x.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + sl);
        float sc = 0.f;
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          const float4 gw = p_g[(k * kCBK + ah * 32) / 4 + e4];
          const float gv[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
          for (int e = 4 * e4; e < 4 * e4 + 4; ++e) {
            sc += xs[e];
            gl = fmaf(xs[e], gv[e - 4 * e4], gl);
          }
        }
        const float mc = sc * (1.f / 32.f);
        float m2c = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) m2c = fmaf(xs[e] - mc, xs[e] - mc, m2c);
        const float n = cnt + 32.f;
        const float dl = mc - mean;
        mean += dl * (32.f / n);
        m2 += m2c + dl * dl * (cnt * 32.f / n);
        cnt = n;
      }
      if (!ok) break;
      {
        const float cnt_o = __shfl_xor_sync(0xffffffffu, cnt, 16);
        const float mean_o = __shfl_xor_sync(0xffffffffu, mean, 16);
        const float m2_o = __shfl_xor_sync(0xffffffffu, m2, 16);
        const float n = cnt + cnt_o;
        const float dl = mean_o - mean;
        mean = mean + dl * (cnt_o / n);
        m2 = m2 + m2_o + dl * dl * (cnt * cnt_o / n);
        gl += __shfl_xor_sync(0xffffffffu, gl, 16);
      }
      const float rstd = 1.f / sqrtf(m2 / (float)d + 1e-5f);
      // ---- normalise, clock projection in fp32, bf16 operand for Qc / Kc ------------------------------------------
      float u0 = 0.f, u1 = 0.f;
      for (int k = 0; k < nk; ++k, ++q) {
        const int sl = q % kCSlots;
        if (!(ok = mbar_wait(full + sl, (q / kCSlots) & 1, status))) break;
        const uint8_t* hs = sH + sl * kCSlot + ah * (kCSlot / 2) + ar * 128;
        const int a2 = j * nk + k, st = a2 & 1;
        if (a2 >= 2 && !(ok = mbar_wait(aempty + st, ((a2 >> 1) - 1) & 1, status))) break;
        uint8_t* dstA = sA + st * kCStageA;
        const int c0 = k * kCBK + ah * 32;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float hn[8];
          const float4 x0 = *reinterpret_cast<const float4*>(hs + (((2 * c) ^ (ar & 7)) << 4));
          const float4 x1 = *reinterpret_cast<const float4*>(hs + (((2 * c + 1) ^ (ar & 7)) << 4));
          const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          const int j4 = (c0 + c * 8) / 4;
          const float4 lw0 = p_lnw[j4], lw1 = p_lnw[j4 + 1], lb0 = p_lnb[j4], lb1 = p_lnb[j4 + 1];
          const float4 w00 = p_w0[j4], w01 = p_w0[j4 + 1], w10 = p_w1[j4], w11 = p_w1[j4 + 1];
          const float lw[8] = {lw0.x, lw0.y, lw0.z, lw0.w, lw1.x, lw1.y, lw1.z, lw1.w};
          const float lb[8] = {lb0.x, lb0.y, lb0.z, lb0.w, lb1.x, lb1.y, lb1.z, lb1.w};
          const float wa[8] = {w00.x, w00.y, w00.z, w00.w, w01.x, w01.y, w01.z, w01.w};
          const float wb[8] = {w10.x, w10.y, w10.z, w10.w, w11.x, w11.y, w11.z, w11.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            hn[e] = (xs[e] - mean) * rstd * lw[e] + lb[e];
            u0 = fmaf(hn[e], wa[e], u0);
            u1 = fmaf(hn[e], wb[e], u1);
          }
          *reinterpret_cast<uint4*>(dstA + sw128_offset(ar, ah * 4 + c)) =
              make_uint4(pack_bf16x2(hn[0], hn[1]), pack_bf16x2(hn[2], hn[3]), pack_bf16x2(hn[4], hn[5]),
                         pack_bf16x2(hn[6], hn[7]));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(empty + sl);
          mbar_arrive(afull + st);
        }
      }
      if (!ok) break;
      // scalar outputs (the partner threads of a row combine their halves)
      u0 += __shfl_xor_sync(0xffffffffu, u0, 16);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 16);
      if (ah == 0 && row_ok) {
        u0 += a.b_reloj[0];
        u1 += a.b_reloj[1];
        a.beta[ag] = (double)fminf(softplus_t(u0), a.beta_max);
        a.log_alfa[ag] = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
        a.glogit[ag] = gl + a.g_b[0];
        a.sig[ag] = (float)a.tokens[ag];
      }
      // Qc, Kc of the tile from accumulator j % 2 (warps 0-3: TMEM lanes 32 w .. + 31 are tile rows)
      if (wid < 4) {
        const int b = j & 1;
        if (!(ok = mbar_wait(tfull + b, (j >> 1) & 1, status))) break;
        tc_fence_after();
        const int r = wid * 32 + lane;
        const int64_t g = m0 + r;
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(wid * 32) << 16) + (uint32_t)(b * 32), v);
        if (g < M) {   // cf == 16: two 32-byte rows
          uint4* qq = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.Qc) + g * 16);
          uint4* kk = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.Kc) + g * 16);
          qq[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                             pack_bf16x2(v[6], v[7]));
          qq[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                             pack_bf16x2(v[14], v[15]));
          kk[0] = make_uint4(pack_bf16x2(v[16], v[17]), pack_bf16x2(v[18], v[19]), pack_bf16x2(v[20], v[21]),
                             pack_bf16x2(v[22], v[23]));
          kk[1] = make_uint4(pack_bf16x2(v[24], v[25]), pack_bf16x2(v[26], v[27]), pack_bf16x2(v[28], v[29]),
                             pack_bf16x2(v[30], v[31]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + b);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

static size_t context_tc_smem(int d, int cf) {
  return 1024 + (size_t)kCSlots * kCSlot + 2 * (size_t)kCStageA + (size_t)(d / kCBK) * (2 * cf) * 128 +
         kCBarBytes + 5 * (size_t)d * 4;
}

bool context_tc_supported(const ContextArgs& a) {
  return a.tokens != nullptr && a.d % kCBK == 0 && a.cf == 16 && context_tc_smem(a.d, a.cf) <= 227 * 1024;
}

int launch_context_tc(const ContextArgs& a, int* status, cudaStream_t s) {
  CUtensorMap map, hmap;
  const int64_t M = a.B * a.L;
  if (!make_tmap_bf16(&map, a.wctx, (uint64_t)a.d, (uint64_t)(2 * a.cf), (uint64_t)a.d * 2, 64, (uint32_t)(2 * a.cf)) ||
      !make_tmap_f32_sw128(&hmap, a.h, (uint64_t)a.d, (uint64_t)M, (uint64_t)a.d * 4, 32, kCTM))
    return ASRN_ERR_CUDA;
  const size_t smem = context_tc_smem(a.d, a.cf);
  if (smem > 227 * 1024) return ASRN_ERR_UNSUPPORTED;
  cudaFuncSetAttribute(k_context_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t ntiles = (M + kCTM - 1) / kCTM;
  if (ntiles >= ((int64_t)1 << 31)) return ASRN_ERR_UNSUPPORTED;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    nsm = 148;
  const int grid = (int)(ntiles < nsm ? ntiles : nsm);
  k_context_tc<<<grid, kCThreads, smem, s>>>(map, hmap, a, status, (int)ntiles);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
