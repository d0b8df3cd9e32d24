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
constexpr int kCTM = 128, kCBK = 64, kCThreads = 256;
constexpr int kCStageA = kCTM * 128;
}  // namespace

__global__ void __launch_bounds__(kCThreads, 2)
k_context_tc(const __grid_constant__ CUtensorMap tmap_wctx, ContextArgs a, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  const int N = 2 * a.cf;
  const int stageB = N * 128;
  uint8_t* sA = sm;
  uint8_t* sB = sm + 2 * kCStageA;                  // all d / 64 weight chunks, resident (2cf x 64 each)
  uint8_t* tail = sB + (a.d / kCBK) * stageB;
  uint64_t* full_b = reinterpret_cast<uint64_t*>(tail);
  uint64_t* mma_done = full_b + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(full_b + 4);
  int* abort_s = reinterpret_cast<int*>(tmem_base_s + 1);
  // per-column parameters, read as float4 from shared memory: ln_w, ln_b, w_reloj[0], w_reloj[1], g_w
  float* s_par = reinterpret_cast<float*>(tail + 64);

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int d = a.d;
  const int nk = d / kCBK;
  const int64_t M = a.B * a.L;
  const int64_t m0 = (int64_t)blockIdx.x * kCTM;
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(full_b + i, 1);
    *abort_s = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_wctx);
  }
  if (wid == 0) {
    tmem_alloc(tmem_base_s, 32);
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
  const float4* p_lnw = reinterpret_cast<const float4*>(s_par);
  const float4* p_lnb = reinterpret_cast<const float4*>(s_par + d);
  const float4* p_w0 = reinterpret_cast<const float4*>(s_par + 2 * d);
  const float4* p_w1 = reinterpret_cast<const float4*>(s_par + 3 * d);
  const float4* p_g = reinterpret_cast<const float4*>(s_par + 4 * d);

  const int ar = tid >> 1, ah = tid & 1;
  const int64_t ag = m0 + ar;
  const bool row_ok = ag < M;
  const float* hrow = a.h + (row_ok ? ag : 0) * (int64_t)d + ah * 32;

  // ---- statistics: Welford over this thread's half row, merged with the partner thread; g(h) partial --------------
  // per 32-value chunk: its mean and centred sum of squares, merged into the running (count, mean, M2) (Chan et al.)
  float cnt = 0.f, mean = 0.f, m2 = 0.f, gl = 0.f;
  for (int k = 0; k < nk; ++k) {
    float xs[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 x = row_ok ? __ldg(reinterpret_cast<const float4*>(hrow + k * kCBK) + i)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      xs[4 * i] = x.x; xs[4 * i + 1] = x.y; xs[4 * i + 2] = x.z; xs[4 * i + 3] = x.w;
    }
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
  {
    const float cnt_o = __shfl_xor_sync(0xffffffffu, cnt, 1);
    const float mean_o = __shfl_xor_sync(0xffffffffu, mean, 1);
    const float m2_o = __shfl_xor_sync(0xffffffffu, m2, 1);
    const float n = cnt + cnt_o;
    const float dl = mean_o - mean;
    mean = mean + dl * (cnt_o / n);
    m2 = m2 + m2_o + dl * dl * (cnt * cnt_o / n);
    gl += __shfl_xor_sync(0xffffffffu, gl, 1);
  }
  const float rstd = 1.f / sqrtf(m2 / (float)d + 1e-5f);

  // ---- main loop: normalise, clock projection in fp32, bf16 operand for Qc/Kc --------------------------------------
  float4 pre[8];
  auto load_chunk = [&](int k) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pre[i] = row_ok ? __ldg(reinterpret_cast<const float4*>(hrow + k * kCBK) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  load_chunk(0);
  float u0 = 0.f, u1 = 0.f;
  const uint32_t idesc = idesc_bf16(kCTM, N);
  bool ok = true;
  for (int k = 0; k < nk; ++k) {
    const int s = k & 1;
    if (k >= 2) ok = mbar_wait(mma_done + s, ((k - 2) >> 1) & 1, status) && ok;
    if (k == 0 && tid == 0) {        // the whole [cq; ck] at once, on one barrier: no per-chunk weight wait
      mbar_expect_tx(full_b, (uint32_t)(nk * stageB));
      for (int kk = 0; kk < nk; ++kk) tma_load_2d(sB + kk * stageB, &tmap_wctx, kk * kCBK, 0, full_b);
    }
    uint8_t* dstA = sA + s * kCStageA;
    const int c0 = k * kCBK + ah * 32;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float hn[8];
      const float4 x0 = pre[2 * c], x1 = pre[2 * c + 1];
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
    if (k + 1 < nk) load_chunk(k + 1);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (ok && k == 0) ok = mbar_wait(full_b, 0u, status);
      if (ok) {
        const uint32_t a0 = smem_u32(dstA), b0 = smem_u32(sB + k * stageB);
#pragma unroll
        for (int j = 0; j < kCBK / 16; ++j)
          mma_bf16(tmem, desc_sw128(a0 + j * 32), desc_sw128(b0 + j * 32), idesc, (k > 0 || j > 0) ? 1u : 0u);
      }
      mma_commit(mma_done + s);
      if (!ok) *abort_s = 1;
    }
  }
  // scalar outputs (the partner threads of a row combine their halves)
  u0 += __shfl_xor_sync(0xffffffffu, u0, 1);
  u1 += __shfl_xor_sync(0xffffffffu, u1, 1);
  if (ah == 0 && row_ok) {
    u0 += a.b_reloj[0];
    u1 += a.b_reloj[1];
    a.beta[ag] = (double)fminf(softplus_t(u0), a.beta_max);
    a.log_alfa[ag] = fmaxf(logsigmoid_t(u1) + 0.693147180559945309f, a.log_alfa_min);
    a.glogit[ag] = gl + a.g_b[0];
    a.sig[ag] = (float)a.tokens[ag];
  }
  ok = mbar_wait(mma_done + ((nk - 1) & 1), ((nk - 1) >> 1) & 1, status) && ok;
  if (nk >= 2) ok = mbar_wait(mma_done + ((nk - 2) & 1), ((nk - 2) >> 1) & 1, status) && ok;
  tc_fence_after();
  __syncthreads();
  if (!ok) *abort_s = 1;
  __syncthreads();
  if (*abort_s == 0 && wid < 4) {
    const int r = wid * 32 + lane;
    const int64_t g = m0 + r;
    float v[32];
    tmem_ld32(tmem + ((uint32_t)(wid * 32) << 16), v);
    if (g < M) {   // cf == 16: two 32-byte rows
      uint4* q = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.Qc) + g * 16);
      uint4* kk = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.Kc) + g * 16);
      q[0] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
      q[1] = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                        pack_bf16x2(v[14], v[15]));
      kk[0] = make_uint4(pack_bf16x2(v[16], v[17]), pack_bf16x2(v[18], v[19]), pack_bf16x2(v[20], v[21]),
                         pack_bf16x2(v[22], v[23]));
      kk[1] = make_uint4(pack_bf16x2(v[24], v[25]), pack_bf16x2(v[26], v[27]), pack_bf16x2(v[28], v[29]),
                         pack_bf16x2(v[30], v[31]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

bool context_tc_supported(const ContextArgs& a) {
  return a.tokens != nullptr && a.d % kCBK == 0 && a.d <= 1024 && a.cf == 16;
}

int launch_context_tc(const ContextArgs& a, int* status, cudaStream_t s) {
  CUtensorMap map;
  if (!make_tmap_bf16(&map, a.wctx, (uint64_t)a.d, (uint64_t)(2 * a.cf), (uint64_t)a.d * 2, 64, (uint32_t)(2 * a.cf)))
    return ASRN_ERR_CUDA;
  const size_t smem = 1024 + 2 * (size_t)kCStageA + (size_t)(a.d / kCBK) * (2 * a.cf) * 128 + 64 + 5 * (size_t)a.d * 4;
  cudaFuncSetAttribute(k_context_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t M = a.B * a.L;
  k_context_tc<<<(unsigned)((M + kCTM - 1) / kCTM), kCThreads, smem, s>>>(map, a, status);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
