// Sign-hash projection on the 5th-generation tensor cores (bf16 autocast mode).
// Same computation as k_hash_simt (asrn/nucleo.py:644-664): per token
//   [hp | ca | cb] = E_t . [pal0; ctx0[:, :d]; ctx0[:, d:]]^T        (one M=128 x N=3m x K=d tcgen05 GEMM)
//   g1 = bf16(gelu(bf16(hp + b))),  g2 = bf16(gelu(bf16(ca_t + cb_{t-1} + b)))
//   phi = bf16([g1 | g2] . blockdiag(pal2, ctx2)^T + b2)               (one M=128 x N=Np x K=2m tcgen05 GEMM)
//   ids = sign bits of phi
// A tile covers 128 consecutive token rows starting one row early (stride 127): its first row only supplies
// cb_{t-1} of the second. The fp32 rows of E are loaded by the threads, rounded to bf16 (written out as Ea, the
// value rows the scoring kernel gathers) and stored in the 128-byte-swizzled K-major layout; the weight tiles
// arrive by TMA; the fp32 accumulators live in TMEM (256 columns, so two blocks share an SM).
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

using namespace umma;

namespace {
constexpr int kTM = 128;             // rows per tile (TMEM lanes)
constexpr int kOut = 127;            // output rows per tile
constexpr int kBK = 64;              // K per stage (one 128-byte swizzle atom of bf16)
constexpr int kStageA = kTM * 128;   // 16 KB
constexpr int kThreads = 256;
}  // namespace

struct HashTcParams {
  int64_t M, L;
  int d, m, T, Tw, nb, P, Np;
  const float* E;
  __nv_bfloat16* Ea;
  const float* b1;
  const float* b2;
  __nv_bfloat16* phi;
  uint16_t* ids_rows;
  int* status;
};

__global__ void __launch_bounds__(kThreads, 2)
k_hash_tc(const __grid_constant__ CUtensorMap tmap_w1, const __grid_constant__ CUtensorMap tmap_w2, HashTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  const int N1 = 3 * p.m;
  const int stageB = N1 * 128;
  uint8_t* sA = sm;                                   // [2][kStageA]
  uint8_t* sB = sm + 2 * kStageA;                     // [2][stageB]
  uint8_t* sG = sm;                                   // after the main loop: [2 atoms][128 rows][128 B]
  uint8_t* sW2 = sm + 2 * kStageA;                    // after the main loop: [2 atoms][Np rows][128 B]
  uint8_t* tail = sm + 2 * kStageA + 2 * stageB;
  uint64_t* full_b = reinterpret_cast<uint64_t*>(tail);        // [2]
  uint64_t* mma_done = full_b + 2;                             // [2]
  uint64_t* w2_full = full_b + 4;
  uint64_t* phi_done = full_b + 5;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(full_b + 6);
  int* abort_s = reinterpret_cast<int*>(tmem_base_s + 1);
  float* xch = reinterpret_cast<float*>(tmem_base_s + 4);      // [4 warps][64] cb of each warp's last row

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t g0 = (int64_t)blockIdx.x * kOut - 1;          // global row of tile row 0
  const int d = p.d;
  const int nk = d / kBK;

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(full_b + i, 1);
    *abort_s = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_w1);
    prefetch_tensormap(&tmap_w2);
  }
  if (wid == 0) {
    tmem_alloc(tmem_base_s, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  // A-operand producer mapping: thread -> (row r, 32-column half h) of each 128 x 64 chunk
  const int ar = tid >> 1, ah = tid & 1;
  const int64_t ag = g0 + ar;
  const bool arow_ok = ag >= 0 && ag < p.M;
  const float* erow = p.E + (arow_ok ? ag : 0) * (int64_t)d + ah * 32;
  float4 pre[8];
  auto load_chunk = [&](int k) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      pre[i] = arow_ok ? __ldg(reinterpret_cast<const float4*>(erow + k * kBK) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  load_chunk(0);
  const uint32_t idesc1 = idesc_bf16(kTM, N1);
  // weight chunk k arrives one step ahead: chunk 0 here, chunk k + 1 once the MMAs of chunk k - 1 (its stage) are done
  auto issue_w1 = [&](int k) {
    const int s = k & 1;
    mbar_expect_tx(full_b + s, (uint32_t)stageB);
    tma_load_2d(sB + s * stageB, &tmap_w1, k * kBK, 0, full_b + s);
  };
  if (tid == 0) issue_w1(0);
  bool ok = true;
  for (int k = 0; k < nk; ++k) {
    const int s = k & 1;
    if (k >= 2) ok = mbar_wait(mma_done + s, ((k - 2) >> 1) & 1, p.status) && ok;
    // convert this thread's 32 fp32 values to bf16: 4 chunks of 16 bytes
    uint8_t* dstA = sA + s * kStageA;
    uint4 q[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 x0 = pre[2 * c], x1 = pre[2 * c + 1];
      q[c] = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                        pack_bf16x2(x1.z, x1.w));
      *reinterpret_cast<uint4*>(dstA + sw128_offset(ar, ah * 4 + c)) = q[c];
    }
    if (arow_ok && ar >= 1) {
      uint4* ea = reinterpret_cast<uint4*>(p.Ea + ag * (int64_t)d + k * kBK + ah * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c) ea[c] = q[c];
    }
    if (k + 1 < nk) load_chunk(k + 1);
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      if (ok) ok = mbar_wait(full_b + s, (k >> 1) & 1, p.status);
      if (ok) {
        const uint32_t a0 = smem_u32(dstA), b0 = smem_u32(sB + s * stageB);
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j)
          mma_bf16(tmem, desc_sw128(a0 + j * 32), desc_sw128(b0 + j * 32), idesc1, (k > 0 || j > 0) ? 1u : 0u);
      }
      mma_commit(mma_done + s);
      if (ok && k + 1 < nk) {
        if (k >= 1) ok = mbar_wait(mma_done + (s ^ 1), ((k - 1) >> 1) & 1, p.status);
        if (ok) issue_w1(k + 1);
      }
      if (!ok) *abort_s = 1;
    }
  }
  ok = mbar_wait(mma_done + ((nk - 1) & 1), ((nk - 1) >> 1) & 1, p.status) && ok;
  if (nk >= 2) ok = mbar_wait(mma_done + ((nk - 2) & 1), ((nk - 2) >> 1) & 1, p.status) && ok;
  tc_fence_after();
  __syncthreads();
  if (!ok) *abort_s = 1;
  __syncthreads();
  const bool aborted = *abort_s != 0;

  // the stage buffers are free: bring in the second-layer weights while the first epilogue runs
  if (tid == 0 && !aborted) {
    const uint32_t atom_w2 = (uint32_t)p.Np * 128;
    mbar_expect_tx(w2_full, 2 * atom_w2);
    tma_load_2d(sW2, &tmap_w2, 0, 0, w2_full);
    tma_load_2d(sW2 + atom_w2, &tmap_w2, 64, 0, w2_full);
  }

  // ---- epilogue 1: hp -> g1 (warps 0-3), [ca, cb] -> g2 (warps 4-7); rows are TMEM lanes -------------------------
  const int q4 = wid & 3;
  const int r = q4 * 32 + lane;                      // tile row of this thread
  const int64_t g = g0 + r;
  const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
  if (!aborted) {
    if (wid < 4) {
      for (int hh = 0; hh < 2; ++hh) {
        float v[32];
        tmem_ld32(trow + hh * 32, v);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c0 = hh * 32 + 2 * i;
          const float a0 = gelu_t(round_bf16(v[2 * i] + p.b1[c0]));
          const float a1 = gelu_t(round_bf16(v[2 * i + 1] + p.b1[c0 + 1]));
          w[i] = pack_bf16x2(a0, a1);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(sG + sw128_offset(r, hh * 4 + c)) = make_uint4(w[4 * c], w[4 * c + 1],
                                                                                   w[4 * c + 2], w[4 * c + 3]);
      }
    } else {
      const bool seq_start = (g >= 0) && (g % p.L == 0);
      for (int hh = 0; hh < 2; ++hh) {
        float cb[32], ca[32];
        tmem_ld32(trow + 2 * p.m + hh * 32, cb);
        tmem_ld32(trow + p.m + hh * 32, ca);
        if (lane == 31) {
#pragma unroll
          for (int i = 0; i < 32; ++i) xch[q4 * 64 + hh * 32 + i] = cb[i];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float pr[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float up = __shfl_up_sync(0xffffffffu, cb[i + e], 1);
            if (lane == 0) up = (q4 > 0) ? xch[(q4 - 1) * 64 + hh * 32 + i + e] : 0.f;
            if (seq_start) up = 0.f;
            const int col = p.m + hh * 32 + i + e;
            pr[e] = gelu_t(round_bf16((ca[i + e] + up) + p.b1[col]));
          }
          w[i / 2] = pack_bf16x2(pr[0], pr[1]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(sG + 16384 + sw128_offset(r, hh * 4 + c)) =
              make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && !aborted) {
    tc_fence_after();
    bool ok2 = mbar_wait(w2_full, 0, p.status);
    if (ok2) {
      const uint32_t g_a = smem_u32(sG), w_a = smem_u32(sW2);
      const uint32_t atom_w2 = (uint32_t)p.Np * 128;
      const uint32_t idesc2 = idesc_bf16(kTM, p.Np);
#pragma unroll
      for (int atom = 0; atom < 2; ++atom)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16(tmem, desc_sw128(g_a + atom * 16384 + j * 32), desc_sw128(w_a + atom * atom_w2 + j * 32), idesc2,
                   (atom > 0 || j > 0) ? 1u : 0u);
    } else {
      *abort_s = 1;
    }
    mma_commit(phi_done);
  }
  __syncthreads();
  bool ok3 = !aborted && *abort_s == 0;
  if (ok3) ok3 = mbar_wait(phi_done, 0, p.status);
  tc_fence_after();

  // ---- epilogue 2: phi = bf16(acc + b2), its sign bits -> bucket ids (warps 0-3) ---------------------------------
  // tcgen05.ld is warp-collective: every lane of warps 0-3 loads, only output rows store
  if (ok3 && wid < 4) {
    const bool out_row = r >= 1 && g < p.M;
    const int64_t gs = out_row ? g : 0;
    const int64_t b = gs / p.L, t = gs % p.L;
    uint32_t ids[kMaxTables];
#pragma unroll
    for (int i = 0; i < kMaxTables; ++i) ids[i] = 0;
    __nv_bfloat16* prow = p.phi + gs * (int64_t)p.P;
    for (int qc = 0; qc * 32 < p.P; ++qc) {
      float v[32];
      tmem_ld32(trow + qc * 32, v);
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int o = qc * 32 + i;
        float x = 0.f;
        if (o < p.P) {
          x = round_bf16(v[i] + p.b2[o]);
          const int tau = o / p.nb;
#pragma unroll
          for (int tt = 0; tt < kMaxTables; ++tt)
            if (tt == tau && x > 0.f) ids[tt] |= 1u << (o - tau * p.nb);
        }
        v[i] = x;
      }
      if (out_row) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
        const int nvalid = min(32, p.P - qc * 32);
        if (nvalid == 32 && (p.P % 8) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(prow + qc * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c) dst[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
        } else {
          for (int i = 0; i < nvalid; ++i) prow[qc * 32 + i] = __float2bfloat16_rn(v[i]);
        }
      }
    }
    if (out_row)
      for (int tau = 0; tau < p.T; ++tau) p.ids_rows[((int64_t)b * p.T + tau) * p.L + t] = (uint16_t)ids[tau];
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

size_t hash_tc_smem_bytes(int m) { return 1024 + 2 * (size_t)kStageA + 2 * (size_t)(3 * m) * 128 + 64 + 16 + 4 * 64 * 4; }

bool hash_tc_supported(const HashArgs& a) {
  return a.m == 64 && a.d % kBK == 0 && a.d >= kBK && a.P <= 256 && a.T <= kMaxTables && a.nb <= 16;
}

int launch_hash_tc(const HashArgs& a, const CUtensorMap& w1, const CUtensorMap& w2, cudaStream_t s) {
  HashTcParams p;
  p.M = a.B * a.L;
  p.L = a.L;
  p.d = a.d; p.m = a.m; p.T = a.T; p.Tw = a.Tw; p.nb = a.nb; p.P = a.P; p.Np = (a.P + 15) / 16 * 16;
  p.E = a.E;
  p.Ea = reinterpret_cast<__nv_bfloat16*>(a.Ea);
  p.b1 = a.b1;
  p.b2 = a.b2;
  p.phi = reinterpret_cast<__nv_bfloat16*>(a.phi);
  p.ids_rows = a.ids_rows;
  p.status = a.status;
  const size_t smem = hash_tc_smem_bytes(a.m);
  cudaFuncSetAttribute(k_hash_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const unsigned grid = (unsigned)((p.M + kOut - 1) / kOut);
  k_hash_tc<<<grid, kThreads, smem, s>>>(w1, w2, p);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
