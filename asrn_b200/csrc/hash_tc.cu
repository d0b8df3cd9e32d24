// Sign-hash projection on the 5th-generation tensor cores (bf16 autocast mode).
// Same computation as k_hash_simt (asrn/nucleo.py:644-664): per token
//   [hp | ca | cb] = E_t . [pal0; ctx0[:, :d]; ctx0[:, d:]]^T        (one M=128 x N=3m x K=d tcgen05 GEMM)
//   g1 = bf16(gelu(bf16(hp + b))),  g2 = bf16(gelu(bf16(ca_t + cb_{t-1} + b)))
//   phi = bf16([g1 | g2] . blockdiag(pal2, ctx2)^T + b2)               (one M=128 x N=Np x K=2m tcgen05 GEMM)
//   ids = sign bits of phi
// A tile covers 128 consecutive token rows starting one row early (stride 127): its first row only supplies
// cb_{t-1} of the second.
//
// Persistent and warp-specialised, one block per SM walking the tiles, so that the stream of E (the kernel's
// dominant traffic: 3 KB per token in, 1.5 KB of Ea out) never waits for an epilogue:
//   warp 4 (E producer) streams each tile's fp32 rows by TMA, 64 columns at a time (two 128 x 32 boxes, 128-byte
//     swizzle) through kES slots;
//   warps 0-3 (converters, one thread per tile row) round each chunk to bf16 into a two-stage operand ring in the
//     MMA's 128-byte-swizzled K-major layout and write it out as Ea (the value rows the scoring kernel gathers);
//   warp 5 streams the first-layer weight chunks (re-read from L2 for every tile) and, once, the resident second
//     layer; warp 6 issues the MMAs: each tile's first GEMM into one of two 256-column TMEM accumulators, and the
//     previous tile's second GEMM into the same accumulator once its epilogue has read it;
//   warps 8-15 (epilogue) drain the first GEMM (GELU of the word half by warps 8-11, of the context half with the
//     previous row's cb by warps 12-15), then the second one (phi and the ids, warps 8-11), while the next tile
//     streams in.
#include "common.cuh"
#include "layout.h"
#include "umma.cuh"

namespace asrn {

using namespace umma;

namespace {
constexpr int kTM = 128;             // rows per tile (TMEM lanes)
constexpr int kOut = 127;            // output rows per tile
constexpr int kBK = 64;              // K per chunk (one 128-byte swizzle atom of bf16)
constexpr int kStageA = kTM * 128;   // 16 KB
constexpr int kES = 2;               // E chunk slots (128 rows x 64 fp32 = 32 KB each)
constexpr int kESlot = 2 * kTM * 128;
constexpr int kThreads = 16 * 32;    // warps 0-3 converters, 4 E, 5 weights, 6 first GEMM, 7 second GEMM, 8-15 epilogue
constexpr int kEpi0 = 8;
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
  int ntiles;
};

__global__ void __launch_bounds__(kThreads, 1)
k_hash_tc(const __grid_constant__ CUtensorMap tmap_w1, const __grid_constant__ CUtensorMap tmap_w2,
          const __grid_constant__ CUtensorMap tmap_e, HashTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023) & ~1023u) - raw);
  const int N1 = 3 * p.m;                             // 192
  const int stageB = N1 * 128;
  const uint32_t atom_w2 = (uint32_t)p.Np * 128;
  uint8_t* sE = sm;                                   // [kES][2 boxes][128 rows][128 B]
  uint8_t* sA = sE + kES * kESlot;                    // [2][128 rows][128 B]
  uint8_t* sB = sA + 2 * kStageA;                     // [2][N1 rows][128 B]
  uint8_t* sG = sB + 2 * stageB;                      // [2 atoms][128 rows][128 B]
  uint8_t* sW2 = sG + 2 * kStageA;                    // [2 atoms][Np rows][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW2 + 2 * atom_w2);
  uint64_t* e_full = bars;          // [2]
  uint64_t* e_empty = bars + 2;     // [2]
  uint64_t* a_full = bars + 4;      // [2]
  uint64_t* a_empty = bars + 6;     // [2]
  uint64_t* w_full = bars + 8;      // [2]
  uint64_t* w_empty = bars + 10;    // [2]
  uint64_t* acc_full = bars + 12;   // [2] first GEMM of a tile done
  uint64_t* acc_empty = bars + 14;  // [2] accumulator drained by the second epilogue
  uint64_t* g_full = bars + 16;     // G written (first epilogue done)
  uint64_t* phi_full = bars + 17;   // second GEMM done (G free again)
  uint64_t* w2_full = bars + 18;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(bars + 20);
  float* xch = reinterpret_cast<float*>(bars + 24);   // [4 warps][64] cb of each warp's last row

  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int d = p.d;
  const int nk = d / kBK;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(e_full + i, 1);
      mbar_init(e_empty + i, 4);          // the four converter warps
      mbar_init(a_full + i, 4);
      mbar_init(a_empty + i, 1);
      mbar_init(w_full + i, 1);
      mbar_init(w_empty + i, 1);
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 4);        // epilogue warps 8-11
    }
    mbar_init(g_full, 8);                 // all eight epilogue warps
    mbar_init(phi_full, 1);
    mbar_init(w2_full, 1);
    fence_mbar_init();
    prefetch_tensormap(&tmap_w1);
    prefetch_tensormap(&tmap_w2);
    prefetch_tensormap(&tmap_e);
  }
  if (wid == 6) {
    tmem_alloc(tmem_base_s, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;
  int* status = p.status;

  if (wid < 4) {
    // ---- converters: thread = tile row ------------------------------------------------------------------------
    const int r = tid;
    int ck = 0;                                       // chunk counter over all tiles
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
      const int64_t g = (int64_t)tile * kOut - 1 + r;
      const bool store_ea = r >= 1 && g < p.M;
      uint4* ea = reinterpret_cast<uint4*>(p.Ea + (store_ea ? g : 0) * (int64_t)d);
      for (int k = 0; k < nk; ++k, ++ck) {
        const int es = ck % kES, as = ck & 1;
        if (!(ok = mbar_wait(e_full + es, (uint32_t)((ck / kES) & 1), status))) break;
        if (ck >= 2 && !(ok = mbar_wait(a_empty + as, (uint32_t)(((ck - 2) >> 1) & 1), status))) break;
        const uint8_t* src = sE + es * kESlot + r * 128;
        uint8_t* dstA = sA + as * kStageA;
        uint4 q[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {           // 16-byte granule c of the 64-column chunk: box c / 4, granule 2 c, + 1
          const uint8_t* bx = src + (c >> 2) * (kTM * 128);
          const int g0 = (2 * c) & 7;
          const float4 x0 = *reinterpret_cast<const float4*>(bx + ((g0 ^ (r & 7)) << 4));
          const float4 x1 = *reinterpret_cast<const float4*>(bx + (((g0 + 1) ^ (r & 7)) << 4));
          q[c] = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                            pack_bf16x2(x1.z, x1.w));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(e_empty + es);   // the fp32 slot is read
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dstA + sw128_offset(r, c)) = q[c];
        if (store_ea) {
#pragma unroll
          for (int c = 0; c < 8; ++c) ea[k * 8 + c] = q[c];
        }
        fence_proxy_async();                      // the operand stores precede the tensor cores' reads
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + as);
      }
    }
  } else if (wid == 4) {
    // ---- E producer -----------------------------------------------------------------------------------------------
    if (lane == 0) {
      int ck = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
        const int y = tile * kOut - 1;            // row -1 of the first tile reads zeros
        for (int k = 0; k < nk; ++k, ++ck) {
          const int es = ck % kES;
          if (ck >= kES && !(ok = mbar_wait(e_empty + es, (uint32_t)(((ck / kES) - 1) & 1), status))) break;
          mbar_expect_tx(e_full + es, (uint32_t)kESlot);
          tma_load_2d(sE + es * kESlot, &tmap_e, k * kBK, y, e_full + es);
          tma_load_2d(sE + es * kESlot + kTM * 128, &tmap_e, k * kBK + 32, y, e_full + es);
        }
      }
      // every issued copy has landed before the block may exit (bounded)
      if (ck > 0) mbar_wait(e_full + ((ck - 1) % kES), (uint32_t)(((ck - 1) / kES) & 1), status);
    }
  } else if (wid == 5) {
    // ---- weights: the resident second layer once, the first layer's chunks for every tile ---------------------------
    if (lane == 0) {
      mbar_expect_tx(w2_full, 2 * atom_w2);
      tma_load_2d(sW2, &tmap_w2, 0, 0, w2_full);
      tma_load_2d(sW2 + atom_w2, &tmap_w2, 64, 0, w2_full);
      int ck = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
        for (int k = 0; k < nk; ++k, ++ck) {
          const int ws = ck & 1;
          if (ck >= 2 && !(ok = mbar_wait(w_empty + ws, (uint32_t)(((ck - 2) >> 1) & 1), status))) break;
          mbar_expect_tx(w_full + ws, (uint32_t)stageB);
          tma_load_2d(sB + ws * stageB, &tmap_w1, k * kBK, 0, w_full + ws);
        }
      }
      mbar_wait(w2_full, 0, status);
      if (ck > 0) mbar_wait(w_full + ((ck - 1) & 1), (uint32_t)(((ck - 1) >> 1) & 1), status);
    }
  } else if (wid == 6) {
    // ---- first GEMM issuer ------------------------------------------------------------------------------------------
    if (lane == 0) {
      const uint32_t idesc1 = idesc_bf16(kTM, N1);
      int ck = 0, j = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x, ++j) {
        const int ab = j & 1;
        if (j >= 2) ok = mbar_wait(acc_empty + ab, (uint32_t)(((j - 2) >> 1) & 1), status);
        tc_fence_after();
        for (int k = 0; k < nk && ok; ++k, ++ck) {
          const int as = ck & 1;
          if (!(ok = mbar_wait(a_full + as, (uint32_t)((ck >> 1) & 1), status))) break;
          if (!(ok = mbar_wait(w_full + as, (uint32_t)((ck >> 1) & 1), status))) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + as * kStageA), b0 = smem_u32(sB + as * stageB);
#pragma unroll
          for (int q = 0; q < kBK / 16; ++q)
            mma_bf16(tmem + (uint32_t)(ab * 256), desc_sw128(a0 + q * 32), desc_sw128(b0 + q * 32), idesc1,
                     (k > 0 || q > 0) ? 1u : 0u);
          mma_commit(a_empty + as);
          mma_commit(w_empty + as);
        }
        if (ok) mma_commit(acc_full + ab);
      }
    }
  } else if (wid == 7) {
    // ---- second GEMM issuer: phi of tile j into its accumulator once G is written -----------------------------------
    if (lane == 0) {
      const uint32_t idesc2 = idesc_bf16(kTM, p.Np);
      bool ok = mbar_wait(w2_full, 0, status);
      int j = 0;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x, ++j) {
        const int ab = j & 1;
        if (!(ok = mbar_wait(g_full, (uint32_t)(j & 1), status))) break;
        tc_fence_after();
        const uint32_t g_a = smem_u32(sG), w_a = smem_u32(sW2);
#pragma unroll
        for (int atom = 0; atom < 2; ++atom)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            mma_bf16(tmem + (uint32_t)(ab * 256), desc_sw128(g_a + atom * kStageA + q * 32),
                     desc_sw128(w_a + atom * atom_w2 + q * 32), idesc2, (atom > 0 || q > 0) ? 1u : 0u);
        mma_commit(phi_full);
      }
    }
  } else if (wid >= kEpi0) {
    // ---- epilogue: thread = tile row (TMEM lane) --------------------------------------------------------------------
    const int ew = wid - kEpi0, q4 = ew & 3;
    const int r = q4 * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    int j = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++j) {
      const int ab = j & 1;
      const int64_t g = (int64_t)tile * kOut - 1 + r;
      const uint32_t tacc = trow + (uint32_t)(ab * 256);
      if (!(ok = mbar_wait(acc_full + ab, (uint32_t)((j >> 1) & 1), status))) break;
      // G of the previous tile has been consumed by its second GEMM before it is rewritten
      if (j >= 1 && !(ok = mbar_wait(phi_full, (uint32_t)((j - 1) & 1), status))) break;
      tc_fence_after();
      if (ew < 4) {                              // word tables: g1 = bf16(gelu(bf16(hp + b)))
        for (int hh = 0; hh < 2; ++hh) {
          float v[32];
          tmem_ld32(tacc + hh * 32, v);
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
      } else {                                   // context tables: g2 = bf16(gelu(bf16(ca_t + cb_{t-1} + b)))
        const bool seq_start = (g >= 0) && (g % p.L == 0);
        for (int hh = 0; hh < 2; ++hh) {
          float cb[32], ca[32];
          tmem_ld32(tacc + 2 * p.m + hh * 32, cb);
          tmem_ld32(tacc + p.m + hh * 32, ca);
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
            *reinterpret_cast<uint4*>(sG + kStageA + sw128_offset(r, hh * 4 + c)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      fence_proxy_async();                       // G precedes the second GEMM's reads
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(g_full);
      if (ew < 4) {
        // phi = bf16(acc + b2), its sign bits -> bucket ids (tcgen05.ld is warp-collective: every lane loads)
        if (!(ok = mbar_wait(phi_full, (uint32_t)(j & 1), status))) break;
        tc_fence_after();
        const bool out_row = r >= 1 && g < p.M;
        const int64_t gs = out_row ? g : 0;
        const int64_t b = gs / p.L, t = gs % p.L;
        uint32_t sgn[8] = {0, 0, 0, 0, 0, 0, 0, 0};   // bit o of the 256-bit mask: phi_o > 0
        __nv_bfloat16* prow = p.phi + gs * (int64_t)p.P;
        for (int qc = 0; qc * 32 < p.P; ++qc) {
          float v[32];
          tmem_ld32(tacc + qc * 32, v);
          uint32_t w[16], bits = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int o = qc * 32 + i;
            float x = 0.f;
            if (o < p.P) x = round_bf16(v[i] + p.b2[o]);
            bits |= (x > 0.f ? 1u : 0u) << i;
            v[i] = x;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (i == qc) sgn[i] = bits;
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
        if (out_row) {
          // table tau's id = bits tau nb .. + nb - 1 of the mask (nb <= 16: within two consecutive words)
          for (int tau = 0; tau < p.T; ++tau) {
            const int o0 = tau * p.nb, wi = o0 >> 5, sh = o0 & 31;
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (i == wi) lo = sgn[i];
              if (i == wi + 1) hi = sgn[i];
            }
            const uint32_t id = __funnelshift_r(lo, hi, sh) & ((1u << p.nb) - 1u);
            p.ids_rows[((int64_t)b * p.T + tau) * p.L + t] = (uint16_t)id;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + ab);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 6) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

size_t hash_tc_smem_bytes(int m, int Np) {
  return 1024 + kES * (size_t)kESlot + 2 * (size_t)kStageA + 2 * (size_t)(3 * m) * 128 + 2 * (size_t)kStageA +
         2 * (size_t)Np * 128 + 24 * 8 + 4 * 64 * 4;
}

bool hash_tc_supported(const HashArgs& a) {
  return a.m == 64 && a.d % kBK == 0 && a.d >= kBK && a.P <= 256 && a.T <= kMaxTables && a.nb <= 16;
}

static int sm_count_hash() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
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
  const int64_t ntiles = (p.M + kOut - 1) / kOut;
  if (ntiles >= ((int64_t)1 << 31) || p.Np > 256) return ASRN_ERR_UNSUPPORTED;
  p.ntiles = (int)ntiles;
  // E (fp32, (M, d)) as 128 x 32 boxes with the 128-byte swizzle; rows outside [0, M) read zeros
  CUtensorMap te;
  if (!make_tmap_f32_sw128(&te, a.E, (uint64_t)a.d, (uint64_t)p.M, (uint64_t)a.d * 4, 32, kTM)) return ASRN_ERR_CUDA;
  const size_t smem = hash_tc_smem_bytes(a.m, p.Np);
  if (smem > 227 * 1024) return ASRN_ERR_UNSUPPORTED;
  cudaFuncSetAttribute(k_hash_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const unsigned grid = (unsigned)(ntiles < sm_count_hash() ? ntiles : sm_count_hash());
  k_hash_tc<<<grid, kThreads, smem, s>>>(w1, w2, te, p);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
