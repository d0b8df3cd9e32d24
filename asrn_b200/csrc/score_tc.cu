// Candidate scoring on tensor cores (bf16 autocast mode). Same computation as k_score_simt (asrn/estable.py:204-300,
// asrn/nucleo.py:279-382), organised per block of 32 sorted query slots:
//   window = the 64 sorted slots [q0 - 32, q0 + 32) of the row (the previous block + the current block); features
//   (phi, Qc, Kc, clock, log_alfa, previous signatures) of each slot are gathered once into a 64-slot ring, and so
//   are the value rows Ea[pos + 1] of the slots some query can use (a slot is a candidate of somebody only if the
//   next sorted slot is in the same bucket; other rows are zero-filled without reading memory);
//   S = phi_q . phi_k and Qc . Kc (32 x 64 each) on mma.sync (fp32 accumulate), then the reference's rounding chain,
//   suffix weight, log_alfa_k and the fp64 time difference, the exact-mask softmax per query, and
//   out (32 x d_part) = att (32 x 64, bf16) . V (64 x d_part) on mma.sync, added into acc with vector reductions.
// d is split over ceil(d / 384) blocks per span so that a block's value ring stays small enough for two blocks per SM.
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {
constexpr int kQ = 32;          // queries per sub-tile
constexpr int kW = 64;          // window slots
constexpr int kSpanTc = 512;    // sorted slots per block
constexpr int kThreadsTc = 256;

struct TcSmem {
  int* pos;
  int* id;
  int* used;
  double* bt;
  float* la;
  float* pf;
  __nv_bfloat16* phi;   // [64][Pp]
  __nv_bfloat16* qc;    // [64][Cp]
  __nv_bfloat16* kc;    // [64][Cp]
  __nv_bfloat16* v;     // [64][Dp]
  float* sc;            // [32][65]
  __nv_bfloat16* att;   // [32][72]
  int* qhay;            // [32]
  int Pp, Cp, Dp, K;
};

__host__ __device__ inline int pad16(int x) { return (x + 15) / 16 * 16; }

__host__ __device__ inline size_t tc_smem_bytes(int P, int cf, int K, int dpart) {
  const int Pp = pad16(P) + 8, Cp = pad16(cf) + 8, Dp = dpart + 8;
  size_t b = 0;
  b += kW * 8;                    // bt
  b += kW * 4 * 3;                // pos, id, used
  b += kW * 4;                    // la
  b += kW * 4 * (size_t)K;        // pf
  b = (b + 15) / 16 * 16;
  b += (size_t)kW * Pp * 2 + 2 * (size_t)kW * Cp * 2 + (size_t)kW * Dp * 2;
  b += (size_t)kQ * 65 * 4;
  b += (size_t)kQ * 72 * 2;
  b += kQ * 4;
  return b + 16;
}

__device__ inline TcSmem carve_tc(char* base, int P, int cf, int K, int dpart) {
  TcSmem s;
  s.Pp = pad16(P) + 8;
  s.Cp = pad16(cf) + 8;
  s.Dp = dpart + 8;
  s.K = K;
  char* p = base;
  s.bt = reinterpret_cast<double*>(p); p += kW * 8;
  s.pos = reinterpret_cast<int*>(p); p += kW * 4;
  s.id = reinterpret_cast<int*>(p); p += kW * 4;
  s.used = reinterpret_cast<int*>(p); p += kW * 4;
  s.la = reinterpret_cast<float*>(p); p += kW * 4;
  s.pf = reinterpret_cast<float*>(p); p += kW * 4 * K;
  p = base + ((p - base) + 15) / 16 * 16;
  s.phi = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kW * s.Pp * 2;
  s.qc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kW * s.Cp * 2;
  s.kc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kW * s.Cp * 2;
  s.v = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kW * s.Dp * 2;
  s.sc = reinterpret_cast<float*>(p); p += kQ * 65 * 4;
  s.att = reinterpret_cast<__nv_bfloat16*>(p); p += kQ * 72 * 2;
  s.qhay = reinterpret_cast<int*>(p);
  return s;
}

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}
}  // namespace

// Gather slots [s_begin, s_end) of row r into the ring (features by plain and asynchronous copies, value rows by
// asynchronous copies with zero fill for rows no query uses).
__device__ __forceinline__ void tc_load_slots(const ScoreArgs& a, const TcSmem& S, int64_t r, int64_t b,
                                              int64_t s_begin, int64_t s_end, int dp0, int dpart, int Ppad,
                                              int Cpad) {
  const __nv_bfloat16* phi = reinterpret_cast<const __nv_bfloat16*>(a.phi);
  const __nv_bfloat16* Qc = reinterpret_cast<const __nv_bfloat16*>(a.Qc);
  const __nv_bfloat16* Kc = reinterpret_cast<const __nv_bfloat16*>(a.Kc);
  const __nv_bfloat16* Ea = reinterpret_cast<const __nv_bfloat16*>(a.Ea);
  const int n = (int)(s_end - s_begin);
  // scalars: one thread per slot
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t s = s_begin + i;
    const int ri = (int)(s & (kW - 1));
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? a.orden[r * a.L + s] : 0;
    const int id = real ? (int)a.ids_o[r * a.L + s] : -1;
    const bool used = real && s + 1 < a.L && (int)a.ids_o[r * a.L + s + 1] == id && pos + 1 < a.L;
    const int64_t g = b * a.L + pos;
    S.pos[ri] = pos;
    S.id[ri] = id;
    S.used[ri] = used ? 1 : 0;
    S.bt[ri] = real ? a.Bt[g] : 0.0;
    S.la[ri] = real ? a.log_alfa[g] : 0.f;
    for (int c = 0; c < a.K; ++c) {
      const int t = pos - 1 - c;
      S.pf[ri * a.K + c] = (real && t >= 0) ? a.sig[b * a.L + t] : __int_as_float(0x7fc00000);
    }
  }
  // vector rows: 16-byte chunks
  const int cph = Ppad / 8, cpc = Cpad / 8, cpv = dpart / 8;
  const int per_slot = cph + 2 * cpc + cpv;
  for (int e = threadIdx.x; e < n * per_slot; e += blockDim.x) {
    const int i = e / per_slot, c = e % per_slot;
    const int64_t s = s_begin + i;
    const int ri = (int)(s & (kW - 1));
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? a.orden[r * a.L + s] : 0;
    const int64_t g = b * a.L + pos;
    if (c < cph) {
      const int col = c * 8;
      const bool ok = real && col < a.P;
      cp_async16(S.phi + ri * S.Pp + col, phi + g * a.P + (ok ? col : 0), ok);
    } else if (c < cph + cpc) {
      const int col = (c - cph) * 8;
      const bool ok = real && col < a.cf;
      cp_async16(S.qc + ri * S.Cp + col, Qc + g * a.cf + (ok ? col : 0), ok);
    } else if (c < cph + 2 * cpc) {
      const int col = (c - cph - cpc) * 8;
      const bool ok = real && col < a.cf;
      cp_async16(S.kc + ri * S.Cp + col, Kc + g * a.cf + (ok ? col : 0), ok);
    } else {
      const int col = (c - cph - 2 * cpc) * 8;
      bool ok = real && s + 1 < a.L && pos + 1 < a.L;
      if (ok) ok = (int)a.ids_o[r * a.L + s + 1] == (int)a.ids_o[r * a.L + s];
      cp_async16(S.v + ri * S.Dp + col, Ea + (b * a.L + (ok ? pos + 1 : 0)) * (int64_t)a.d + dp0 + col, ok);
    }
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(kThreadsTc, 2) k_score_tc(ScoreArgs a, int nds, int dpart) {
  extern __shared__ __align__(16) char smem_raw[];
  const TcSmem S = carve_tc(smem_raw, a.P, a.cf, a.K, dpart);
  const int64_t r = blockIdx.y;
  const int64_t b = r / a.T;
  const int tau = (int)(r % a.T);
  const int part = blockIdx.x % nds;
  const int64_t S0 = (int64_t)(blockIdx.x / nds) * kSpanTc;
  const int64_t S1 = min(S0 + kSpanTc, a.L);
  const int dp0 = part * dpart;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const float tasa = a.tasa[tau];
  const int Ppad = pad16(a.P), Cpad = pad16(a.cf);
  const int C = a.C;
  const bool write_signals = part == 0;

  for (int64_t q0 = S0; q0 < S1; q0 += kQ) {
    tc_load_slots(a, S, r, b, q0 == S0 ? q0 - kQ : q0, q0 + kQ, dp0, dpart, Ppad, Cpad);
    cp_async_wait_all();
    __syncthreads();

    // ---- scores: warp w -> m-tile (w >> 2), n-tiles 2 (w & 3), 2 (w & 3) + 1 ------------------------------------
    {
      const int mt = wid >> 2;
      const int nt0 = (wid & 3) * 2;
      float cphi[2][4] = {}, cqk[2][4] = {};
      // A rows: queries mt*16 + (lane & 15), k offset (lane >> 4) * 8
      const int qa = mt * 16 + (lane & 15);
      const int ra = (int)((q0 + qa) & (kW - 1));
      const int ka = (lane >> 4) * 8;
      for (int k0 = 0; k0 < Ppad; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(su32(S.phi + ra * S.Pp + k0 + ka), a0, a1, a2, a3);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int key = (nt0 + j) * 8 + (lane & 7);
          const int rk = (int)((q0 - kQ + key) & (kW - 1));
          uint32_t b0, b1;
          ldsm_x2(su32(S.phi + rk * S.Pp + k0 + ((lane >> 3) & 1) * 8), b0, b1);
          mma16816(cphi[j], a0, a1, a2, a3, b0, b1);
        }
      }
      for (int k0 = 0; k0 < Cpad; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(su32(S.qc + ra * S.Cp + k0 + ka), a0, a1, a2, a3);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int key = (nt0 + j) * 8 + (lane & 7);
          const int rk = (int)((q0 - kQ + key) & (kW - 1));
          uint32_t b0, b1;
          ldsm_x2(su32(S.kc + rk * S.Cp + k0 + ((lane >> 3) & 1) * 8), b0, b1);
          mma16816(cqk[j], a0, a1, a2, a3, b0, b1);
        }
      }
      // finish each element: rounding chain, suffix, log_alfa_k, time; invalid -> -inf
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi = mt * 16 + (lane >> 2) + (e >> 1) * 8;
          const int kj = (nt0 + j) * 8 + (lane & 3) * 2 + (e & 1);
          const int64_t sq = q0 + qi, sk = q0 - kQ + kj;
          const int rq = (int)(sq & (kW - 1)), rk = (int)(sk & (kW - 1));
          float val = -INFINITY;
          const bool valid = sq < a.L && sk >= 0 && sk < sq && sk >= sq - C && S.id[rk] == S.id[rq];
          if (valid) {
            const float s1 = round_bf16(__fdiv_rn(round_bf16(cphi[j][e]), a.inv_temp_div));
            const float s2 = round_bf16(__fmul_rn(round_bf16(cqk[j][e]), a.esc_c));
            float t1 = round_bf16(__fadd_rn(s1, s2));
            int ln = 0;
            for (int c = 0; c < a.K; ++c) {
              if (S.pf[rq * a.K + c] == S.pf[rk * a.K + c]) ++ln; else break;
            }
            t1 = __fadd_rn(t1, a.w_suf[ln]);
            t1 = __fadd_rn(t1, S.la[rk]);
            const float dt = __double2float_rn(S.bt[rk] - S.bt[rq]);
            val = __fadd_rn(t1, __fmul_rn(dt, tasa));
          }
          S.sc[qi * 65 + kj] = val;
        }
    }
    __syncthreads();

    // ---- softmax per query (warp w: queries 4w .. 4w+3; lane -> keys lane, lane + 32) -------------------------------
    for (int qi = wid * 4; qi < wid * 4 + 4; ++qi) {
      const int64_t sq = q0 + qi;
      const float x0 = S.sc[qi * 65 + lane], x1 = S.sc[qi * 65 + lane + 32];
      const bool v0 = x0 != -INFINITY, v1 = x1 != -INFINITY;
      const int nv = __popc(__ballot_sync(0xffffffffu, v0)) + __popc(__ballot_sync(0xffffffffu, v1));
      float w0 = 0.f, w1 = 0.f;
      if (nv > 0) {
        const float mx = warp_max(fmaxf(x0, x1));
        const float e0 = v0 ? expf(__fsub_rn(x0, mx)) : 0.f;
        const float e1 = v1 ? expf(__fsub_rn(x1, mx)) : 0.f;
        const float sum = warp_sum(e0 + e1);
        w0 = __fdiv_rn(e0, sum);
        w1 = __fdiv_rn(e1, sum);
        const float peak = warp_max(fmaxf(w0, w1));
        if (lane == 0 && write_signals && sq < S1) {
          const int64_t gq = b * a.L + S.pos[(int)(sq & (kW - 1))];
          a.sen_hay[gq * a.T + tau] = 1;
          a.sen_mx[gq * a.T + tau] = mx;
          a.sen_pk[gq * a.T + tau] = peak;
        }
      } else if (lane == 0 && write_signals && sq < S1) {
        const int64_t gq = b * a.L + S.pos[(int)(sq & (kW - 1))];
        a.sen_hay[gq * a.T + tau] = 0;
        a.sen_mx[gq * a.T + tau] = kProhibido;
        a.sen_pk[gq * a.T + tau] = 0.f;
      }
      S.att[qi * 72 + lane] = __float2bfloat16_rn(w0);
      S.att[qi * 72 + lane + 32] = __float2bfloat16_rn(w1);
      if (lane == 0) S.qhay[qi] = (nv > 0 && sq < S1) ? 1 : 0;
    }
    __syncthreads();

    // ---- out = att . V on tensor cores; warp w owns columns [w * dpart / 8, (w + 1) * dpart / 8) -----------------
    {
      const int cols = dpart / 8;           // multiple of 8
      const int c0w = wid * cols;
      const int nn = cols / 8;              // n8 tiles of this warp (<= 6)
      for (int mt = 0; mt < 2; ++mt) {
        const int qbase = mt * 16;
        const bool any = S.qhay[qbase + (lane & 15)] != 0;
        if (!__any_sync(0xffffffffu, any)) continue;
        float acc[6][4];
#pragma unroll
        for (int j = 0; j < 6; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        // queries of m-tile mt use window keys [qbase, qbase + 47]
        for (int ks = mt; ks < mt + 3; ++ks) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(su32(S.att + (qbase + (lane & 15)) * 72 + ks * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
          const int key = ks * 16 + (lane & 15);
          const int rk = (int)((q0 - kQ + key) & (kW - 1));
#pragma unroll
          for (int j = 0; j < 6; ++j) {
            if (j < nn) {
              uint32_t b0, b1;
              ldsm_x2_t(su32(S.v + rk * S.Dp + c0w + j * 8), b0, b1);
              mma16816(acc[j], a0, a1, a2, a3, b0, b1);
            }
          }
        }
        // reductions into acc rows of the queries that have candidates
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
          const int qi = qbase + (lane >> 2) + hrow * 8;
          if (!S.qhay[qi]) continue;
          const int64_t gq = b * a.L + S.pos[(int)((q0 + qi) & (kW - 1))];
          float* dst = a.acc + gq * a.d + dp0 + c0w + (lane & 3) * 2;
#pragma unroll
          for (int j = 0; j < 6; ++j)
            if (j < nn) red_add_v2(dst + j * 8, acc[j][hrow * 2], acc[j][hrow * 2 + 1]);
        }
      }
    }
    __syncthreads();
  }
}

// cp.async moves 16-byte chunks: phi, Qc, Kc and Ea rows must be multiples of 8 bf16 (rows stay 16-byte aligned).
bool score_tc_supported(const ScoreArgs& a) {
  return a.d % 64 == 0 && a.d <= 1024 && a.C <= 32 && a.P <= kMaxPhi && a.P % 8 == 0 && a.cf <= kMaxConfirm &&
         a.cf % 8 == 0 && a.K <= kMaxSuffix;
}

int launch_score_tc(const ScoreArgs& a, cudaStream_t s) {
  int nds = (a.d + 383) / 384;
  while (a.d % (nds * 64) != 0) ++nds;
  const int dpart = a.d / nds;
  if (dpart / 8 / 8 > 6) return ASRN_ERR_UNSUPPORTED;
  const size_t smem = tc_smem_bytes(a.P, a.cf, a.K, dpart);
  cudaFuncSetAttribute(k_score_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)(((a.L + kSpanTc - 1) / kSpanTc) * nds), (unsigned)(a.B * a.T));
  k_score_tc<<<grid, kThreadsTc, smem, s>>>(a, nds, dpart);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
