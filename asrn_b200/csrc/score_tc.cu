// Candidate scoring on tensor cores (bf16 autocast mode). Same computation as k_score_simt (asrn/estable.py:204-300,
// asrn/nucleo.py:279-382), organised per block of 32 sorted query slots:
//   window = the 64 sorted slots [q0 - 32, q0 + 32) of the row (the previous block + the current block); features
//   (phi, Qc, Kc, clock, log_alfa, previous signatures) of each slot are gathered once into a 64-slot ring, and so
//   are the value rows Ea[pos + 1] of the slots some query can use (a slot is a candidate of somebody only if the
//   next sorted slot is in the same bucket; other rows are zero-filled without reading memory);
//   S = phi_q . phi_k and Qc . Kc (32 x 64 each) on mma.sync (fp32 accumulate), then the reference's rounding chain,
//   suffix weight, log_alfa_k and the fp64 time difference, the exact-mask softmax per query, and
//   out (32 x d_part) = att (32 x 64, bf16) . V (64 x d_part) on mma.sync, added into acc with vector reductions.
// One block of 16 warps per (row, span of 512 slots); the ring holds 96 slots so the next sub-tile's rows arrive by
// cp.async while the current one computes. d is split over two blocks only when d > 768.
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {
constexpr int kQ = 32;          // queries per sub-tile
constexpr int kW = 64;          // window slots [q0 - 32, q0 + 32)
constexpr int kR = 96;          // ring slots: the window plus the next sub-tile's 32 slots (prefetched)
constexpr int kSpanTc = 512;    // sorted slots per block
constexpr int kThreadsTc = 512; // 16 warps

constexpr int kStage = 3;        // staging buffers of sorted-row entries (sub-tiles j + 1, j + 2 and one being freed)
constexpr int kStageIds = 40;    // ids staged per sub-tile: its 32 slots and the next 8 (the `used` test reads s + 1)

struct TcSmem {
  int* st_pos;          // [kStage][kQ] orden entries of a staged sub-tile
  uint16_t* st_id;      // [kStage][kStageIds] ids_o entries
  int* pos;
  int* id;
  int* used;
  double* bt;
  float* la;
  float* pf;
  __nv_bfloat16* phi;   // [kR][Pp]
  __nv_bfloat16* qc;    // [kR][Cp]
  __nv_bfloat16* kc;    // [kR][Cp]
  __nv_bfloat16* v;     // [kR][Dp]
  float* sc;            // [32][65]
  __nv_bfloat16* att;   // [32][72]
  int* qhay;            // [32]
  int Pp, Cp, Dp, K;
};

__host__ __device__ inline int pad16(int x) { return (x + 15) / 16 * 16; }

__host__ __device__ inline size_t tc_smem_bytes(int P, int cf, int K, int dpart) {
  const int Pp = pad16(P) + 8, Cp = pad16(cf) + 8, Dp = dpart + 8;
  size_t b = 0;
  b += kStage * kQ * 4 + kStage * kStageIds * 2;   // staging
  b = (b + 15) / 16 * 16;
  b += kR * 8;                    // bt
  b += kR * 4 * 3;                // pos, id, used
  b += kR * 4;                    // la
  b = (b + 15) / 16 * 16;
  b += kR * 4 * (size_t)kMaxSuffix;   // pf (rows of 8, 16-byte aligned)
  b += (size_t)kR * Pp * 2 + 2 * (size_t)kR * Cp * 2 + (size_t)kR * Dp * 2;
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
  s.st_pos = reinterpret_cast<int*>(p); p += kStage * kQ * 4;
  s.st_id = reinterpret_cast<uint16_t*>(p); p += kStage * kStageIds * 2;
  p = base + ((p - base) + 15) / 16 * 16;
  s.bt = reinterpret_cast<double*>(p); p += kR * 8;
  s.pos = reinterpret_cast<int*>(p); p += kR * 4;
  s.id = reinterpret_cast<int*>(p); p += kR * 4;
  s.used = reinterpret_cast<int*>(p); p += kR * 4;
  s.la = reinterpret_cast<float*>(p); p += kR * 4;
  p = base + ((p - base) + 15) / 16 * 16;
  s.pf = reinterpret_cast<float*>(p); p += kR * 4 * kMaxSuffix;
  s.phi = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kR * s.Pp * 2;
  s.qc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kR * s.Cp * 2;
  s.kc = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kR * s.Cp * 2;
  s.v = reinterpret_cast<__nv_bfloat16*>(p); p += (size_t)kR * s.Dp * 2;
  s.sc = reinterpret_cast<float*>(p); p += kQ * 65 * 4;
  s.att = reinterpret_cast<__nv_bfloat16*>(p); p += kQ * 72 * 2;
  s.qhay = reinterpret_cast<int*>(p);
  return s;
}

__device__ __forceinline__ int ring(int64_t slot) { return (int)((slot + kR) % kR); }   // slot >= -kR

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(su32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(su32(dst)), "l"(src) : "memory");
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

// Stage 1 (two sub-tiles ahead): the sub-tile's 32 orden entries and 40 ids_o entries of row r, slots
// [s0, s0 + 32 / 40), into staging buffer `buf` by 16-byte cp.async (zero-filled outside [0, L); rows are 16-byte
// aligned: L % 8 == 0). Threads 0-7 copy orden, 8-12 ids.
__device__ __forceinline__ void tc_stage1(const ScoreArgs& a, const TcSmem& S, int64_t r, int64_t s0, int buf) {
  const int t = threadIdx.x;
  if (t < kQ / 4) {
    const int64_t s = s0 + 4 * t;
    const bool ok = s >= 0 && s < a.L;
    cp_async16(S.st_pos + buf * kQ + 4 * t, a.orden + r * a.L + (ok ? s : 0), ok);
  } else if (t < kQ / 4 + kStageIds / 8) {
    const int c = t - kQ / 4;
    const int64_t s = s0 + 8 * c;
    const bool ok = s >= 0 && s < a.L;
    cp_async16(S.st_id + buf * kStageIds + 8 * c, a.ids_o + r * a.L + (ok ? s : 0), ok);
  }
}

// Stage 2 (one sub-tile ahead): for the 32 slots [s0, s0 + 32) staged in `buf`, one warp per slot: lane 0 derives
// (position, id, used) from the staging buffer and writes them to the slot's ring row; the lanes gather by cp.async
// the clock (8 B), log_alfa and the K previous signatures (4 B each) of the position and its vector rows (phi, Qc,
// Kc and, when some query can use it, the value row Ea[pos + 1]; 16 B each, zero-filled otherwise).
__device__ __forceinline__ void tc_stage2(const ScoreArgs& a, const TcSmem& S, int64_t b, int64_t s0, int buf,
                                          int dp0, int dpart, int Ppad, int Cpad) {
  const __nv_bfloat16* phi = reinterpret_cast<const __nv_bfloat16*>(a.phi);
  const __nv_bfloat16* Qc = reinterpret_cast<const __nv_bfloat16*>(a.Qc);
  const __nv_bfloat16* Kc = reinterpret_cast<const __nv_bfloat16*>(a.Kc);
  const __nv_bfloat16* Ea = reinterpret_cast<const __nv_bfloat16*>(a.Ea);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int cph = Ppad / 8, cpc = Cpad / 8, cpv = dpart / 8;
  const int per_slot = cph + 2 * cpc + cpv;
  for (int i = wid; i < kQ; i += nw) {
    const int64_t s = s0 + i;
    const int ri = ring(s);
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? S.st_pos[buf * kQ + i] : 0;
    const int id = real ? (int)S.st_id[buf * kStageIds + i] : -1;
    const bool used = real && s + 1 < a.L && (int)S.st_id[buf * kStageIds + i + 1] == id && pos + 1 < a.Lf;
    const int64_t g = b * a.Lf + pos;
    if (lane == 0) {
      S.pos[ri] = pos;
      S.id[ri] = id;
      S.used[ri] = used ? 1 : 0;
      if (real) cp_async8(S.bt + ri, a.Bt + g);
      else S.bt[ri] = 0.0;
      if (real) cp_async4(S.la + ri, a.log_alfa + g);
      else S.la[ri] = 0.f;
    } else if (lane <= kMaxSuffix) {
      // previous signatures sig[pos - 1 - c]; NaN (never equal) before the text and past K
      const int c = lane - 1;
      const int64_t t = (int64_t)pos - 1 - c;
      if (real && c < a.K && t >= 0) cp_async4(S.pf + ri * kMaxSuffix + c, a.sig + b * a.Lf + t);
      else S.pf[ri * kMaxSuffix + c] = __int_as_float(0x7fc00000);
    }
    const __nv_bfloat16* vsrc = Ea + (b * a.Lf + (used ? pos + 1 : 0)) * (int64_t)a.d + dp0;
    for (int c = lane; c < per_slot; c += 32) {
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
        cp_async16(S.v + ri * S.Dp + col, vsrc + (used ? col : 0), used);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreadsTc, 1) k_score_tc(ScoreArgs a, int nds, int dpart) {
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

  // Pipeline over sub-tiles j = -1 (the window's first half, slots [S0 - 32, S0)), 0, 1, ...: staging buffer of
  // sub-tile j = (j + 1) % kStage; stage 1 of j + 2 and stage 2 of j + 1 are issued while sub-tile j computes.
  const int ntile = (int)((S1 - S0 + kQ - 1) / kQ);
  tc_stage1(a, S, r, S0 - kQ, 0);
  tc_stage1(a, S, r, S0, 1);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  tc_stage2(a, S, b, S0 - kQ, 0, dp0, dpart, Ppad, Cpad);
  tc_stage2(a, S, b, S0, 1, dp0, dpart, Ppad, Cpad);
  if (ntile > 1) tc_stage1(a, S, r, S0 + kQ, 2);
  cp_async_commit();

  for (int j = 0; j < ntile; ++j) {
    const int64_t q0 = S0 + (int64_t)j * kQ;
    // ring rows: window key k (slot q0 - 32 + k) -> wrow(k); query i (slot q0 + i) -> wrow(32 + i)
    const int rbase = ring(q0 - kQ);
    auto wrow = [rbase](int k) { const int x = rbase + k; return x >= kR ? x - kR : x; };
    cp_async_wait_all();
    __syncthreads();
    if (j + 1 < ntile) tc_stage2(a, S, b, q0 + kQ, (j + 2) % kStage, dp0, dpart, Ppad, Cpad);
    if (j + 2 < ntile) tc_stage1(a, S, r, q0 + 2 * kQ, (j + 3) % kStage);
    cp_async_commit();

    // ---- scores: warp w -> m-tile (w >> 3), n-tile (w & 7) --------------------------------------------------------
    {
      const int mt = wid >> 3;
      const int nt = wid & 7;
      float cphi[4] = {0.f, 0.f, 0.f, 0.f}, cqk[4] = {0.f, 0.f, 0.f, 0.f};
      // band: this tile's keys [8 nt, 8 nt + 8) meet queries [16 mt, 16 mt + 16) only if some key is within C before
      const int key_lo = nt * 8, q_lo = mt * 16;
      const bool band = key_lo + 7 >= q_lo + 32 - C && key_lo < q_lo + 16 + 32;
      if (band) {
        const int qa = mt * 16 + (lane & 15);
        const int ra = wrow(kQ + qa);
        const int ka = (lane >> 4) * 8;
        const int key = nt * 8 + (lane & 7);
        const int rk = wrow(key);
        const int kb = ((lane >> 3) & 1) * 8;
        const uint32_t phi_a = su32(S.phi) + 2u * (uint32_t)(ra * S.Pp + ka);
        const uint32_t phi_b = su32(S.phi) + 2u * (uint32_t)(rk * S.Pp + kb);
        const uint32_t qc_a = su32(S.qc) + 2u * (uint32_t)(ra * S.Cp + ka);
        const uint32_t kc_b = su32(S.kc) + 2u * (uint32_t)(rk * S.Cp + kb);
        for (int k0 = 0; k0 < Ppad; k0 += 16) {
          uint32_t a0, a1, a2, a3, b0, b1;
          ldsm_x4(phi_a + 2 * k0, a0, a1, a2, a3);
          ldsm_x2(phi_b + 2 * k0, b0, b1);
          mma16816(cphi, a0, a1, a2, a3, b0, b1);
        }
        for (int k0 = 0; k0 < Cpad; k0 += 16) {
          uint32_t a0, a1, a2, a3, b0, b1;
          ldsm_x4(qc_a + 2 * k0, a0, a1, a2, a3);
          ldsm_x2(kc_b + 2 * k0, b0, b1);
          mma16816(cqk, a0, a1, a2, a3, b0, b1);
        }
      }
      // this lane's two query rows (qi0, qi0 + 8) and two key columns (kj0, kj0 + 1): their ring-row scalars are
      // read once, the suffix length is the count of leading equal previous signatures (compare mask, no branches)
      const int qi0 = mt * 16 + (lane >> 2), kj0 = nt * 8 + (lane & 3) * 2;
      int q_id[2], k_id[2];
      float4 q_pf[2][2], k_pf[2][2];
      double q_bt[2], k_bt[2];
      float k_la[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int rq = wrow(kQ + qi0 + 8 * u), rk = wrow(kj0 + u);
        q_id[u] = S.id[rq];
        k_id[u] = S.id[rk];
        q_pf[u][0] = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix);
        q_pf[u][1] = *reinterpret_cast<const float4*>(S.pf + rq * kMaxSuffix + 4);
        k_pf[u][0] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix);
        k_pf[u][1] = *reinterpret_cast<const float4*>(S.pf + rk * kMaxSuffix + 4);
        q_bt[u] = S.bt[rq];
        k_bt[u] = S.bt[rk];
        k_la[u] = S.la[rk];
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int uq = e >> 1, uk = e & 1;
        const int qi = qi0 + 8 * uq;
        const int kj = kj0 + uk;
        const int64_t sq = q0 + qi, sk = q0 - kQ + kj;
        float val = -INFINITY;
        if (band && kj < qi + 32 && kj >= qi + 32 - C && sq < a.L && sk >= 0 && k_id[uk] == q_id[uq]) {
          const float s1 = round_bf16(__fdiv_rn(round_bf16(cphi[e]), a.inv_temp_div));
          const float s2 = round_bf16(__fmul_rn(round_bf16(cqk[e]), a.esc_c));
          float t1 = round_bf16(__fadd_rn(s1, s2));
          const float4 qa = q_pf[uq][0], qb = q_pf[uq][1], ka = k_pf[uk][0], kb = k_pf[uk][1];
          const uint32_t eq = (qa.x == ka.x ? 1u : 0u) | (qa.y == ka.y ? 2u : 0u) | (qa.z == ka.z ? 4u : 0u) |
                              (qa.w == ka.w ? 8u : 0u) | (qb.x == kb.x ? 16u : 0u) | (qb.y == kb.y ? 32u : 0u) |
                              (qb.z == kb.z ? 64u : 0u) | (qb.w == kb.w ? 128u : 0u);
          const int ln = __ffs(~eq) - 1;          // leading equal entries (entries past K are NaN: never equal)
          t1 = __fadd_rn(t1, a.w_suf[ln]);
          t1 = __fadd_rn(t1, k_la[uk]);
          const float dt = __double2float_rn(k_bt[uk] - q_bt[uq]);
          val = __fadd_rn(t1, __fmul_rn(dt, tasa));
        }
        S.sc[qi * 65 + kj] = val;
      }
    }
    __syncthreads();

    // ---- softmax per query (warp w: queries 2w, 2w + 1 together; lane -> keys lane, lane + 32) ----------------------
    {
      const int qa = wid * 2;
      float x[2][2];
      bool vv[2][2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        x[u][0] = S.sc[(qa + u) * 65 + lane];
        x[u][1] = S.sc[(qa + u) * 65 + lane + 32];
        vv[u][0] = x[u][0] != -INFINITY;
        vv[u][1] = x[u][1] != -INFINITY;
      }
      const unsigned bal0 = __ballot_sync(0xffffffffu, vv[0][0] || vv[0][1]);
      const unsigned bal1 = __ballot_sync(0xffffffffu, vv[1][0] || vv[1][1]);
      float m0 = fmaxf(x[0][0], x[0][1]), m1 = fmaxf(x[1][0], x[1][1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
      }
      const float mxs[2] = {m0, m1};
      float e[2][2], sum[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        e[u][0] = vv[u][0] ? expf(__fsub_rn(x[u][0], mxs[u])) : 0.f;
        e[u][1] = vv[u][1] ? expf(__fsub_rn(x[u][1], mxs[u])) : 0.f;
        sum[u] = e[u][0] + e[u][1];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sum[0] += __shfl_xor_sync(0xffffffffu, sum[0], o);
        sum[1] += __shfl_xor_sync(0xffffffffu, sum[1], o);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int qi = qa + u;
        const int64_t sq = q0 + qi;
        const bool anyv = (u == 0 ? bal0 : bal1) != 0;
        const int posq = S.pos[wrow(kQ + qi)];
        const bool mine = sq < S1 && posq >= a.q_lo && posq < a.q_hi;   // else a key only (another shard's position)
        const int64_t gq = b * (a.q_hi - a.q_lo) + (posq - a.q_lo);
        float w0 = 0.f, w1 = 0.f;
        if (anyv) {
          w0 = __fdiv_rn(e[u][0], sum[u]);
          w1 = __fdiv_rn(e[u][1], sum[u]);
          // the largest weight is the maximum's: exp(0) / sum
          if (lane == 0 && write_signals && mine) {
            a.sen_hay[gq * a.T + tau] = 1;
            a.sen_mx[gq * a.T + tau] = mxs[u];
            a.sen_pk[gq * a.T + tau] = __fdiv_rn(1.f, sum[u]);
          }
        } else if (lane == 0 && write_signals && mine) {
          a.sen_hay[gq * a.T + tau] = 0;
          a.sen_mx[gq * a.T + tau] = kProhibido;
          a.sen_pk[gq * a.T + tau] = 0.f;
        }
        S.att[qi * 72 + lane] = __float2bfloat16_rn(w0);
        S.att[qi * 72 + lane + 32] = __float2bfloat16_rn(w1);
        if (lane == 0) S.qhay[qi] = (anyv && mine) ? 1 : 0;
      }
    }
    __syncthreads();

    // ---- out = att . V on tensor cores; warp w owns n8 tiles w, w + 16, ... of the d_part columns -----------------
    {
      const int ntiles = dpart / 8;
      for (int mt = 0; mt < 2; ++mt) {
        const int qbase = mt * 16;
        const bool any = S.qhay[qbase + (lane & 15)] != 0;
        if (!__any_sync(0xffffffffu, any)) continue;
        if (wid >= ntiles) continue;
        float acc[6][4];
#pragma unroll
        for (int j = 0; j < 6; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        // queries of m-tile mt use window keys [qbase, qbase + 47]
        const uint32_t att_a = su32(S.att) + 2u * (uint32_t)((qbase + (lane & 15)) * 72 + (lane >> 4) * 8);
        for (int ks = mt; ks < mt + 3; ++ks) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(att_a + 2u * (uint32_t)(ks * 16), a0, a1, a2, a3);
          const int rk = wrow(ks * 16 + (lane & 15));
          const uint32_t v_row = su32(S.v) + 2u * (uint32_t)(rk * S.Dp);
#pragma unroll
          for (int j = 0; j < 6; ++j) {
            const int tile = wid + 16 * j;
            if (tile < ntiles) {
              uint32_t b0, b1;
              ldsm_x2_t(v_row + 2u * (uint32_t)(tile * 8), b0, b1);
              mma16816(acc[j], a0, a1, a2, a3, b0, b1);
            }
          }
        }
        // one 16-byte reduction per lane and tile: lanes q and q ^ 1 of a quad swap halves so that the even lane
        // holds columns 4 (q >> 1) .. + 3 of row r and the odd lane the same columns of row r + 8
        const int qd = lane & 3;
        const int rowq = qbase + (lane >> 2) + ((qd & 1) ? 8 : 0);
        const bool hasq = S.qhay[rowq] != 0;
        const int64_t gq = b * (a.q_hi - a.q_lo) + (S.pos[wrow(kQ + rowq)] - a.q_lo);
        float* dst = a.acc + gq * a.d + dp0 + (qd >> 1) * 4;
#pragma unroll
        for (int j = 0; j < 6; ++j) {
          const int tile = wid + 16 * j;
          if (tile < ntiles) {
            const bool odd = qd & 1;
            const float s0 = odd ? acc[j][0] : acc[j][2], s1 = odd ? acc[j][1] : acc[j][3];
            const float r0 = __shfl_xor_sync(0xffffffffu, s0, 1), r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
            const float v0 = odd ? r0 : acc[j][0], v1 = odd ? r1 : acc[j][1];
            const float v2 = odd ? acc[j][2] : r0, v3 = odd ? acc[j][3] : r1;
            if (hasq) red_add_v4(dst + tile * 8, v0, v1, v2, v3);
          }
        }
      }
    }
  }
  cp_async_wait_all();
}

bool score_tc_supported(const ScoreArgs& a) {
  return a.d % 64 == 0 && a.d <= 1024 && a.C <= 32 && a.P <= kMaxPhi && a.P % 8 == 0 && a.cf <= kMaxConfirm &&
         a.cf % 8 == 0 && a.K <= kMaxSuffix && a.K <= 31 && a.L % 8 == 0;
}

int launch_score_tc(const ScoreArgs& a, cudaStream_t s) {
  // the whole width in one block when its 96-row value ring fits next to the features (d <= 768), else halves
  int nds = (a.d + 767) / 768;
  while (a.d % (nds * 64) != 0) ++nds;
  const int dpart = a.d / nds;
  if (dpart / 8 > 16 * 6) return ASRN_ERR_UNSUPPORTED;
  const size_t smem = tc_smem_bytes(a.P, a.cf, a.K, dpart);
  cudaFuncSetAttribute(k_score_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)(((a.L + kSpanTc - 1) / kSpanTc) * nds), (unsigned)(a.B * a.T));
  k_score_tc<<<grid, kThreadsTc, smem, s>>>(a, nds, dpart);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
