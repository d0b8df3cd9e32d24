// Training kernels: the bucket attention forward and backward over the bucket-sorted rows, and the linear-recurrence
// scan forward and backward (asrn/nucleo.py:279-451, 461-537 -- the kernels asrn/estable.py:282-291 calls in its
// exact-mask, 64-bit-clock mode; the same arithmetic as the CPU path asrn/estable.py:204-263).
//
// Bucket attention. Row r = b T + table holds the L positions of sequence b sorted by (bucket, position); block j of
// the row is its sorted slots [j C, j C + C): C queries, each against the 2C keys of blocks j - 1 and j, of which the
// valid ones are those in the query's bucket among its C predecessors in sorted order. One CTA per (row, block)
// recomputes the scores
//   sc = phi_q . phi_k * scale_phi + Qc_q . Kc_k * scale_c + w_suf[suffix length] + log_alfa_k + tasa (B_k - B_q)
// (tasa = gamma[table] / C; the clock difference from a 64-bit clock passed as fp32 high and low parts) and the
// exact-mask softmax (max over the valid keys, invalid keys weigh exactly 0). Forward: out = att . V per table row
// and the signals (any valid key, max valid score, max weight). Backward (nothing stored by the forward, scores
// recomputed): dV = att^T dO, dP = dO V^T, dS = att (dP - rowsum(att dP)), and from dS the gradients of phi, Qc, Kc,
// the clock and log_alfa. No atomics: every query slot is written once per table (its block), every key slot twice
// -- as a current-block key (place 1) and as a previous-block key of the next block (place 0; the last block writes
// zeros there) -- and the gamma / w_suf sums go to one row of partials per CTA; the caller adds them up in a fixed
// order. Scores and sums in fp32; under bf16 the operands are bf16 and rounded where the reference's kernel rounds
// (att and dS to the operand type before their products), and every product runs on mma.sync tiles from bf16
// shared-memory tiles with fp32 accumulation: the scores [phi | Qc] . [phi | Kc]^T, the value-width products (att . V
// forward; dO . V^T and att^T . dO backward, in 64-column chunks of the values) and the feature gradients dS . [phi_k
// | Kc] and dS^T . [phi_q | Qc]. In fp32 every product stays on CUDA cores (exact fp32 sums).
//
// Scan. S_i = a_i S_{i-1} + b_i along each row (S_{-1} = 0); its backward is the same recurrence right to left:
// l_i = g_i + a_{i+1} l_{i+1}, dL/db_i = l_i, dL/da_i = l_i S_{i-1}. One CTA per row: each thread composes the affine
// maps of a contiguous chunk, a block-wide scan of the chunk maps gives each chunk its incoming value, then each
// thread replays its chunk.
#include "common.cuh"
#include "layout.h"

namespace asrn {

namespace {

constexpr int kBaThreads = 256;
constexpr int kBaMaxC = 32;
constexpr int kBaBd = 64;             // value columns per staged chunk
constexpr int kBaLdb = 72;            // bf16 row stride of the tensor-core tiles (64 + 8: ldmatrix rows on distinct banks)

template <bool Half>
struct BaT {
  using T = float;
};
template <>
struct BaT<true> {
  using T = __nv_bfloat16;
};

template <bool Half>
__device__ __forceinline__ float ba_ld(const typename BaT<Half>::T* p, int64_t i) {
  if constexpr (Half) return __bfloat162float(p[i]);
  else return p[i];
}
template <bool Half>
__device__ __forceinline__ void ba_st(typename BaT<Half>::T* p, int64_t i, float v) {
  if constexpr (Half) p[i] = __float2bfloat16_rn(v);
  else p[i] = v;
}
template <bool Half>
__device__ __forceinline__ float ba_round(float v) {
  return Half ? round_bf16(v) : v;
}

__device__ __forceinline__ void ba_ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ba_ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ba_mma(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct BaArgs {
  int64_t B, L;
  int T, C, P, CF, K, D, NB;
  const void* phi;                    // (B, L, P)
  const void* qc;                     // (B, L, CF)
  const void* kc;                     // (B, L, CF)
  const void* v;                      // (B, L, D)
  const float* pf;                    // (B, L, K) previous signatures (NaN before the start)
  const float* bt_hi;                 // (B, L)
  const float* bt_lo;                 // (B, L)
  const float* la;                    // (B, L)
  const int32_t* orden;               // (B T, L)
  const int32_t* ids_o;               // (B T, L)
  const float* w_suf;                 // (K + 1)
  const float* gamma;                 // (T)
  float scale_phi, scale_c;
  // forward
  void* out;                          // (B T, L, D)
  float* sen;                         // (B T, L, 3)
  // backward
  const void* dout;                   // (B, L, D)
  void* g_phi_q;                      // (B T, L, P)
  void* g_qc;                         // (B T, L, CF)
  float* g_b_q;                       // (B T, L)
  void* g_phi_k;                      // (2, B T, L, P)
  void* g_kc;                         // (2, B T, L, CF)
  void* g_v;                          // (2, B T, L, D)
  float* g_la;                        // (2, B T, L)
  float* g_b_k;                       // (2, B T, L)
  float* partes;                      // (B T, NB, K + 2)
};

// Shared-memory layout of one (row, block) CTA.
struct BaSmem {
  int64_t* filq;   // C: row of each query in (B L, .)
  int64_t* filk;   // 2C
  int* qpos;       // C: text position
  int* kpos;       // 2C
  int* qid;        // C
  int* kid;        // 2C
  float* phq;      // C x (P + 1)
  float* phk;      // 2C x (P + 1)
  float* qcs;      // C x (CF + 1)
  float* kcs;      // 2C x (CF + 1)
  float* pfq;      // C x K
  float* pfk;      // 2C x K
  float* bq;       // C x 2 (high, low)
  float* bk;       // 2C x 2
  float* lak;      // 2C
  float* att;      // C x (2C + 1): scores, then weights
  float* ds;       // C x (2C + 1): dP, then dS
  unsigned char* largo;   // C x 2C
  float* vs;       // 2C x (kBaBd + 1)
  float* os;       // C x (kBaBd + 1)
  float* red;      // 32
  // bf16 tiles of the tensor-core products (bf16 operands), padded to 32 queries x 64 keys
  __nv_bfloat16* attb;   // 32 x kBaLdb: att rounded to bf16 (zero outside C x 2C)
  __nv_bfloat16* vb;     // 64 x kBaLdb: value rows of the chunk
  __nv_bfloat16* ob;     // 32 x kBaLdb: output-gradient rows of the chunk
  __nv_bfloat16* fq;     // 32 x (Fp + 8): the queries' [phi | Qc] rows, each part zero-padded to a multiple of 16
  __nv_bfloat16* fk;     // 64 x (Fp + 8): the keys' [phi | Kc] rows
};

__host__ __device__ inline int ba_pad16(int x) { return (x + 15) / 16 * 16; }
__host__ __device__ inline int ba_fp(int P, int CF) { return ba_pad16(P) + ba_pad16(CF); }

// half: the bf16 path, which reads its features and values from the bf16 tiles only (the fp32 copies get no space)
__host__ __device__ inline size_t ba_smem_bytes(int C, int P, int CF, int K, bool half) {
  const size_t C2 = 2 * (size_t)C, f32 = half ? 0 : 1;
  size_t n = 0;
  n += (C + C2) * 8;                                       // filq, filk
  n += (C + C2) * 4 * 2;                                   // qpos, kpos, qid, kid
  n += f32 * ((C + C2) * (P + 1) * 4 + (C + C2) * (CF + 1) * 4);
  n += (C + C2) * (K > 0 ? K : 1) * 4;
  n += (C + C2) * 2 * 4 + C2 * 4;
  n += 2 * (size_t)C * (C2 + 1) * 4;
  n += (size_t)C * C2;
  n = (n + 15) / 16 * 16;
  n += f32 * (C2 + C) * (kBaBd + 1) * 4;
  n += 32 * 4;
  n += 16 + (size_t)(32 + 64 + 32) * kBaLdb * 2;
  n += 16 + (size_t)(32 + 64) * (ba_fp(P, CF) + 8) * 2;
  return n + 64;
}

__device__ inline BaSmem ba_carve(unsigned char* base, int C, int P, int CF, int K, bool half) {
  BaSmem s;
  const int C2 = 2 * C;
  const size_t f32 = half ? 0 : 1;
  unsigned char* p = base;
  auto take = [&](size_t bytes) {
    unsigned char* q = p;
    p += bytes;
    return q;
  };
  s.filq = reinterpret_cast<int64_t*>(take((size_t)C * 8));
  s.filk = reinterpret_cast<int64_t*>(take((size_t)C2 * 8));
  s.qpos = reinterpret_cast<int*>(take((size_t)C * 4));
  s.kpos = reinterpret_cast<int*>(take((size_t)C2 * 4));
  s.qid = reinterpret_cast<int*>(take((size_t)C * 4));
  s.kid = reinterpret_cast<int*>(take((size_t)C2 * 4));
  s.phq = reinterpret_cast<float*>(take(f32 * C * (P + 1) * 4));
  s.phk = reinterpret_cast<float*>(take(f32 * C2 * (P + 1) * 4));
  s.qcs = reinterpret_cast<float*>(take(f32 * C * (CF + 1) * 4));
  s.kcs = reinterpret_cast<float*>(take(f32 * C2 * (CF + 1) * 4));
  s.pfq = reinterpret_cast<float*>(take((size_t)C * (K > 0 ? K : 1) * 4));
  s.pfk = reinterpret_cast<float*>(take((size_t)C2 * (K > 0 ? K : 1) * 4));
  s.bq = reinterpret_cast<float*>(take((size_t)C * 2 * 4));
  s.bk = reinterpret_cast<float*>(take((size_t)C2 * 2 * 4));
  s.lak = reinterpret_cast<float*>(take((size_t)C2 * 4));
  s.att = reinterpret_cast<float*>(take((size_t)C * (C2 + 1) * 4));
  s.ds = reinterpret_cast<float*>(take((size_t)C * (C2 + 1) * 4));
  s.largo = take((size_t)C * C2);
  p = base + ((p - base + 15) / 16 * 16);
  s.vs = reinterpret_cast<float*>(take(f32 * C2 * (kBaBd + 1) * 4));
  s.os = reinterpret_cast<float*>(take(f32 * C * (kBaBd + 1) * 4));
  s.red = reinterpret_cast<float*>(take(32 * 4));
  p = base + ((p - base + 15) / 16 * 16);
  s.attb = reinterpret_cast<__nv_bfloat16*>(take((size_t)32 * kBaLdb * 2));
  s.vb = reinterpret_cast<__nv_bfloat16*>(take((size_t)64 * kBaLdb * 2));
  s.ob = reinterpret_cast<__nv_bfloat16*>(take((size_t)32 * kBaLdb * 2));
  p = base + ((p - base + 15) / 16 * 16);
  s.fq = reinterpret_cast<__nv_bfloat16*>(take((size_t)32 * (ba_fp(P, CF) + 8) * 2));
  s.fk = reinterpret_cast<__nv_bfloat16*>(take((size_t)64 * (ba_fp(P, CF) + 8) * 2));
  return s;
}

// Loads the block's slots and features and computes the scores and the exact-mask softmax into s.att; the signals of
// the queries go to sen when it is not null. Returns nothing; every thread takes part.
template <bool Half>
__device__ void ba_scores(const BaArgs& a, const BaSmem& s, int64_t r, int j, float* sen) {
  using T = typename BaT<Half>::T;
  const int C = a.C, C2 = 2 * C, P = a.P, CF = a.CF, K = a.K;
  const int64_t L = a.L, b = r / a.T;
  const int tid = threadIdx.x;
  for (int i = tid; i < C + C2; i += kBaThreads) {
    const bool is_q = i < C;
    const int64_t slot = is_q ? (int64_t)j * C + i : (int64_t)j * C - C + (i - C);
    const bool ok = slot >= 0 && slot < L;
    const int pos = ok ? a.orden[r * L + slot] : 0;
    const int id = ok ? a.ids_o[r * L + slot] : (is_q ? -1 : -2);
    if (is_q) {
      s.qpos[i] = ok ? pos : -1;
      s.qid[i] = id;
      s.filq[i] = b * L + pos;
    } else {
      s.kpos[i - C] = ok ? pos : -1;
      s.kid[i - C] = id;
      s.filk[i - C] = b * L + pos;
    }
  }
  __syncthreads();
  const T* phi = reinterpret_cast<const T*>(a.phi);
  const T* qc = reinterpret_cast<const T*>(a.qc);
  const T* kc = reinterpret_cast<const T*>(a.kc);
  if constexpr (Half) {
    // [phi | Qc] of the queries and [phi | Kc] of the keys as bf16 tiles (zero rows / columns outside)
    const int Pp = ba_pad16(P), Fp = ba_fp(P, CF), ldf = Fp + 8;
    if (P % 8 == 0 && CF % 8 == 0) {               // 16-byte pieces (8 features) when rows allow them
      const int nc8 = Fp / 8;
      for (int e = tid; e < 96 * nc8; e += kBaThreads) {
        const int i = e / nc8, c = (e % nc8) * 8;
        const bool is_q = i < 32;
        const int row = is_q ? i : i - 32;
        const bool ok = is_q ? (row < C && s.qpos[row] >= 0) : (row < C2 && s.kpos[row] >= 0);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (ok) {
          const int64_t fil = is_q ? s.filq[row] : s.filk[row];
          if (c < P) v = *reinterpret_cast<const uint4*>(phi + fil * P + c);
          else if (c >= Pp && c - Pp < CF) v = *reinterpret_cast<const uint4*>((is_q ? qc : kc) + fil * CF + (c - Pp));
        }
        *reinterpret_cast<uint4*>((is_q ? s.fq : s.fk) + row * ldf + c) = v;
      }
    } else
    for (int e = tid; e < 96 * Fp; e += kBaThreads) {
      const int i = e / Fp, c = e % Fp;
      const bool is_q = i < 32;
      const int row = is_q ? i : i - 32;
      const bool ok = is_q ? (row < C && s.qpos[row] >= 0) : (row < C2 && s.kpos[row] >= 0);
      __nv_bfloat16 v = __float2bfloat16_rn(0.f);
      if (ok) {
        const int64_t fil = is_q ? s.filq[row] : s.filk[row];
        if (c < P) v = phi[fil * P + c];
        else if (c >= Pp && c - Pp < CF) v = (is_q ? qc : kc)[fil * CF + (c - Pp)];
      }
      (is_q ? s.fq : s.fk)[row * ldf + c] = v;
    }
  } else {
  for (int e = tid; e < C * P; e += kBaThreads) {
    const int i = e / P, c = e % P;
    s.phq[i * (P + 1) + c] = s.qpos[i] >= 0 ? ba_ld<Half>(phi, s.filq[i] * P + c) : 0.f;
  }
  for (int e = tid; e < C2 * P; e += kBaThreads) {
    const int i = e / P, c = e % P;
    s.phk[i * (P + 1) + c] = s.kpos[i] >= 0 ? ba_ld<Half>(phi, s.filk[i] * P + c) : 0.f;
  }
  for (int e = tid; e < C * CF; e += kBaThreads) {
    const int i = e / CF, c = e % CF;
    s.qcs[i * (CF + 1) + c] = s.qpos[i] >= 0 ? ba_ld<Half>(qc, s.filq[i] * CF + c) : 0.f;
  }
  for (int e = tid; e < C2 * CF; e += kBaThreads) {
    const int i = e / CF, c = e % CF;
    s.kcs[i * (CF + 1) + c] = s.kpos[i] >= 0 ? ba_ld<Half>(kc, s.filk[i] * CF + c) : 0.f;
  }
  }
  for (int e = tid; e < C * K; e += kBaThreads) {
    const int i = e / K, c = e % K;
    s.pfq[e] = s.qpos[i] >= 0 ? a.pf[s.filq[i] * K + c] : 0.f;
  }
  for (int e = tid; e < C2 * K; e += kBaThreads) {
    const int i = e / K, c = e % K;
    s.pfk[e] = s.kpos[i] >= 0 ? a.pf[s.filk[i] * K + c] : 0.f;
  }
  for (int i = tid; i < C; i += kBaThreads) {
    const bool ok = s.qpos[i] >= 0;
    s.bq[2 * i] = ok ? a.bt_hi[s.filq[i]] : 0.f;
    s.bq[2 * i + 1] = ok ? a.bt_lo[s.filq[i]] : 0.f;
  }
  for (int i = tid; i < C2; i += kBaThreads) {
    const bool ok = s.kpos[i] >= 0;
    s.bk[2 * i] = ok ? a.bt_hi[s.filk[i]] : 0.f;
    s.bk[2 * i + 1] = ok ? a.bt_lo[s.filk[i]] : 0.f;
    s.lak[i] = ok ? a.la[s.filk[i]] : 0.f;
  }
  __syncthreads();
  if constexpr (Half) {
    // phi_q . phi_k and Qc . Kc (32 x 64 each) on mma.sync; the scaled sum goes to s.ds as scratch
    const int lane = tid & 31, wid = tid >> 5, i4 = lane >> 3, g = lane >> 2, t4 = lane & 3;
    const int mt = wid & 1, nt = wid >> 1, Pp = ba_pad16(P), Fp = ba_fp(P, CF), ldf = Fp + 8;
    float a1[2][4] = {}, a2[2][4] = {};
    auto tile_product = [&](float(&acc)[2][4], int k0, int k1) {
      for (int kk = k0; kk < k1; kk += 16) {
        uint32_t x0, x1, x2, x3, y0, y1, y2, y3;
        ba_ldsm_x4(s.fq + (16 * mt + (lane & 15)) * ldf + kk + (lane >> 4) * 8, x0, x1, x2, x3);
        ba_ldsm_x4(s.fk + (16 * nt + (i4 >> 1) * 8 + (lane & 7)) * ldf + kk + (i4 & 1) * 8, y0, y1, y2, y3);
        ba_mma(acc[0], x0, x1, x2, x3, y0, y1);
        ba_mma(acc[1], x0, x1, x2, x3, y2, y3);
      }
    };
    tile_product(a1, 0, Pp);
    tile_product(a2, Pp, Fp);
#pragma unroll
    for (int jn = 0; jn < 2; ++jn)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = 16 * mt + g + 8 * (e >> 1), k = 16 * nt + 8 * jn + 2 * t4 + (e & 1);
        if (q < C && k < C2)
          s.ds[q * (C2 + 1) + k] = __fadd_rn(__fmul_rn(a1[jn][e], a.scale_phi), __fmul_rn(a2[jn][e], a.scale_c));
      }
    __syncthreads();
  }
  const float tasa = a.gamma[r % a.T] / (float)C;
  // thread -> query tid / 8, keys tid % 8 + 8 u
  const int iq = tid >> 3;
  if (iq < C) {
    for (int ik = tid & 7; ik < C2; ik += 8) {
      const bool qm = s.qpos[iq] >= 0, km = s.kpos[ik] >= 0;
      float s1 = 0.f, s2 = 0.f;
      if constexpr (!Half) {
        for (int c = 0; c < P; ++c) s1 = fmaf(s.phq[iq * (P + 1) + c], s.phk[ik * (P + 1) + c], s1);
        for (int c = 0; c < CF; ++c) s2 = fmaf(s.qcs[iq * (CF + 1) + c], s.kcs[ik * (CF + 1) + c], s2);
      }
      bool sigue = qm && km;
      int largo = 0;
      for (int c = 0; c < K; ++c) {
        sigue = sigue && (s.pfq[iq * K + c] == s.pfk[ik * K + c]);
        largo += sigue ? 1 : 0;
      }
      const float dt = __fadd_rn(__fsub_rn(s.bk[2 * ik], s.bq[2 * iq]), __fsub_rn(s.bk[2 * ik + 1], s.bq[2 * iq + 1]));
      float sc = Half ? s.ds[iq * (C2 + 1) + ik] : __fadd_rn(__fmul_rn(s1, a.scale_phi), __fmul_rn(s2, a.scale_c));
      sc = __fadd_rn(__fadd_rn(__fadd_rn(sc, a.w_suf[largo]), s.lak[ik]), __fmul_rn(tasa, dt));
      const bool valido = ik >= iq && ik < C + iq && s.qid[iq] == s.kid[ik] && km && qm;
      s.att[iq * (C2 + 1) + ik] = valido ? sc : -INFINITY;       // -inf marks an invalid key (weight exactly 0)
      s.largo[iq * C2 + ik] = (unsigned char)largo;
    }
  }
  __syncthreads();
  // exact-mask softmax, one warp per query row
  const int lane = tid & 31, wid = tid >> 5;
  for (int q = wid; q < C; q += kBaThreads / 32) {
    float* row = s.att + q * (C2 + 1);
    float m = -INFINITY;
    for (int k = lane; k < C2; k += 32) m = fmaxf(m, row[k]);
    m = warp_max(m);
    const bool hay = m != -INFINITY;
    const float ref = hay ? m : 0.f;
    float sum = 0.f;
    for (int k = lane; k < C2; k += 32) {
      const float e = row[k] == -INFINITY ? 0.f : expf(row[k] - ref);
      row[k] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv_den = hay ? sum : 1.f;
    float pk = 0.f;
    for (int k = lane; k < C2; k += 32) {
      row[k] = row[k] / inv_den;
      pk = fmaxf(pk, row[k]);
    }
    pk = warp_max(pk);
    if (sen && lane == 0 && s.qpos[q] >= 0) {
      float* o = sen + (r * L + s.qpos[q]) * 3;
      o[0] = hay ? 1.f : 0.f;
      o[1] = ref;
      o[2] = pk;
    }
  }
  __syncthreads();
}

// att (C x 2C fp32) -> attb (32 x 64 bf16, zero outside C x 2C)
__device__ __forceinline__ void ba_fill_attb(const BaSmem& s, int C) {
  const int C2 = 2 * C;
  for (int e = threadIdx.x; e < 32 * 64; e += kBaThreads) {
    const int q = e >> 6, k = e & 63;
    s.attb[q * kBaLdb + k] = __float2bfloat16_rn(q < C && k < C2 ? s.att[q * (C2 + 1) + k] : 0.f);
  }
}

// Rows of a bf16 (., D) tensor into a 64-column bf16 tile: tile[i][c] = src[row(i) * D + d0 + c] for c < bd and a
// valid row, else 0; n rows.
__device__ __forceinline__ void ba_fill_tile(__nv_bfloat16* tile, const __nv_bfloat16* src, const int64_t* rows,
                                             const int* pos, int n_valid, int n, int D, int d0, int bd) {
  const bool vec = (D % 8) == 0 && bd == kBaBd;
  if (vec) {                                         // 16-byte loads: 8 columns per thread
    for (int e = threadIdx.x; e < n * 8; e += kBaThreads) {
      const int i = e >> 3, c = (e & 7) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (i < n_valid && pos[i] >= 0) v = *reinterpret_cast<const uint4*>(src + rows[i] * D + d0 + c);
      *reinterpret_cast<uint4*>(tile + i * kBaLdb + c) = v;
    }
  } else {
    for (int e = threadIdx.x; e < n * 64; e += kBaThreads) {
      const int i = e >> 6, c = e & 63;
      tile[i * kBaLdb + c] = (i < n_valid && pos[i] >= 0 && c < bd) ? src[rows[i] * D + d0 + c]
                                                                   : __float2bfloat16_rn(0.f);
    }
  }
}

template <bool Half>
__global__ void __launch_bounds__(kBaThreads) k_bucket_attn_fwd(const BaArgs a) {
  using T = typename BaT<Half>::T;
  extern __shared__ __align__(16) unsigned char ba_smem[];
  const BaSmem s = ba_carve(ba_smem, a.C, a.P, a.CF, a.K, Half);
  const int64_t r = blockIdx.x;
  const int j = blockIdx.y, C = a.C, C2 = 2 * C, D = a.D, tid = threadIdx.x;
  ba_scores<Half>(a, s, r, j, a.sen);
  const T* V = reinterpret_cast<const T*>(a.v);
  T* out = reinterpret_cast<T*>(a.out);
  if constexpr (Half) {
    // out (32 x 64 per chunk) = attb (32 x 64 keys) . vb (64 keys x 64 columns) on mma.sync; warp: rows 16 (w % 2),
    // columns 16 (w / 2)
    const int lane = tid & 31, wid = tid >> 5, mt = wid & 1, nt = wid >> 1;
    ba_fill_attb(s, C);
    for (int d0 = 0; d0 < D; d0 += kBaBd) {
      const int bd = min(kBaBd, D - d0);
      ba_fill_tile(s.vb, V, s.filk, s.kpos, C2, 64, D, d0, bd);
      __syncthreads();
      float acc[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 64; kk += 16) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ba_ldsm_x4(s.attb + (16 * mt + (lane & 15)) * kBaLdb + kk + (lane >> 4) * 8, a0, a1, a2, a3);
        const int i = lane >> 3;                     // matrix i: k half i % 2, n block i / 2
        ba_ldsm_x4_t(s.vb + (kk + (i & 1) * 8 + (lane & 7)) * kBaLdb + 16 * nt + (i >> 1) * 8, b0, b1, b2, b3);
        ba_mma(acc[0], a0, a1, a2, a3, b0, b1);
        ba_mma(acc[1], a0, a1, a2, a3, b2, b3);
      }
      const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
      for (int jn = 0; jn < 2; ++jn) {
        const int c = 16 * nt + 8 * jn + 2 * t4;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int q = 16 * mt + g + 8 * hh;
          if (q >= C || s.qpos[q] < 0 || c >= bd) continue;
          const int64_t o = (r * a.L + s.qpos[q]) * D + d0 + c;
          out[o] = __float2bfloat16_rn(acc[jn][2 * hh]);
          if (c + 1 < bd) out[o + 1] = __float2bfloat16_rn(acc[jn][2 * hh + 1]);
        }
      }
      __syncthreads();
    }
    return;
  }
  for (int d0 = 0; d0 < D; d0 += kBaBd) {
    const int bd = min(kBaBd, D - d0);
    for (int e = tid; e < C2 * kBaBd; e += kBaThreads) {
      const int k = e / kBaBd, c = e % kBaBd;
      s.vs[k * (kBaBd + 1) + c] = (c < bd && s.kpos[k] >= 0) ? ba_ld<Half>(V, s.filk[k] * D + d0 + c) : 0.f;
    }
    __syncthreads();
    for (int e = tid; e < C * kBaBd; e += kBaThreads) {
      const int q = e / kBaBd, c = e % kBaBd;
      if (c >= bd || s.qpos[q] < 0) continue;
      float acc = 0.f;
      for (int k = 0; k < C2; ++k)
        acc = fmaf(ba_round<Half>(s.att[q * (C2 + 1) + k]), s.vs[k * (kBaBd + 1) + c], acc);
      ba_st<Half>(out, (r * a.L + s.qpos[q]) * D + d0 + c, acc);
    }
    __syncthreads();
  }
}

template <bool Half>
__global__ void __launch_bounds__(kBaThreads) k_bucket_attn_bwd(const BaArgs a) {
  using T = typename BaT<Half>::T;
  extern __shared__ __align__(16) unsigned char ba_smem[];
  const BaSmem s = ba_carve(ba_smem, a.C, a.P, a.CF, a.K, Half);
  const int64_t r = blockIdx.x, L = a.L, BT = a.B * a.T;
  const int j = blockIdx.y, C = a.C, C2 = 2 * C, D = a.D, P = a.P, CF = a.CF, K = a.K, tid = threadIdx.x;
  const int lane = tid & 31, wid = tid >> 5;
  ba_scores<Half>(a, s, r, j, nullptr);
  const T* V = reinterpret_cast<const T*>(a.v);
  const T* dO = reinterpret_cast<const T*>(a.dout);
  T* gv = reinterpret_cast<T*>(a.g_v);
  const bool last_block = j == a.NB - 1;
  // place of key slot k: 1 (current block) or 0 (previous block), row r, text position kpos
  auto lugar_k = [&](int k) { return ((int64_t)(k >= C ? 1 : 0) * BT + r) * L + s.kpos[k]; };
  // dP = dO V^T (per thread: query tid / 8, keys tid % 8 + 8 u) and dV = att^T dO, over chunks of the value columns
  const int iq = tid >> 3;
  float dp[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) dp[u] = 0.f;
  if constexpr (Half) {
    // dP (32 x 64) += ob (32 x chunk) . vb^T and dV chunk (64 keys x 64) = attb^T . ob on mma.sync
    const int g = lane >> 2, t4 = lane & 3, i4 = lane >> 3;
    const int mt = wid & 1, nt = wid >> 1;        // dP tile of this warp: queries 16 mt .., keys 16 nt ..
    const int mk = wid & 3, nh = wid >> 2;        // dV tile: keys 16 mk .., columns 32 nh ..
    float pacc[2][4] = {};
    ba_fill_attb(s, C);
    for (int d0 = 0; d0 < D; d0 += kBaBd) {
      const int bd = min(kBaBd, D - d0);
      ba_fill_tile(s.vb, V, s.filk, s.kpos, C2, 64, D, d0, bd);
      ba_fill_tile(s.ob, dO, s.filq, s.qpos, C, 32, D, d0, bd);
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < 64; kk += 16) {       // K = the chunk's columns
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ba_ldsm_x4(s.ob + (16 * mt + (lane & 15)) * kBaLdb + kk + (lane >> 4) * 8, a0, a1, a2, a3);
        ba_ldsm_x4(s.vb + (16 * nt + (i4 >> 1) * 8 + (lane & 7)) * kBaLdb + kk + (i4 & 1) * 8, b0, b1, b2, b3);
        ba_mma(pacc[0], a0, a1, a2, a3, b0, b1);
        ba_mma(pacc[1], a0, a1, a2, a3, b2, b3);
      }
      float vacc[4][4] = {};
#pragma unroll
      for (int kq = 0; kq < 32; kq += 16) {       // K = the queries
        uint32_t a0, a1, a2, a3;
        // A = att^T (keys x queries) from attb (queries x keys): matrix i = (key half i % 2, query half i / 2)
        ba_ldsm_x4_t(s.attb + (kq + (i4 >> 1) * 8 + (lane & 7)) * kBaLdb + 16 * mk + (i4 & 1) * 8, a0, a1, a2, a3);
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          uint32_t b0, b1, b2, b3;
          ba_ldsm_x4_t(s.ob + (kq + (i4 & 1) * 8 + (lane & 7)) * kBaLdb + 32 * nh + 16 * nb + (i4 >> 1) * 8, b0, b1,
                       b2, b3);
          ba_mma(vacc[2 * nb], a0, a1, a2, a3, b0, b1);
          ba_mma(vacc[2 * nb + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int jn = 0; jn < 4; ++jn) {
        const int c = 32 * nh + 8 * jn + 2 * t4;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int k = 16 * mk + g + 8 * hh;
          if (k >= C2 || s.kpos[k] < 0 || c >= bd) continue;
          const int64_t lk = lugar_k(k) * D + d0 + c, zk = (r * L + s.kpos[k]) * D + d0 + c;
          const bool zero = last_block && k >= C;
          gv[lk] = __float2bfloat16_rn(vacc[jn][2 * hh]);
          if (zero) gv[zk] = __float2bfloat16_rn(0.f);
          if (c + 1 < bd) {
            gv[lk + 1] = __float2bfloat16_rn(vacc[jn][2 * hh + 1]);
            if (zero) gv[zk + 1] = __float2bfloat16_rn(0.f);
          }
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int jn = 0; jn < 2; ++jn) {
      const int k = 16 * nt + 8 * jn + 2 * t4;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int q = 16 * mt + g + 8 * hh;
        if (q < C) {
          if (k < C2) s.ds[q * (C2 + 1) + k] = pacc[jn][2 * hh];
          if (k + 1 < C2) s.ds[q * (C2 + 1) + k + 1] = pacc[jn][2 * hh + 1];
        }
      }
    }
    __syncthreads();
  } else {
  for (int d0 = 0; d0 < D; d0 += kBaBd) {
    const int bd = min(kBaBd, D - d0);
    for (int e = tid; e < C2 * kBaBd; e += kBaThreads) {
      const int k = e / kBaBd, c = e % kBaBd;
      s.vs[k * (kBaBd + 1) + c] = (c < bd && s.kpos[k] >= 0) ? ba_ld<Half>(V, s.filk[k] * D + d0 + c) : 0.f;
    }
    for (int e = tid; e < C * kBaBd; e += kBaThreads) {
      const int q = e / kBaBd, c = e % kBaBd;
      s.os[q * (kBaBd + 1) + c] = (c < bd && s.qpos[q] >= 0) ? ba_ld<Half>(dO, s.filq[q] * D + d0 + c) : 0.f;
    }
    __syncthreads();
    if (iq < C) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int k = (tid & 7) + 8 * u;
        if (k < C2) {
          float acc = dp[u];
          for (int c = 0; c < bd; ++c) acc = fmaf(s.os[iq * (kBaBd + 1) + c], s.vs[k * (kBaBd + 1) + c], acc);
          dp[u] = acc;
        }
      }
    }
    for (int e = tid; e < C2 * kBaBd; e += kBaThreads) {
      const int k = e / kBaBd, c = e % kBaBd;
      if (c >= bd || s.kpos[k] < 0) continue;
      float acc = 0.f;
      for (int q = 0; q < C; ++q)
        acc = fmaf(ba_round<Half>(s.att[q * (C2 + 1) + k]), s.os[q * (kBaBd + 1) + c], acc);
      ba_st<Half>(gv, lugar_k(k) * D + d0 + c, acc);
      if (last_block && k >= C) ba_st<Half>(gv, (r * L + s.kpos[k]) * D + d0 + c, 0.f);
    }
    __syncthreads();
  }
  if (iq < C) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int k = (tid & 7) + 8 * u;
      if (k < C2) s.ds[iq * (C2 + 1) + k] = dp[u];
    }
  }
  __syncthreads();
  }
  // dS = att (dP - sum_k att dP), one warp per query row
  for (int q = wid; q < C; q += kBaThreads / 32) {
    const float* at = s.att + q * (C2 + 1);
    float* dr = s.ds + q * (C2 + 1);
    float t = 0.f;
    for (int k = lane; k < C2; k += 32) t += at[k] * dr[k];
    t = warp_sum(t);
    for (int k = lane; k < C2; k += 32) dr[k] = at[k] * (dr[k] - t);
  }
  __syncthreads();
  const float tasa = a.gamma[r % a.T] / (float)C;
  T* gpq = reinterpret_cast<T*>(a.g_phi_q);
  T* gpk = reinterpret_cast<T*>(a.g_phi_k);
  T* gqc = reinterpret_cast<T*>(a.g_qc);
  T* gkc = reinterpret_cast<T*>(a.g_kc);
  if constexpr (Half) {
    // dS rounded to bf16 into attb (free after the value products), then [dphi_q | dQc] = dS . [phi_k | Kc] and
    // [dphi_k | dKc] = dS^T . [phi_q | Qc] on mma.sync, 16 x 16 output tiles round-robin over the warps
    for (int e = tid; e < 32 * 64; e += kBaThreads) {
      const int q = e >> 6, k = e & 63;
      s.attb[q * kBaLdb + k] = __float2bfloat16_rn(q < C && k < C2 ? s.ds[q * (C2 + 1) + k] : 0.f);
    }
    __syncthreads();
    const int g = lane >> 2, t4 = lane & 3, i4 = lane >> 3;
    const int Pp = ba_pad16(P), Fp = ba_fp(P, CF), ldf = Fp + 8, nfb = Fp / 16;
    // queries: 2 row tiles x nfb column blocks, K = the 64 keys
    for (int tile = wid; tile < 2 * nfb; tile += kBaThreads / 32) {
      const int mt = tile & 1, nb = tile >> 1;
      float acc[2][4] = {};
#pragma unroll
      for (int kk = 0; kk < 64; kk += 16) {
        uint32_t x0, x1, x2, x3, y0, y1, y2, y3;
        ba_ldsm_x4(s.attb + (16 * mt + (lane & 15)) * kBaLdb + kk + (lane >> 4) * 8, x0, x1, x2, x3);
        ba_ldsm_x4_t(s.fk + (kk + (i4 & 1) * 8 + (lane & 7)) * ldf + 16 * nb + (i4 >> 1) * 8, y0, y1, y2, y3);
        ba_mma(acc[0], x0, x1, x2, x3, y0, y1);
        ba_mma(acc[1], x0, x1, x2, x3, y2, y3);
      }
#pragma unroll
      for (int jn = 0; jn < 2; ++jn)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int q = 16 * mt + g + 8 * (e >> 1), c = 16 * nb + 8 * jn + 2 * t4 + (e & 1);
          if (q >= C || s.qpos[q] < 0) continue;
          const int64_t lq = r * L + s.qpos[q];
          if (c < P) gpq[lq * P + c] = __float2bfloat16_rn(acc[jn][e] * a.scale_phi);
          else if (c >= Pp && c - Pp < CF) gqc[lq * CF + (c - Pp)] = __float2bfloat16_rn(acc[jn][e] * a.scale_c);
        }
    }
    // keys: 4 row tiles x nfb column blocks, K = the 32 queries
    for (int tile = wid; tile < 4 * nfb; tile += kBaThreads / 32) {
      const int mk = tile & 3, nb = tile >> 2;
      float acc[2][4] = {};
#pragma unroll
      for (int kq = 0; kq < 32; kq += 16) {
        uint32_t x0, x1, x2, x3, y0, y1, y2, y3;
        ba_ldsm_x4_t(s.attb + (kq + (i4 >> 1) * 8 + (lane & 7)) * kBaLdb + 16 * mk + (i4 & 1) * 8, x0, x1, x2, x3);
        ba_ldsm_x4_t(s.fq + (kq + (i4 & 1) * 8 + (lane & 7)) * ldf + 16 * nb + (i4 >> 1) * 8, y0, y1, y2, y3);
        ba_mma(acc[0], x0, x1, x2, x3, y0, y1);
        ba_mma(acc[1], x0, x1, x2, x3, y2, y3);
      }
#pragma unroll
      for (int jn = 0; jn < 2; ++jn)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 16 * mk + g + 8 * (e >> 1), c = 16 * nb + 8 * jn + 2 * t4 + (e & 1);
          if (k >= C2 || s.kpos[k] < 0) continue;
          const int64_t lk = lugar_k(k), zk = r * L + s.kpos[k];
          const bool zero = last_block && k >= C;
          if (c < P) {
            gpk[lk * P + c] = __float2bfloat16_rn(acc[jn][e] * a.scale_phi);
            if (zero) gpk[zk * P + c] = __float2bfloat16_rn(0.f);
          } else if (c >= Pp && c - Pp < CF) {
            gkc[lk * CF + (c - Pp)] = __float2bfloat16_rn(acc[jn][e] * a.scale_c);
            if (zero) gkc[zk * CF + (c - Pp)] = __float2bfloat16_rn(0.f);
          }
        }
    }
  } else {
  // query-side gradients: dphi_q = dS phi_k, dQc = dS Kc
  for (int e = tid; e < C * (P + CF); e += kBaThreads) {
    const int q = e / (P + CF), c = e % (P + CF);
    if (s.qpos[q] < 0) continue;
    const int64_t lq = r * L + s.qpos[q];
    float acc = 0.f;
    if (c < P) {
      for (int k = 0; k < C2; ++k) acc = fmaf(ba_round<Half>(s.ds[q * (C2 + 1) + k]), s.phk[k * (P + 1) + c], acc);
      ba_st<Half>(gpq, lq * P + c, acc * a.scale_phi);
    } else {
      const int cc = c - P;
      for (int k = 0; k < C2; ++k) acc = fmaf(ba_round<Half>(s.ds[q * (C2 + 1) + k]), s.kcs[k * (CF + 1) + cc], acc);
      ba_st<Half>(gqc, lq * CF + cc, acc * a.scale_c);
    }
  }
  // key-side gradients: dphi_k = dS^T phi_q, dKc = dS^T Qc
  for (int e = tid; e < C2 * (P + CF); e += kBaThreads) {
    const int k = e / (P + CF), c = e % (P + CF);
    if (s.kpos[k] < 0) continue;
    const int64_t lk = lugar_k(k), zk = r * L + s.kpos[k];
    const bool zero = last_block && k >= C;
    float acc = 0.f;
    if (c < P) {
      for (int q = 0; q < C; ++q) acc = fmaf(ba_round<Half>(s.ds[q * (C2 + 1) + k]), s.phq[q * (P + 1) + c], acc);
      ba_st<Half>(gpk, lk * P + c, acc * a.scale_phi);
      if (zero) ba_st<Half>(gpk, zk * P + c, 0.f);
    } else {
      const int cc = c - P;
      for (int q = 0; q < C; ++q) acc = fmaf(ba_round<Half>(s.ds[q * (C2 + 1) + k]), s.qcs[q * (CF + 1) + cc], acc);
      ba_st<Half>(gkc, lk * CF + cc, acc * a.scale_c);
      if (zero) ba_st<Half>(gkc, zk * CF + cc, 0.f);
    }
  }
  }
  // per-key column sums (log_alfa, clock of the key), per-query row sums (clock of the query)
  for (int k = tid; k < C2; k += kBaThreads) {
    if (s.kpos[k] < 0) continue;
    float col = 0.f;
    for (int q = 0; q < C; ++q) col += s.ds[q * (C2 + 1) + k];
    const int64_t lk = lugar_k(k);
    a.g_la[lk] = col;
    a.g_b_k[lk] = tasa * col;
    if (last_block && k >= C) {
      a.g_la[r * L + s.kpos[k]] = 0.f;
      a.g_b_k[r * L + s.kpos[k]] = 0.f;
    }
  }
  for (int q = tid; q < C; q += kBaThreads) {
    if (s.qpos[q] < 0) continue;
    float row = 0.f;
    for (int k = 0; k < C2; ++k) row += s.ds[q * (C2 + 1) + k];
    a.g_b_q[r * L + s.qpos[q]] = -tasa * row;
  }
  // partials of this CTA: sum dS dt (gamma), sum of dS per suffix length (w_suf)
  for (int c = -1; c <= K; ++c) {
    float part = 0.f;
    for (int e = tid; e < C * C2; e += kBaThreads) {
      const int q = e / C2, k = e % C2;
      const float d = s.ds[q * (C2 + 1) + k];
      if (c < 0) {
        const float dt =
            __fadd_rn(__fsub_rn(s.bk[2 * k], s.bq[2 * q]), __fsub_rn(s.bk[2 * k + 1], s.bq[2 * q + 1]));
        part += d * dt;
      } else if (s.largo[q * C2 + k] == c) {
        part += d;
      }
    }
    part = warp_sum(part);
    if (lane == 0) s.red[wid] = part;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < kBaThreads / 32; ++w) t += s.red[w];
      a.partes[(r * a.NB + j) * (K + 2) + 1 + c] = t;
    }
    __syncthreads();
  }
}

// ---- linear-recurrence scan ------------------------------------------------------------------------------------------

constexpr int kScanThreads = 1024;

struct Aff {
  float a, b;                         // x -> a x + b
};
// first f then g: x -> g(f(x))
__device__ __forceinline__ Aff aff_then(Aff f, Aff g) { return {g.a * f.a, fmaf(g.a, f.b, g.b)}; }

// Exclusive block scan of the per-thread maps in thread order; returns the composition of the maps of the threads
// before this one (identity for thread 0).
__device__ Aff block_scan_excl(Aff m, Aff* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  Aff inc = m;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float pa = __shfl_up_sync(0xffffffffu, inc.a, o), pb = __shfl_up_sync(0xffffffffu, inc.b, o);
    if (lane >= o) inc = aff_then(Aff{pa, pb}, inc);
  }
  if (lane == 31) sh[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    Aff w = lane < (int)(blockDim.x >> 5) ? sh[lane] : Aff{1.f, 0.f};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float pa = __shfl_up_sync(0xffffffffu, w.a, o), pb = __shfl_up_sync(0xffffffffu, w.b, o);
      if (lane >= o) w = aff_then(Aff{pa, pb}, w);
    }
    sh[32 + lane] = w;                // inclusive over warps
  }
  __syncthreads();
  const Aff before_warp = wid > 0 ? sh[32 + wid - 1] : Aff{1.f, 0.f};
  float ea = __shfl_up_sync(0xffffffffu, inc.a, 1), eb = __shfl_up_sync(0xffffffffu, inc.b, 1);
  const Aff excl_lane = lane > 0 ? Aff{ea, eb} : Aff{1.f, 0.f};
  return aff_then(before_warp, excl_lane);
}

// S_i = a_i S_{i-1} + b_i (S_{-1} = 0)
__global__ void __launch_bounds__(kScanThreads) k_scan_fwd(int64_t L, const float* a, const float* b, float* S) {
  __shared__ Aff sh[64];
  const int64_t row = blockIdx.x;
  const int64_t per = (L + kScanThreads - 1) / kScanThreads;
  const int64_t lo = threadIdx.x * per, hi = min(L, lo + per);
  const float* ar = a + row * L;
  const float* br = b + row * L;
  Aff m{1.f, 0.f};
  for (int64_t i = lo; i < hi; ++i) m = aff_then(m, Aff{ar[i], br[i]});
  const Aff pre = block_scan_excl(m, sh);
  float x = pre.b;                    // S_{lo - 1} = pre(0)
  for (int64_t i = lo; i < hi; ++i) {
    x = fmaf(ar[i], x, br[i]);
    S[row * L + i] = x;
  }
}

// l_i = g_i + a_{i+1} l_{i+1}; ga_i = l_i S_{i-1}; gb_i = l_i (thread t takes the chunk t counted from the right)
__global__ void __launch_bounds__(kScanThreads) k_scan_bwd(int64_t L, const float* a, const float* S, const float* g,
                                                          float* ga, float* gb) {
  __shared__ Aff sh[64];
  const int64_t row = blockIdx.x;
  const int64_t per = (L + kScanThreads - 1) / kScanThreads;
  const int64_t lo_r = threadIdx.x * per, hi_r = min(L, lo_r + per);   // in reversed index k = L - 1 - i
  const float* ar = a + row * L;
  const float* gr = g + row * L;
  Aff m{1.f, 0.f};
  for (int64_t k = lo_r; k < hi_r; ++k) {
    const int64_t i = L - 1 - k;
    m = aff_then(m, Aff{i + 1 < L ? ar[i + 1] : 0.f, gr[i]});
  }
  const Aff pre = block_scan_excl(m, sh);
  float lam = pre.b;
  for (int64_t k = lo_r; k < hi_r; ++k) {
    const int64_t i = L - 1 - k;
    lam = fmaf(i + 1 < L ? ar[i + 1] : 0.f, lam, gr[i]);
    if (gb) gb[row * L + i] = lam;
    if (ga) ga[row * L + i] = i > 0 ? lam * S[row * L + i - 1] : 0.f;
  }
}

int ba_check(int64_t B, int64_t L, int T, int C, int P, int CF, int K, int D) {
  if (B < 0 || L < 0 || T <= 0 || C <= 0 || P <= 0 || CF < 0 || K < 0 || D <= 0) return ASRN_ERR_ARG;
  if (C > kBaMaxC || P > kMaxPhi || CF > kMaxConfirm || K > kMaxSuffix) return ASRN_ERR_UNSUPPORTED;
  if (ba_smem_bytes(C, P, CF, K, false) > 220 * 1024) return ASRN_ERR_UNSUPPORTED;
  return ASRN_OK;
}

BaArgs ba_args(int64_t B, int64_t L, int T, int C, int P, int CF, int K, int D, const void* phi, const void* Qc,
               const void* Kc, const void* V, const float* Pf, const float* bt_hi, const float* bt_lo,
               const float* log_alfa, const int32_t* orden, const int32_t* ids_o, const float* w_suf,
               const float* gamma, float scale_phi, float scale_c) {
  BaArgs a = {};
  a.B = B;
  a.L = L;
  a.T = T;
  a.C = C;
  a.P = P;
  a.CF = CF;
  a.K = K;
  a.D = D;
  a.NB = (int)((L + C - 1) / C);
  a.phi = phi;
  a.qc = Qc;
  a.kc = Kc;
  a.v = V;
  a.pf = Pf;
  a.bt_hi = bt_hi;
  a.bt_lo = bt_lo;
  a.la = log_alfa;
  a.orden = orden;
  a.ids_o = ids_o;
  a.w_suf = w_suf;
  a.gamma = gamma;
  a.scale_phi = scale_phi;
  a.scale_c = scale_c;
  return a;
}

}  // namespace
}  // namespace asrn

extern "C" {

int asrn_bucket_attn_forward(int64_t B, int64_t L, int32_t T, int32_t C, int32_t P, int32_t CF, int32_t K, int32_t D,
                             const void* phi, const void* Qc, const void* Kc, const void* V, const float* Pf,
                             const float* Bt_hi, const float* Bt_lo, const float* log_alfa, const int32_t* orden,
                             const int32_t* ids_o, const float* w_suf, const float* gamma, float scale_phi,
                             float scale_c, int32_t half, void* out, float* sen, void* stream) {
  using namespace asrn;
  const int chk = ba_check(B, L, T, C, P, CF, K, D);
  if (chk != ASRN_OK) return chk;
  if (B == 0 || L == 0) return ASRN_OK;
  if (!phi || !Qc || !Kc || !V || (K > 0 && !Pf) || !Bt_hi || !Bt_lo || !log_alfa || !orden || !ids_o || !w_suf ||
      !gamma || !out || !sen)
    return ASRN_ERR_ARG;
  BaArgs a = ba_args(B, L, T, C, P, CF, K, D, phi, Qc, Kc, V, Pf, Bt_hi, Bt_lo, log_alfa, orden, ids_o, w_suf, gamma,
                     scale_phi, scale_c);
  a.out = out;
  a.sen = sen;
  const size_t smem = ba_smem_bytes(C, P, CF, K, half != 0);
  const dim3 grid((unsigned)(B * T), (unsigned)a.NB);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (half) {
    cudaFuncSetAttribute(k_bucket_attn_fwd<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bucket_attn_fwd<true><<<grid, kBaThreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(k_bucket_attn_fwd<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bucket_attn_fwd<false><<<grid, kBaThreads, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int asrn_bucket_attn_backward(int64_t B, int64_t L, int32_t T, int32_t C, int32_t P, int32_t CF, int32_t K, int32_t D,
                              const void* phi, const void* Qc, const void* Kc, const void* V, const float* Pf,
                              const float* Bt_hi, const float* Bt_lo, const float* log_alfa, const int32_t* orden,
                              const int32_t* ids_o, const float* w_suf, const float* gamma, float scale_phi,
                              float scale_c, int32_t half, const void* dout, void* g_phi_q, void* g_qc, float* g_b_q,
                              void* g_phi_k, void* g_kc, void* g_v, float* g_la, float* g_b_k, float* partes,
                              void* stream) {
  using namespace asrn;
  const int chk = ba_check(B, L, T, C, P, CF, K, D);
  if (chk != ASRN_OK) return chk;
  if (B == 0 || L == 0) return ASRN_OK;
  if (!phi || !Qc || !Kc || !V || (K > 0 && !Pf) || !Bt_hi || !Bt_lo || !log_alfa || !orden || !ids_o || !w_suf ||
      !gamma || !dout || !g_phi_q || !g_qc || !g_b_q || !g_phi_k || !g_kc || !g_v || !g_la || !g_b_k || !partes)
    return ASRN_ERR_ARG;
  BaArgs a = ba_args(B, L, T, C, P, CF, K, D, phi, Qc, Kc, V, Pf, Bt_hi, Bt_lo, log_alfa, orden, ids_o, w_suf, gamma,
                     scale_phi, scale_c);
  a.dout = dout;
  a.g_phi_q = g_phi_q;
  a.g_qc = g_qc;
  a.g_b_q = g_b_q;
  a.g_phi_k = g_phi_k;
  a.g_kc = g_kc;
  a.g_v = g_v;
  a.g_la = g_la;
  a.g_b_k = g_b_k;
  a.partes = partes;
  const size_t smem = ba_smem_bytes(C, P, CF, K, half != 0);
  const dim3 grid((unsigned)(B * T), (unsigned)a.NB);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (half) {
    cudaFuncSetAttribute(k_bucket_attn_bwd<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bucket_attn_bwd<true><<<grid, kBaThreads, smem, s>>>(a);
  } else {
    cudaFuncSetAttribute(k_bucket_attn_bwd<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_bucket_attn_bwd<false><<<grid, kBaThreads, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int asrn_scan_forward(int64_t rows, int64_t L, const float* a, const float* b, float* S, void* stream) {
  using namespace asrn;
  if (rows < 0 || L < 0) return ASRN_ERR_ARG;
  if (rows == 0 || L == 0) return ASRN_OK;
  if (!a || !b || !S) return ASRN_ERR_ARG;
  k_scan_fwd<<<(unsigned)rows, kScanThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(L, a, b, S);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int asrn_scan_backward(int64_t rows, int64_t L, const float* a, const float* S, const float* g, float* ga, float* gb,
                       void* stream) {
  using namespace asrn;
  if (rows < 0 || L < 0) return ASRN_ERR_ARG;
  if (rows == 0 || L == 0) return ASRN_OK;
  if (!a || !S || !g || (!ga && !gb)) return ASRN_ERR_ARG;
  k_scan_bwd<<<(unsigned)rows, kScanThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(L, a, S, g, ga, gb);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // extern "C"
