// Candidate scoring ("bucket attention") of every (table row, sorted slot).
// Reference: CapaASRNEstable._acumular (asrn/estable.py:204-300) and its fused seam _casilleros_ida
// (asrn/nucleo.py:279-382). For the query at sorted slot s of row r = b*T + tau the candidates are the sorted slots
// [s - C, s) with the same bucket id (the "previous + current block" window restricted by `anteriores`,
// asrn/estable.py:262-265) -- because the row is sorted by id they are a contiguous run just before s. Score:
//   sc = <phi_q, phi_k> / temperature + <Qc_q, Kc_k> cf^-1/2 + w_sufijo[suffix length] + log_alfa_k
//        + (gamma_tau / C) * float(B_k - B_q)                      (clock difference in fp64, asrn/estable.py:101-118)
// in exactly that order of fp32 additions (bf16 rounding of the two dot-product terms under autocast), exact-mask
// softmax over the candidates (asrn/estable.py:121-138), and the copy of the next token's value: the kernel adds
// att * Ea[k + 1] into acc[b, t_q] (the table sum of _DesordenarSumar, asrn/nucleo.py:116-133) with vector
// reductions in L2 (fp32, or bf16 into the bf16 accumulator of autocast mode); the gate applies W_o W_v to it.
// Per-table gate signals (hay, max, peak) go to (B, L, T).
//
// Blocks run row-major over (b, tau) so every table of a sequence is scored together and the sequence's
// accumulator stays resident in L2 while its T tables add into it.
#include "common.cuh"
#include "layout.h"

namespace asrn {

constexpr int kSpan = 256;   // sorted slots per block
constexpr int kRing = 64;    // ring of slot features: the 32 queries of a sub-tile plus up to 32 earlier slots

struct ScoreSmem {
  int* pos;
  int* id;
  double* bt;
  float* la;
  float* pf;
  float* phi;
  float* qc;
  float* kc;
  int Pp, Cp, K;
};

__device__ __forceinline__ ScoreSmem carve_score(char* base, int P, int cf, int K) {
  ScoreSmem s;
  s.Pp = P + 1;
  s.Cp = cf + 1;
  s.K = K;
  s.bt = reinterpret_cast<double*>(base);
  s.pos = reinterpret_cast<int*>(s.bt + kRing);
  s.id = s.pos + kRing;
  s.la = reinterpret_cast<float*>(s.id + kRing);
  s.pf = s.la + kRing;
  s.phi = s.pf + kRing * K;
  s.qc = s.phi + kRing * s.Pp;
  s.kc = s.qc + kRing * s.Cp;
  return s;
}

static size_t score_smem_bytes(int P, int cf, int K) {
  return (size_t)kRing * (8 + 4 + 4 + 4 + 4 * K + 4 * (P + 1) + 8 * (cf + 1));
}

template <bool Half>
__device__ __forceinline__ void load_slots(const ScoreArgs& a, const ScoreSmem& S, int64_t r, int64_t b, int tau,
                                           int64_t s_begin, int64_t s_end) {
  using A = Act<Half>;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const typename A::T* phi = reinterpret_cast<const typename A::T*>(a.phi);
  const typename A::T* Qc = reinterpret_cast<const typename A::T*>(a.Qc);
  const typename A::T* Kc = reinterpret_cast<const typename A::T*>(a.Kc);
  for (int64_t s = s_begin + wid; s < s_end; s += 8) {
    const int ri = (int)(s & (kRing - 1));
    const bool real = s >= 0 && s < a.L;
    const int pos = real ? a.orden[r * a.L + s] : 0;
    const int64_t g = b * a.Lf + pos;
    if (lane == 0) {
      S.pos[ri] = pos;
      S.id[ri] = real ? (int)a.ids_o[r * a.L + s] : -1;
      S.bt[ri] = real ? a.Bt[g] : 0.0;
      S.la[ri] = real ? a.log_alfa[g] : 0.f;
    }
    if (lane < S.K) {
      const int t = pos - 1 - lane;
      S.pf[ri * S.K + lane] = (real && t >= 0) ? a.sig[b * a.Lf + t] : __int_as_float(0x7fc00000);
    }
    if (real) {
      for (int p = lane; p < a.P; p += 32) S.phi[ri * S.Pp + p] = A::load(phi + g * a.P + p);
      for (int c = lane; c < a.cf; c += 32) {
        S.qc[ri * S.Cp + c] = A::load(Qc + g * a.cf + c);
        S.kc[ri * S.Cp + c] = A::load(Kc + g * a.cf + c);
      }
    }
  }
}

template <bool Half> struct Vec4Load;
template <> struct Vec4Load<false> {
  static ASRN_DEV float4 load(const float* p) { return *reinterpret_cast<const float4*>(p); }
};
template <> struct Vec4Load<true> {
  static ASRN_DEV float4 load(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    return make_float4(a.x, a.y, b.x, b.y);
  }
};

template <bool Half, bool Vec>
__global__ void __launch_bounds__(256) k_score_simt(ScoreArgs a) {
  using A = Act<Half>;
  extern __shared__ __align__(16) char smem_raw[];
  const ScoreSmem S = carve_score(smem_raw, a.P, a.cf, a.K);
  const int64_t r = blockIdx.y;
  const int64_t b = r / a.T;
  const int tau = (int)(r % a.T);
  const int64_t S0 = (int64_t)blockIdx.x * kSpan;
  const int64_t S1 = min(min(S0 + kSpan, a.L), a.row_len ? a.row_len[r] : a.L);
  if (S0 >= S1) return;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const float tasa = a.tasa[tau];
  const typename A::T* Ea = reinterpret_cast<const typename A::T*>(a.Ea);
  const int d = a.d;
  constexpr int kMaxChunks = 8;   // d <= 1024: float4 chunks per lane
  for (int64_t q0 = S0; q0 < S1; q0 += 32) {
    load_slots<Half>(a, S, r, b, tau, q0 == S0 ? q0 - a.C : q0, q0 + 32);
    __syncthreads();
    for (int qi = wid; qi < 32; qi += 8) {
      const int64_t q = q0 + qi;
      if (q >= S1) break;
      const int rq = (int)(q & (kRing - 1));
      const int idq = S.id[rq];
      const int64_t ks = q - 1 - lane;
      const bool ok = lane < a.C && ks >= 0 && S.id[ks & (kRing - 1)] == idq;
      const int nv = __popc(__ballot_sync(0xffffffffu, ok));
      const int pos_q = S.pos[rq];
      if (pos_q < a.q_lo || pos_q >= a.q_hi) continue;    // a key only (positions of another shard)
      const int64_t gq = b * (a.q_hi - a.q_lo) + (pos_q - a.q_lo);
      if (nv == 0) {
        if (lane == 0) {
          a.sen_hay[gq * a.T + tau] = 0;
          a.sen_mx[gq * a.T + tau] = kProhibido;
          a.sen_pk[gq * a.T + tau] = 0.f;
        }
        continue;
      }
      float sc = -INFINITY;
      int kpos = 0;
      if (lane < nv) {
        const int rk = (int)(ks & (kRing - 1));
        kpos = S.pos[rk];
        const float* pq = S.phi + rq * S.Pp;
        const float* pk = S.phi + rk * S.Pp;
        float dphi = 0.f;
        for (int p = 0; p < a.P; ++p) dphi = fmaf(pq[p], pk[p], dphi);
        const float* cq = S.qc + rq * S.Cp;
        const float* ck = S.kc + rk * S.Cp;
        float dqk = 0.f;
        for (int c = 0; c < a.cf; ++c) dqk = fmaf(cq[c], ck[c], dqk);
        float t1;
        if (Half) {
          const float s1 = round_bf16(__fdiv_rn(round_bf16(dphi), a.inv_temp_div));
          const float s2 = round_bf16(__fmul_rn(round_bf16(dqk), a.esc_c));
          t1 = round_bf16(__fadd_rn(s1, s2));
        } else {
          t1 = __fadd_rn(__fdiv_rn(dphi, a.inv_temp_div), __fmul_rn(dqk, a.esc_c));
        }
        int ln = 0;
        for (int c = 0; c < a.K; ++c) {
          if (S.pf[rq * S.K + c] == S.pf[rk * S.K + c]) ++ln; else break;
        }
        t1 = __fadd_rn(t1, a.w_suf[ln]);
        t1 = __fadd_rn(t1, S.la[rk]);
        const float dt = __double2float_rn(S.bt[rk] - S.bt[rq]);
        t1 = __fadd_rn(t1, __fmul_rn(dt, tasa));
        sc = t1;
      }
      const float mx = warp_max(sc);
      const float e = (lane < nv) ? expf(__fsub_rn(sc, mx)) : 0.f;
      const float sum = warp_sum(e);
      const float att = __fdiv_rn(e, sum);
      const float peak = warp_max(att);
      if (lane == 0) {
        a.sen_hay[gq * a.T + tau] = 1;
        a.sen_mx[gq * a.T + tau] = mx;
        a.sen_pk[gq * a.T + tau] = peak;
      }
      const float w = Half ? round_bf16(att) : att;
      float* dst = reinterpret_cast<float*>(a.acc) + gq * d;                       // fp32 accumulator
      __nv_bfloat16* dst16 = reinterpret_cast<__nv_bfloat16*>(a.acc) + gq * d;    // bf16 accumulator
      if (Vec) {
        const int nch = d >> 2;
        float4 o[kMaxChunks];
#pragma unroll
        for (int i = 0; i < kMaxChunks; ++i) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < nv; ++j) {
          const float wj = __shfl_sync(0xffffffffu, w, j);
          const int kp = __shfl_sync(0xffffffffu, kpos, j);
          if (kp + 1 >= a.Lf) continue;
          const typename A::T* row = Ea + (b * a.Lf + kp + 1) * (int64_t)d;
#pragma unroll
          for (int i = 0; i < kMaxChunks; ++i) {
            const int c4 = lane + 32 * i;
            if (c4 < nch) {
              const float4 v = Vec4Load<Half>::load(row + 4 * c4);
              o[i].x = fmaf(wj, v.x, o[i].x);
              o[i].y = fmaf(wj, v.y, o[i].y);
              o[i].z = fmaf(wj, v.z, o[i].z);
              o[i].w = fmaf(wj, v.w, o[i].w);
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kMaxChunks; ++i) {
          const int c4 = lane + 32 * i;
          if (c4 < nch) {
            if (Half) red_add_bf16x4(dst16 + 4 * c4, o[i].x, o[i].y, o[i].z, o[i].w);
            else red_add_v4(dst + 4 * c4, o[i].x, o[i].y, o[i].z, o[i].w);
          }
        }
      } else {
        for (int c = lane; c < d; c += 32) {
          float o = 0.f;
          for (int j = 0; j < nv; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const int kp = __shfl_sync(0xffffffffu, kpos, j);
            if (kp + 1 < a.Lf) o = fmaf(wj, A::load(Ea + (b * a.Lf + kp + 1) * (int64_t)d + c), o);
          }
          if (Half) red_add_bf16(dst16 + c, o);
          else red_add_f32(dst + c, o);
        }
      }
    }
    __syncthreads();
  }
}

// Debug view of the candidate windows (the selection rule of k_score_simt, on global arrays): for (row r, slot s),
// cand[(r*L + s)*C + j] = text position of slot s-1-j if it is a bucket mate (else -1) and suffix[...] its
// suffix-match length with the query (asrn/nucleo.py:98-108, NaN signature before the start never matches).
__global__ void k_candidates(int64_t L, int T, int C, int K, const int32_t* __restrict__ orden,
                             const uint16_t* __restrict__ ids_o, const float* __restrict__ sig,
                             int32_t* __restrict__ cand, uint8_t* __restrict__ suffix, int64_t rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * L) return;
  const int64_t r = i / L, s = i % L;
  const int64_t b = r / T;
  const uint16_t idq = ids_o[r * L + s];
  const int pq = orden[r * L + s];
  bool run = true;
  for (int j = 0; j < C; ++j) {
    const int64_t k = s - 1 - j;
    run = run && k >= 0 && ids_o[r * L + k] == idq;
    int32_t pos = -1;
    int ln = 0;
    if (run) {
      pos = orden[r * L + k];
      for (int c = 0; c < K; ++c) {
        const int64_t tq = pq - 1 - c, tk = pos - 1 - c;
        if (tq >= 0 && tk >= 0 && sig[b * L + tq] == sig[b * L + tk]) ++ln; else break;
      }
    }
    cand[i * C + j] = pos;
    suffix[i * C + j] = (uint8_t)ln;
  }
}

int launch_candidates(int64_t B, int64_t L, int T, int C, int K, const int32_t* orden, const uint16_t* ids_o,
                      const float* sig, int32_t* cand, uint8_t* suffix, cudaStream_t s) {
  const int64_t n = B * T * L;
  if (n == 0) return ASRN_OK;
  if (C < 1 || C > 32 || K < 1 || K > kMaxSuffix) return ASRN_ERR_ARG;
  k_candidates<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(L, T, C, K, orden, ids_o, sig, cand, suffix, B * T);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

template <bool Half, bool Vec>
static void launch_score_t(const ScoreArgs& a, cudaStream_t s, size_t smem) {
  cudaFuncSetAttribute(k_score_simt<Half, Vec>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((unsigned)((a.L + kSpan - 1) / kSpan), (unsigned)(a.B * a.T));
  k_score_simt<Half, Vec><<<grid, 256, smem, s>>>(a);
}

bool score_tc_supported(const ScoreArgs& a);
int launch_score_tc(const ScoreArgs& a, cudaStream_t s);

int launch_score(const ScoreArgs& a, bool half, cudaStream_t s) {
  if (a.B == 0 || a.L == 0) return ASRN_OK;
  if (a.C < 1 || a.C > 32 || a.d > 1024 || a.P > kMaxPhi || a.cf > kMaxConfirm || a.K > kMaxSuffix)
    return ASRN_ERR_UNSUPPORTED;
  if (half && tensor_cores_enabled() && score_tc_supported(a)) return launch_score_tc(a, s);
  const size_t smem = score_smem_bytes(a.P, a.cf, a.K);
  const bool vec = (a.d % 4) == 0;
  if (half) {
    if (vec) launch_score_t<true, true>(a, s, smem); else launch_score_t<true, false>(a, s, smem);
  } else {
    if (vec) launch_score_t<false, true>(a, s, smem); else launch_score_t<false, false>(a, s, smem);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
