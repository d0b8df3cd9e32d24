// O(1) generation step: per-bucket rings, the n-gram Hawkes table and one new token against its candidates.
// Reference: the writer _Escritor (asrn/nucleo.py:1717-1854): rings _anillo_desde / _anillo_meter / _candidatos
// (asrn/nucleo.py:1585-1631), _MemoriaHawkes.cargar / paso (asrn/nucleo.py:1634-1714), _repeticion_o1
// (asrn/nucleo.py:953-960) and the candidate attention _atender_cand (asrn/estable.py:359-372).
//
// Device state per layer (caller-allocated):
//   ring  (B, T, 2^nb, C) int32: text positions of the C most recent bucket mates (slot = rank % C), -1 = empty
//   count (B, T, 2^nb) int32: positions ever put in the bucket
//   hawkes table (B, n, cap) entries {key bits u64, Bu f64, A f32}: per (sequence, n-gram order) an open-addressing
//     table keyed by the fp64 n-gram key (-0.0 stored as +0.0), linear probing, cap a power of two
// Caches per sequence (caller-allocated, position-major): sig (cap_t) f32, Bt f64, log_alfa f32, phi (P) act,
// Kc (cf) act, and the bf16 rows of E (shared by every layer; the value of position k is E[k + 1]).
//
// The position t of the new token is read from device memory (t_pos), so a step is a fixed sequence of launches
// that a CUDA graph can replay; the step kernels append the new token's clock / log_alfa (k_gen_hawkes) and
// phi / Kc (k_gen_attend) to the caches. A t outside [1, cap) sets ASRN_ERR_ARG in the status word and writes
// nothing.
#include "common.cuh"
#include "gate.cuh"
#include "layout.h"

namespace asrn {

namespace {
constexpr uint64_t kEmptyKey = 0xFFF8000000000001ull;   // a NaN payload real keys never have (NaN keys are skipped)

__device__ __forceinline__ uint64_t key_bits(double k) {
  if (k == 0.0) k = 0.0;
  return (uint64_t)__double_as_longlong(k);
}
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x ^= x >> 33; x *= 0xff51afd7ed558ccdull; x ^= x >> 33; x *= 0xc4ceb9fe1a85ec53ull; x ^= x >> 33;
  return x;
}

struct HawkesEntry {
  uint64_t key;
  double bu;
  float a;
  int32_t last;   // while the prompt's table is built: the key's last position; -1 afterwards
};

// Slot of `key` in a table of `cap` entries (power of two); inserts it if absent. found = it was present.
// Returns -1 if the table is full (bounded: at most cap probes).
__device__ __forceinline__ int64_t hawkes_slot(HawkesEntry* tab, int64_t cap, uint64_t key, bool* found) {
  int64_t i = (int64_t)(mix64(key) & (uint64_t)(cap - 1));
  for (int64_t p = 0; p < cap; ++p) {
    const uint64_t k = tab[i].key;
    if (k == key) { *found = true; return i; }
    if (k == kEmptyKey) { tab[i].key = key; *found = false; return i; }
    i = (i + 1) & (cap - 1);
  }
  *found = false;
  return -1;
}

// Lock-free variant for the parallel build: claims an empty slot with a 64-bit CAS (bounded: at most cap probes).
__device__ __forceinline__ int64_t hawkes_slot_atomic(HawkesEntry* tab, int64_t cap, uint64_t key) {
  int64_t i = (int64_t)(mix64(key) & (uint64_t)(cap - 1));
  for (int64_t p = 0; p < cap; ++p) {
    const unsigned long long prev = atomicCAS(reinterpret_cast<unsigned long long*>(&tab[i].key),
                                              (unsigned long long)kEmptyKey, (unsigned long long)key);
    if (prev == kEmptyKey || prev == key) return i;
    i = (i + 1) & (cap - 1);
  }
  return -1;
}

// fp64 key of the (ni + 1) tokens ending at position t (asrn/nucleo.py:175-185: same operations, same order).
__device__ __forceinline__ double ngram_key(const float* sig, int64_t t, int ni, const double* c) {
  double key = 0.0;
  for (int j = 0; j <= ni; ++j) {
    const int64_t p = t - j;
    const double s = (p >= 0) ? (double)sig[p] : __longlong_as_double(0x7ff8000000000000ll);
    key = __dadd_rn(key, __dmul_rn(s, c[j]));
  }
  return key;
}
}  // namespace

// Rings from the prompt's bucket sort: positions < n_valid, the last C of each bucket (asrn/nucleo.py:1585-1607).
__global__ void k_ring_build(int64_t L, int T, int nb, int C, int64_t n_valid, const int32_t* __restrict__ orden,
                             const uint16_t* __restrict__ ids_o, int32_t* __restrict__ ring,
                             int32_t* __restrict__ count, int64_t rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * L) return;
  const int64_t r = i / L, s = i % L;
  const int32_t* ord = orden + r * L;
  const uint16_t* ids = ids_o + r * L;
  const int pos = ord[s];
  if (pos >= n_valid) return;
  const uint16_t id = ids[s];
  // run of this bucket in the sorted row: [lo, hi); positions ascend inside it
  int64_t lo = 0, hi = s;
  while (lo < hi) { const int64_t m = (lo + hi) >> 1; if (ids[m] < id) lo = m + 1; else hi = m; }
  const int64_t start = lo;
  lo = s; hi = L;
  while (lo < hi) { const int64_t m = (lo + hi) >> 1; if (ids[m] <= id && ord[m] < n_valid) lo = m + 1; else hi = m; }
  const int64_t cnt = lo - start;                     // positions < n_valid in the bucket
  const int64_t rank = s - start;
  const int64_t cell = r * ((int64_t)1 << nb) + id;
  if (rank == 0) count[cell] = (int32_t)cnt;
  if (rank >= cnt - C) ring[cell * C + rank % C] = pos;
}

// Hawkes state at the end of the prompt: for every n-gram key of (b, order) its last occurrence p gives
// Bu = Bt[p], A = hawkes[p] + exp(log_alfa[p]) (asrn/nucleo.py:1656-1681). Two passes: every position inserts its
// key and raises the entry's last position (atomicMax, so the result does not depend on thread order); then every
// entry reads the state of its last position.
__global__ void k_hawkes_insert(int64_t B, int64_t L, int64_t ld, int n, const float* __restrict__ sig,
                                const double* __restrict__ cv, HawkesEntry* tab, int64_t cap, int* status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (b * n + ni) * L + p
  if (i >= B * n * L) return;
  const int64_t row = i / L, p = i % L;
  const int64_t b = row / n;
  const int ni = (int)(row % n);
  const double key = ngram_key(sig + b * ld, p, ni, cv);
  if (key != key) return;
  HawkesEntry* t = tab + row * cap;
  const int64_t e = hawkes_slot_atomic(t, cap, key_bits(key));
  if (e < 0) { atomicCAS(status, ASRN_OK, ASRN_ERR_WORKSPACE); return; }
  atomicMax(&t[e].last, (int32_t)p);
}

__global__ void k_hawkes_fill(int64_t B, int64_t L, int64_t ld, int n, const double* __restrict__ Bt,
                              const float* __restrict__ la, const float* __restrict__ hawkes, HawkesEntry* tab,
                              int64_t cap) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (b * n + ni) * cap + slot
  if (i >= B * n * cap) return;
  HawkesEntry& e = tab[i];
  const int32_t p = e.last;
  if (p < 0) return;
  const int64_t row = i / cap;
  const int64_t b = row / n;
  const int ni = (int)(row % n);
  e.bu = Bt[b * ld + p];
  e.a = hawkes[(b * L + p) * n + ni] + expf(la[b * ld + p]);
  e.last = -1;
}

// One new token per sequence against its candidates (asrn/estable.py:359-372, asrn/nucleo.py:1621-1631).
// Block (b, column slice of kGenCols), warp w = table w (and w + 8, ...): lane j scores ring slot j (its phi and Kc
// rows by 16-byte loads, all in flight together), the warp's softmax, then the warp adds att * E[k + 1] of its 32
// slots for the block's columns (lane: 4 consecutive columns; slots broadcast by shuffles, the 32 row loads unrolled).
// The per-table partial sums are added in table order, so acc (B, d) is written once, deterministically.
constexpr int kGenCols = 128;
constexpr int kGenThreads = 256;
constexpr int kGenWarps = kGenThreads / 32;

template <bool Half>
__device__ __forceinline__ void load4(const typename Act<Half>::T* p, float* v) {
  if constexpr (Half) {
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    const float4 x = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  }
}

// dot of the shared-memory query x with a row of n act values (n a multiple of the 16-byte chunk): batches of 8
// chunk loads in flight
template <bool Half>
__device__ __forceinline__ float dot_act_row(const float* x, const typename Act<Half>::T* row, int n) {
  constexpr int VW = Half ? 8 : 4;
  const int nc = n / VW;
  float acc = 0.f;
  for (int c0 = 0; c0 < nc; c0 += 8) {
    uint4 raw[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      raw[u] = (c0 + u < nc) ? __ldg(reinterpret_cast<const uint4*>(row) + c0 + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (c0 + u >= nc) break;
      const float* xc = x + (c0 + u) * VW;
      if constexpr (Half) {
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(p[e]);
          acc = fmaf(xc[2 * e], f.x, acc);
          acc = fmaf(xc[2 * e + 1], f.y, acc);
        }
      } else {
        const float* f = reinterpret_cast<const float*>(&raw[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc = fmaf(xc[e], f[e], acc);
      }
    }
  }
  return acc;
}

// With ga.cbuf set (bf16 mode), the block also writes the gate's GEMM operand c = bf16(acc / max(1, pt)) for its
// columns, and block (b, 0) the gate value sigma of sequence b (gate_of_token on the block's own table signals), so
// the gate kernel only multiplies.
template <bool Half>
__global__ void __launch_bounds__(kGenThreads) k_gen_attend(GenArgs a, GateArgs ga) {
  using A = Act<Half>;
  const int64_t b = blockIdx.x;
  const int col0 = blockIdx.y * kGenCols;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int T = a.T, C = a.C, P = a.P, cf = a.cf, K = a.K;
  const int64_t t = *a.t_pos;
  if (t < 1 || t >= a.cap) {
    if (threadIdx.x == 0 && b == 0 && blockIdx.y == 0) atomicCAS(a.status, ASRN_OK, ASRN_ERR_ARG);
    return;
  }
  __shared__ float s_q[kMaxPhi + kMaxConfirm];
  __shared__ __align__(16) float s_part[kMaxTables][kGenCols];
  __shared__ uint8_t s_hay[kMaxTables];
  __shared__ float s_mx[kMaxTables], s_pk[kMaxTables];
  const typename A::T* phi_q = reinterpret_cast<const typename A::T*>(a.phi_t) + b * P;
  const typename A::T* qc_q = reinterpret_cast<const typename A::T*>(a.qc_t) + b * cf;
  for (int i = threadIdx.x; i < P + cf; i += blockDim.x) s_q[i] = i < P ? A::load(phi_q + i) : A::load(qc_q + i - P);
  if (blockIdx.y == 0) {   // append the new token's phi and Kc (no candidate of this step is position t)
    typename A::T* pc = reinterpret_cast<typename A::T*>(a.phi_cache_w) + (b * a.cap + t) * P;
    typename A::T* kc = reinterpret_cast<typename A::T*>(a.kc_cache_w) + (b * a.cap + t) * cf;
    const typename A::T* kt = reinterpret_cast<const typename A::T*>(a.kc_t) + b * cf;
    for (int i = threadIdx.x; i < P + cf; i += blockDim.x) {
      if (i < P) pc[i] = phi_q[i];
      else kc[i - P] = kt[i - P];
    }
  }
  __syncthreads();
  const float* sg = a.sig_cache + b * a.cap;
  const double Bq = a.bt_cache[b * a.cap + t];
  float q_prev[kMaxSuffix];
#pragma unroll
  for (int c = 0; c < kMaxSuffix; ++c) q_prev[c] = (c < K && t - 1 - c >= 0) ? sg[t - 1 - c] : 0.f;
  const typename A::T* Ea = reinterpret_cast<const typename A::T*>(a.ea_cache) + b * a.cap * (int64_t)a.d;
  const int jc = col0 + 4 * lane;                  // this lane's 4 columns
  const bool cols_ok = jc < a.d;
  for (int tau = wid; tau < T; tau += kGenWarps) {
    const uint16_t id = a.ids_t[b * T + tau];
    const int32_t* slots = a.ring + ((b * T + tau) * ((int64_t)1 << a.nb) + id) * C;
    const int pos = lane < C ? slots[lane] : -1;
    const bool valid = pos >= 0;
    const int pr = valid ? pos : 0;
    const int64_t gk = b * a.cap + pr;
    const float dphi = dot_act_row<Half>(s_q, reinterpret_cast<const typename A::T*>(a.phi_cache) + gk * P, P);
    const float dqk = dot_act_row<Half>(s_q + P, reinterpret_cast<const typename A::T*>(a.kc_cache) + gk * cf, cf);
    float k_prev[kMaxSuffix];
#pragma unroll
    for (int c = 0; c < kMaxSuffix; ++c) k_prev[c] = (c < K && pr - 1 - c >= 0) ? sg[pr - 1 - c] : 0.f;
    const double bk = a.bt_cache[gk];
    const float lak = a.la_cache[gk];
    float sc = -INFINITY;
    if (valid) {
      float t1;
      if (Half) {
        const float s1 = round_bf16(__fdiv_rn(round_bf16(dphi), a.inv_temp_div));
        const float s2 = round_bf16(__fmul_rn(round_bf16(dqk), a.esc_c));
        t1 = round_bf16(__fadd_rn(s1, s2));
      } else {
        t1 = __fadd_rn(__fdiv_rn(dphi, a.inv_temp_div), __fmul_rn(dqk, a.esc_c));
      }
      int ln = 0;
      bool run = true;
#pragma unroll
      for (int c = 0; c < kMaxSuffix; ++c) {
        if (c < K && run && t - 1 - c >= 0 && pr - 1 - c >= 0 && q_prev[c] == k_prev[c]) ++ln;
        else run = false;
      }
      t1 = __fadd_rn(t1, a.w_suf[ln]);
      // _atender_cand: nucleo = log_alfa_k - (gamma / C) * float(B_q - B_k), added after the suffix weight
      const float dB = __double2float_rn(Bq - bk);
      sc = __fadd_rn(t1, __fsub_rn(lak, __fmul_rn(a.tasa[tau], dB)));
    }
    const bool any = __any_sync(0xffffffffu, valid);
    float att = 0.f;
    if (any) {
      const float mx = warp_max(sc);
      const float e = valid ? expf(__fsub_rn(sc, mx)) : 0.f;
      const float sum = warp_sum(e);
      att = __fdiv_rn(e, sum);
      const float peak = warp_max(att);
      if (lane == 0) {
        s_hay[tau] = 1;
        s_mx[tau] = mx;
        s_pk[tau] = peak;
      }
    } else if (lane == 0) {
      s_hay[tau] = 0;
      s_mx[tau] = kProhibido;
      s_pk[tau] = 0.f;
    }
    if (Half) att = round_bf16(att);
    // sum over this table's slots of att * E[pos + 1][cols] (invalid slots have att 0 and read row 1)
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    if (any) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[16][4];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int pc = __shfl_sync(0xffffffffu, pr, 16 * h + c);
          if (cols_ok) load4<Half>(Ea + (int64_t)(pc + 1) * a.d + jc, v[c]);
          else v[c][0] = v[c][1] = v[c][2] = v[c][3] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float w = __shfl_sync(0xffffffffu, att, 16 * h + c);
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = fmaf(w, v[c][e], o[e]);
        }
      }
    }
    *reinterpret_cast<float4*>(&s_part[tau][4 * lane]) = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (blockIdx.y == 0 && threadIdx.x < T) {
    a.sen_hay[b * T + threadIdx.x] = s_hay[threadIdx.x];
    a.sen_mx[b * T + threadIdx.x] = s_mx[threadIdx.x];
    a.sen_pk[b * T + threadIdx.x] = s_pk[threadIdx.x];
  }
  if (ga.sigma && blockIdx.y == 0 && threadIdx.x == 0) {
    GateArgs g = ga;
    g.sen_hay = s_hay; g.sen_mx = s_mx; g.sen_pk = s_pk;
    g.glogit = ga.glogit + b; g.vistos = ga.vistos + b * ga.n; g.hawkes = ga.hawkes + b * ga.n; g.racha = ga.racha + b;
    float sg, ptc;
    gate_of_token<Half>(g, 0, &sg, &ptc);
    ga.sigma[b] = sg;
  }
  float pt1 = 1.f;
  if (ga.cbuf) {
    float pt = 0.f;
    for (int tau = 0; tau < T; ++tau) pt = __fadd_rn(pt, (float)s_hay[tau]);
    pt1 = fmaxf(pt, 1.f);
  }
  if (threadIdx.x < kGenCols) {
    const int j = col0 + threadIdx.x;
    if (j < a.d) {
      float sum = 0.f;
      for (int tau = 0; tau < T; ++tau) sum = __fadd_rn(sum, s_part[tau][threadIdx.x]);
      a.acc[b * a.d + j] = sum;
      if (ga.cbuf) ga.cbuf[b * a.d + j] = __float2bfloat16_rn(__fdiv_rn(sum, pt1));
    }
  }
}

// n-gram memory of the new token (asrn/nucleo.py:1683-1714) and the streak (asrn/nucleo.py:953-960).
// One thread per (sequence, order): each order has its own table; the order-0 thread appends the clock and
// log_alfa of the new token, the last order's thread updates the streak from its "seen" flag.
__global__ void k_gen_hawkes(GenArgs a, HawkesEntry* tab, int64_t hcap, const double* cv, const float* kappa,
                             const double* beta_t, const float* la_t, float* racha_state, uint8_t* vistos,
                             float* hawkes, float* racha_out, int* status) {
  const int n = a.n;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.B * n) return;
  const int64_t b = i / n;
  const int ni = (int)(i % n);
  const int64_t t = *a.t_pos;
  if (t < 1 || t >= a.cap) {
    if (i == 0) atomicCAS(status, ASRN_OK, ASRN_ERR_ARG);
    return;
  }
  // the new token's clock: the inclusive fp64 sum, one more term
  const double Bq = a.bt_w[b * a.cap + t - 1] + beta_t[b];
  if (ni == 0) {
    a.bt_w[b * a.cap + t] = Bq;
    a.la_w[b * a.cap + t] = la_t[b];
  }
  const float alpha = expf(la_t[b]);
  const double key = ngram_key(a.sig_cache + b * a.cap, t, ni, cv);
  float lam = 0.f;
  bool seen = false;
  if (key == key) {
    bool found;
    HawkesEntry* tb = tab + (b * n + ni) * hcap;
    const int64_t e = hawkes_slot(tb, hcap, key_bits(key), &found);
    if (e < 0) {
      atomicCAS(status, ASRN_OK, ASRN_ERR_WORKSPACE);
    } else {
      if (found) {
        const float dB = __double2float_rn(Bq - tb[e].bu);
        lam = __fmul_rn(expf(__fmul_rn(-kappa[ni], dB)), tb[e].a);
        seen = true;
      }
      tb[e].bu = Bq;
      tb[e].a = __fadd_rn(lam, alpha);
    }
  }
  vistos[b * n + ni] = seen ? 1 : 0;
  hawkes[b * n + ni] = lam;
  if (ni == n - 1) {
    const float r = seen ? 1.f : 0.f;
    const float e = expf(__fmul_rn(-kappa[n], (float)beta_t[b]));
    const float s = __fmul_rn(r, __fadd_rn(__fmul_rn(e, racha_state[b]), 1.f));
    racha_out[b] = s;
    racha_state[b] = s;
  }
}

// Ring insert of position t for every (sequence, table) (asrn/nucleo.py:1610-1618).
__global__ void k_ring_insert(int64_t B, int T, int nb, int C, const int64_t* __restrict__ t_pos,
                              const uint16_t* __restrict__ ids_t, int32_t* __restrict__ ring,
                              int32_t* __restrict__ count) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * T) return;
  const int64_t t = *t_pos;
  const int64_t cell = i * ((int64_t)1 << nb) + ids_t[i];
  const int32_t c = count[cell];
  ring[cell * C + (c % C)] = (int32_t)t;
  count[cell] = c + 1;
}

// ---- launchers ---------------------------------------------------------------------------------------------------

size_t hawkes_table_bytes(int64_t B, int n, int64_t cap) { return (size_t)B * n * cap * sizeof(HawkesEntry); }

int launch_ring_build(int64_t B, int64_t L, int T, int nb, int C, int64_t n_valid, const int32_t* orden,
                      const uint16_t* ids_o, int32_t* ring, int32_t* count, cudaStream_t s) {
  const size_t cells = (size_t)B * T * ((size_t)1 << nb);
  if (cudaMemsetAsync(ring, 0xFF, cells * C * 4, s) != cudaSuccess) return ASRN_ERR_CUDA;
  if (cudaMemsetAsync(count, 0, cells * 4, s) != cudaSuccess) return ASRN_ERR_CUDA;
  const int64_t n = B * T * L;
  if (n > 0) k_ring_build<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(L, T, nb, C, n_valid, orden, ids_o, ring, count,
                                                                      B * T);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

__global__ void k_hawkes_clear(HawkesEntry* tab, int64_t entries) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < entries) {
    tab[i].key = kEmptyKey;
    tab[i].bu = 0.0;
    tab[i].a = 0.f;
    tab[i].last = -1;
  }
}

int launch_hawkes_build(int64_t B, int64_t L, int64_t ld, int n, const float* sig, const double* cv, const double* Bt,
                        const float* la, const float* hawkes, void* table, int64_t cap, int* status, cudaStream_t s) {
  if (cap <= 0 || (cap & (cap - 1)) != 0) return ASRN_ERR_ARG;
  const int64_t entries = B * n * cap;
  HawkesEntry* tab = reinterpret_cast<HawkesEntry*>(table);
  if (entries > 0) k_hawkes_clear<<<(unsigned)((entries + 255) / 256), 256, 0, s>>>(tab, entries);
  const int64_t pts = B * n * L;
  if (pts > 0) {
    k_hawkes_insert<<<(unsigned)((pts + 255) / 256), 256, 0, s>>>(B, L, ld, n, sig, cv, tab, cap, status);
    k_hawkes_fill<<<(unsigned)((entries + 255) / 256), 256, 0, s>>>(B, L, ld, n, Bt, la, hawkes, tab, cap);
  }
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_gen_attend(const GenArgs& a, const GateArgs& ga, bool half, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  if (a.C > 32 || a.P > kMaxPhi || a.cf > kMaxConfirm || a.T > kMaxTables || a.K > kMaxSuffix) return ASRN_ERR_UNSUPPORTED;
  // 16-byte rows of phi / Kc and 4-column value loads
  const int vw = half ? 8 : 4;
  if (a.P % vw != 0 || a.cf % vw != 0 || a.d % 4 != 0) return ASRN_ERR_UNSUPPORTED;
  dim3 grid((unsigned)a.B, (unsigned)((a.d + kGenCols - 1) / kGenCols));
  if (half) k_gen_attend<true><<<grid, kGenThreads, 0, s>>>(a, ga);
  else k_gen_attend<false><<<grid, kGenThreads, 0, s>>>(a, ga);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_gen_memory(const GenArgs& a, void* table, int64_t hcap, const double* cv, const float* kappa,
                      const double* beta_t, const float* la_t, float* racha_state, uint8_t* vistos, float* hawkes,
                      float* racha, int* status, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  if (hcap <= 0 || (hcap & (hcap - 1)) != 0) return ASRN_ERR_ARG;
  const int64_t threads = a.B * a.n;
  k_gen_hawkes<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(a, reinterpret_cast<HawkesEntry*>(table), hcap, cv,
                                                                kappa, beta_t, la_t, racha_state, vistos, hawkes,
                                                                racha, status);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_ring_insert(int64_t B, int T, int nb, int C, const int64_t* t_pos, const uint16_t* ids_t, int32_t* ring,
                       int32_t* count, cudaStream_t s) {
  const int64_t n = B * T;
  if (n == 0) return ASRN_OK;
  k_ring_insert<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(B, T, nb, C, t_pos, ids_t, ring, count);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

}  // namespace asrn
