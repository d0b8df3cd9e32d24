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
// Block (b, column slice of kGenCols): warp w scores the C ring slots of tables w, w + 8, ... (lane j = slot j; every
// column block recomputes these few dot products), then the block sums att * E[k + 1] over all tables for its
// columns: four thread groups take tables g, g + 4, ... in order and their partial sums are added in a fixed order,
// so acc (B, d) is written once, deterministically, with no atomics.
constexpr int kGenCols = 128;
constexpr int kGenThreads = 256;

template <bool Half>
__global__ void __launch_bounds__(kGenThreads) k_gen_attend(GenArgs a) {
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
  __shared__ float s_att[kMaxTables][32];
  __shared__ int s_pos[kMaxTables][32];
  __shared__ float s_part[4][kGenCols];
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
  for (int tau = wid; tau < T; tau += kGenThreads / 32) {
    const uint16_t id = a.ids_t[b * T + tau];
    const int32_t* slots = a.ring + ((b * T + tau) * ((int64_t)1 << a.nb) + id) * C;
    const int pos = lane < C ? slots[lane] : -1;
    const bool valid = pos >= 0;
    float sc = -INFINITY;
    if (valid) {
      const typename A::T* pk = reinterpret_cast<const typename A::T*>(a.phi_cache) + (b * a.cap + pos) * P;
      const typename A::T* kk = reinterpret_cast<const typename A::T*>(a.kc_cache) + (b * a.cap + pos) * cf;
      float dphi = 0.f, dqk = 0.f;
      for (int p = 0; p < P; ++p) dphi = fmaf(s_q[p], A::load(pk + p), dphi);
      for (int c = 0; c < cf; ++c) dqk = fmaf(s_q[P + c], A::load(kk + c), dqk);
      float t1;
      if (Half) {
        const float s1 = round_bf16(__fdiv_rn(round_bf16(dphi), a.inv_temp_div));
        const float s2 = round_bf16(__fmul_rn(round_bf16(dqk), a.esc_c));
        t1 = round_bf16(__fadd_rn(s1, s2));
      } else {
        t1 = __fadd_rn(__fdiv_rn(dphi, a.inv_temp_div), __fmul_rn(dqk, a.esc_c));
      }
      int ln = 0;
      for (int c = 0; c < K; ++c) {
        const int64_t tq = t - 1 - c, tk = (int64_t)pos - 1 - c;
        if (tq >= 0 && tk >= 0 && sg[tq] == sg[tk]) ++ln; else break;
      }
      t1 = __fadd_rn(t1, a.w_suf[ln]);
      // _atender_cand: nucleo = log_alfa_k - (gamma / C) * float(B_q - B_k), added after the suffix weight
      const float dB = __double2float_rn(Bq - a.bt_cache[b * a.cap + pos]);
      const float nuc = __fsub_rn(a.la_cache[b * a.cap + pos], __fmul_rn(a.tasa[tau], dB));
      sc = __fadd_rn(t1, nuc);
    }
    const bool any = __any_sync(0xffffffffu, valid);
    float att = 0.f;
    if (any) {
      const float mx = warp_max(sc);
      const float e = valid ? expf(__fsub_rn(sc, mx)) : 0.f;
      const float sum = warp_sum(e);
      att = __fdiv_rn(e, sum);
      const float peak = warp_max(att);
      if (lane == 0 && blockIdx.y == 0) {
        a.sen_hay[b * T + tau] = 1;
        a.sen_mx[b * T + tau] = mx;
        a.sen_pk[b * T + tau] = peak;
      }
    } else if (lane == 0 && blockIdx.y == 0) {
      a.sen_hay[b * T + tau] = 0;
      a.sen_mx[b * T + tau] = kProhibido;
      a.sen_pk[b * T + tau] = 0.f;
    }
    s_att[tau][lane] = Half ? round_bf16(att) : att;
    s_pos[tau][lane] = valid ? pos : -1;
  }
  __syncthreads();
  // acc[b, j] = sum over tables and slots of att * E[pos + 1][j], j in this block's columns
  const typename A::T* Ea = reinterpret_cast<const typename A::T*>(a.ea_cache) + b * a.cap * (int64_t)a.d;
  const int g = threadIdx.x / (kGenThreads / 4);              // 4 groups of 64 threads
  const int cl = threadIdx.x % (kGenThreads / 4);             // columns col0 + cl and col0 + cl + 64
  const int j0 = col0 + cl, j1 = col0 + cl + kGenThreads / 4;
  float o0 = 0.f, o1 = 0.f;
  for (int tau = g; tau < T; tau += 4) {
    for (int c = 0; c < C; ++c) {
      const int pos = s_pos[tau][c];
      if (pos < 0) continue;
      const float w = s_att[tau][c];
      const typename A::T* row = Ea + (int64_t)(pos + 1) * a.d;
      if (j0 < a.d) o0 = fmaf(w, A::load(row + j0), o0);
      if (j1 < a.d) o1 = fmaf(w, A::load(row + j1), o1);
    }
  }
  s_part[g][cl] = o0;
  s_part[g][cl + kGenThreads / 4] = o1;
  __syncthreads();
  if (threadIdx.x < kGenCols) {
    const int j = col0 + threadIdx.x;
    if (j < a.d) {
      const float* q = &s_part[0][threadIdx.x];
      a.acc[b * a.d + j] = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[kGenCols]), q[2 * kGenCols]), q[3 * kGenCols]);
    }
  }
}

// n-gram memory of the new token (asrn/nucleo.py:1683-1714) and the streak (asrn/nucleo.py:953-960).
// One thread per sequence: its n orders in turn, then the streak from the longest order.
__global__ void k_gen_hawkes(GenArgs a, HawkesEntry* tab, int64_t hcap, const double* cv, const float* kappa,
                             const double* beta_t, const float* la_t, float* racha_state, uint8_t* vistos,
                             float* hawkes, float* racha_out, int* status) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= a.B) return;
  const int n = a.n;
  const int64_t t = *a.t_pos;
  if (t < 1 || t >= a.cap) {
    if (b == 0) atomicCAS(status, ASRN_OK, ASRN_ERR_ARG);
    return;
  }
  // append the new token's clock (the inclusive fp64 sum, one more term) and log_alfa
  const double Bq = a.bt_w[b * a.cap + t - 1] + beta_t[b];
  a.bt_w[b * a.cap + t] = Bq;
  a.la_w[b * a.cap + t] = la_t[b];
  const float alpha = expf(la_t[b]);
  float r = 0.f;
  for (int ni = 0; ni < n; ++ni) {
    const double key = ngram_key(a.sig_cache + b * a.cap, t, ni, cv);
    float lam = 0.f;
    bool seen = false;
    if (key == key) {
      bool found;
      HawkesEntry* tb = tab + (b * n + ni) * hcap;
      const int64_t i = hawkes_slot(tb, hcap, key_bits(key), &found);
      if (i < 0) {
        atomicCAS(status, ASRN_OK, ASRN_ERR_WORKSPACE);
      } else {
        if (found) {
          const float dB = __double2float_rn(Bq - tb[i].bu);
          lam = __fmul_rn(expf(__fmul_rn(-kappa[ni], dB)), tb[i].a);
          seen = true;
        }
        tb[i].bu = Bq;
        tb[i].a = __fadd_rn(lam, alpha);
      }
    }
    vistos[b * n + ni] = seen ? 1 : 0;
    hawkes[b * n + ni] = lam;
    if (ni == n - 1) r = seen ? 1.f : 0.f;
  }
  const float kr = kappa[n];
  const float e = expf(__fmul_rn(-kr, (float)beta_t[b]));
  const float s = __fmul_rn(r, __fadd_rn(__fmul_rn(e, racha_state[b]), 1.f));
  racha_out[b] = s;
  racha_state[b] = s;
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

int launch_gen_attend(const GenArgs& a, bool half, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  if (a.C > 32 || a.P > kMaxPhi || a.cf > kMaxConfirm || a.T > kMaxTables) return ASRN_ERR_UNSUPPORTED;
  dim3 grid((unsigned)a.B, (unsigned)((a.d + kGenCols - 1) / kGenCols));
  if (half) k_gen_attend<true><<<grid, kGenThreads, 0, s>>>(a);
  else k_gen_attend<false><<<grid, kGenThreads, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? ASRN_OK : ASRN_ERR_CUDA;
}

int launch_gen_memory(const GenArgs& a, void* table, int64_t hcap, const double* cv, const float* kappa,
                      const double* beta_t, const float* la_t, float* racha_state, uint8_t* vistos, float* hawkes,
                      float* racha, int* status, cudaStream_t s) {
  if (a.B == 0) return ASRN_OK;
  if (hcap <= 0 || (hcap & (hcap - 1)) != 0) return ASRN_ERR_ARG;
  k_gen_hawkes<<<(unsigned)((a.B + 63) / 64), 64, 0, s>>>(a, reinterpret_cast<HawkesEntry*>(table), hcap, cv, kappa,
                                                          beta_t, la_t, racha_state, vistos, hawkes, racha, status);
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
