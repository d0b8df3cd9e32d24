// Kernel argument structs and the byte layout of the prepared-weights and workspace buffers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/asrn_b200.h"

namespace asrn {

inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }

// Derived weights, computed on the device by asrn_layer_prepare. "act" = bf16 when half, fp32 otherwise.
struct PreparedLayout {
  size_t wctx;    // (2cf, d) act: [cq; ck]
  size_t w1;      // (3m, d) act: [pal0; ctx0[:, :d]; ctx0[:, d:]]
  size_t b1;      // (2m) f32: pal0.bias, ctx0.bias (bf16-rounded when half: autocast rounds biases)
  size_t w2;      // (P, m) act: [pal2; ctx2]
  size_t b2;      // (P) f32 (rounded when half)
  size_t wov;     // (d, d) act: W_o @ W_v
  size_t gconf;   // (8) f32: g_conf weight (4), bias, (rounded when half)
  size_t tasa;    // (T) f32: gamma / C
  size_t kappa;   // (n + 1) f32: exp(log_kappa) (n), exp(log_kappa_racha), floored by kappa_min
  size_t u_racha; // (nodes) f32: cumsum(d_racha)
  size_t w2bd;    // (Np, 2m) bf16: block-diagonal [pal2 | 0 ; 0 | ctx2], Np = P rounded up to 16 (tensor-core path)
  size_t status;  // int: device status word (ASRN_OK or the first error a kernel recorded)
  size_t total;
};

inline PreparedLayout prepared_layout(const asrn_layer_config& c) {
  const size_t es = c.half ? 2 : 4;
  const size_t d = (size_t)c.d, m = (size_t)c.hidden, cf = (size_t)c.confirmar;
  const size_t P = (size_t)c.n_tablas * c.n_bits;
  PreparedLayout p;
  size_t o = 0;
  p.wctx = o; o = align_up(o + 2 * cf * d * es);
  p.w1 = o; o = align_up(o + 3 * m * d * es);
  p.b1 = o; o = align_up(o + 2 * m * 4);
  p.w2 = o; o = align_up(o + P * m * es);
  p.b2 = o; o = align_up(o + P * 4);
  p.wov = o; o = align_up(o + d * d * es);
  p.gconf = o; o = align_up(o + 8 * 4);
  p.tasa = o; o = align_up(o + (size_t)c.n_tablas * 4);
  p.kappa = o; o = align_up(o + ((size_t)c.vistos + 1) * 4);
  p.u_racha = o; o = align_up(o + (size_t)c.nodos_racha * 4);
  p.w2bd = o; o = align_up(o + ((P + 15) / 16 * 16) * 2 * m * 2);
  p.status = o; o = align_up(o + 4);
  p.total = o;
  return p;
}

struct ContextArgs {
  int64_t B, L;
  int d, cf;
  const float* h;
  const float* E;         // only for signatures without token ids
  const int64_t* tokens;  // may be null
  const float *ln_w, *ln_b, *w_reloj, *b_reloj, *g_w, *g_b, *r_firma;
  const void* wctx;       // act (2cf, d)
  float beta_max, log_alfa_min;
  void *Qc, *Kc;
  double* beta;
  float *log_alfa, *glogit, *sig;
  int* status;            // device status word
};

struct HashArgs {
  int64_t B, L;
  int d, m, T, Tw, nb, P;
  const float* E;
  void* Ea;                // act copy of E (written when half)
  const void* w1;          // act (3m, d)
  const float* b1;         // (2m)
  const void* w2;          // act (P, m)
  const float* b2;         // (P)
  const void* w2bd;        // bf16 (Np, 2m) block-diagonal second layer (tensor-core path)
  void* phi;               // act (B, L, P)
  uint16_t* ids_rows;      // (B*T, L)
  int* status;             // device status word
};

struct ScoreArgs {
  int64_t B, L;            // sorted rows (B*T, L)
  int64_t Lf;              // per-position features and the value rows: (B, Lf, ...), indexed by text position
  int64_t q_lo, q_hi;      // slots whose position is in [q_lo, q_hi) are queries; outputs (B, q_hi - q_lo, ...)
  const int64_t* row_len;  // (B*T) slots in use at the start of each sorted row (the rest padding), or null: all L
  int d, T, nb, P, C, cf, K;
  float inv_temp_div;      // temperature (scores are divided by it)
  float esc_c;             // cf^-1/2
  const int32_t* orden;
  const uint16_t* ids_o;
  const void *phi, *Qc, *Kc, *Ea;
  const float* sig;
  const double* Bt;
  const float* log_alfa;
  const float* w_suf;      // (K + 1)
  const float* tasa;       // (T)
  void* acc;               // (B, q_hi - q_lo, d): bf16 in bf16 mode (added to by bf16 reductions), else fp32
  uint8_t* sen_hay;
  float *sen_mx, *sen_pk;
  int* status;             // device status word (bounded waits of the tensor-core path)
};

struct RepetitionArgs {
  int64_t B, L;            // L: positions of the (chunk of the) rows this call sorts and scans
  int64_t Lf, pos0;        // per-position inputs are (B, Lf) rows; local index i is position pos0 + i (Lf = L, pos0 = 0
                           // for whole rows)
  int n;
  const float* sig;
  const double* c;         // c_vistos (n)
  const double* beta;
  const double* Bt;
  const float* log_alfa;
  const float* kappa;      // (n + 1): the last one is the streak rate
  uint8_t* vistos;
  float *hawkes, *racha;
  double* keys;            // optional
  int32_t* orden_ng;       // optional
  uint8_t* repetido;       // optional
  const float* racha_in;   // optional (B): streak value before the first position (0 when null)
  float* racha_map;        // optional (B, 2): the rows' streak maps S_last = A * S_in + B (A, B)
  // The n-gram sort shared by the layers of a model (whole rows only): ng_mode 1 sorts and writes the sorted keys and
  // positions of every (b, n) row to ng_keys / ng_pos and stops; ng_mode 2 takes them from there instead of sorting.
  int ng_mode;
  uint64_t* ng_keys;       // (B, n, L) order-preserving keys, sorted per row
  uint32_t* ng_pos;        // (B, n, L) their positions
  const int64_t* tok;      // optional: signatures are the token ids (as fp32) instead of sig
};

enum { kNgFull = 0, kNgSortOnly = 1, kNgScanOnly = 2 };

struct GateArgs {
  int64_t B, L;
  int d, T, Tc, n, nodes;
  float mejor_max, tope;
  float racha_paso;
  const float *h, *glogit, *acc;
  const uint8_t* sen_hay;
  const float *sen_mx, *sen_pk;
  const uint8_t* vistos;
  const float *hawkes, *racha;
  const void* wov;         // act (d, d)
  const float* gconf;      // (5)
  const float *w_vistos, *u_hawkes, *u_racha, *d_racha;
  float* out;
  int* status;             // device status word
  const __nv_bfloat16* acc16;   // whole-sequence bf16 mode: the scoring's bf16 accumulator (acc unused)
  __nv_bfloat16* cbuf;     // generation step: (B, d) bf16 GEMM operand bf16(acc / max(1, pt)) (precomputed)
  float* sigma;            // gate values: (M) from k_gate_scalars (tensor-core path) or the generation step
  float* rpt;              // tensor-core path: (M) 1 / max(1, pt) from k_gate_scalars (workspace)
};

// Context + sign-hash projection of one new token per sequence (generation step).
struct GenFrontArgs {
  int64_t B;
  int d, cf, m, T, Tw, nb, P;
  const float* h;          // (B, d)
  const float* e_t;        // (B, d) E of the new token
  const float* e_prev;     // (B, d) E of the previous token
  const int64_t* tokens;   // (B)
  const float *ln_w, *ln_b, *w_reloj, *b_reloj, *g_w, *g_b;
  const void* wctx;        // act (2cf, d)
  const void* w1;          // act (3m, d)
  const float* b1;         // (2m)
  const void* w2;          // act (P, m)
  const float* b2;         // (P)
  float beta_max, log_alfa_min;
  void *Qc, *Kc;           // act (B, cf)
  double* beta;            // (B)
  float *log_alfa, *glogit, *sig;  // (B)
  void* phi;               // act (B, P)
  uint16_t* ids;           // (B, T)
  float* dots;             // optional scratch (B, 2cf + 3 + 3m): the front split over more blocks
  int* status;             // device status word (bounded waits)
  const void* y;           // optional act (B, d): the previous local block's MLP output, added to h first
  float* h_sum;            // with y: (B, d) receives h + y (the gate's residual input)
};

// One generation step of one layer: B sequences, the new token at position t of caches of `cap` positions.
struct GenArgs {
  int64_t B, cap;
  const int64_t* t_pos;      // device: position of the new token
  int d, T, nb, P, C, cf, K, n;
  float inv_temp_div, esc_c;
  int* status;               // device status word
  const uint16_t* ids_t;     // (B, T) bucket ids of the new token
  const void* phi_t;         // (B, P) act
  const void* qc_t;          // (B, cf) act
  const void* kc_t;          // (B, cf) act
  void* phi_cache_w;         // phi_cache, written at t
  void* kc_cache_w;          // kc_cache, written at t
  double* bt_w;              // bt_cache, written at t
  float* la_w;               // la_cache, written at t
  const int32_t* ring;       // (B, T, 2^nb, C)
  const float* sig_cache;    // (B, cap) signatures
  const double* bt_cache;    // (B, cap) clock
  const float* la_cache;     // (B, cap) log alfa
  const void* phi_cache;     // (B, cap, P) act
  const void* kc_cache;      // (B, cap, cf) act
  const void* ea_cache;      // (B, cap, d) act rows of E (the value of position k is row k + 1)
  const float* w_suf;        // (K + 1)
  const float* tasa;         // (T)
  float* acc;                // (B, d), zeroed by the caller
  uint8_t* sen_hay;          // (B, T)
  float *sen_mx, *sen_pk;    // (B, T)
};

int launch_context(const ContextArgs& a, bool half, cudaStream_t s);
int launch_local_in(int64_t B, int d, int k, const float* h_prev, const void* y_prev, float* h_out, const float* ln_w,
                    const float* ln_b, float eps, void* win, bool half, cudaStream_t s);
int launch_local_mid(int64_t B, int d, const float* h, const void* z, float* h1, const float* ln_w, const float* ln_b,
                     float eps, void* v_out, bool half, cudaStream_t s);
int launch_local_gelu(int64_t n, void* f, bool half, cudaStream_t s);
int launch_shard_rows(int64_t rows, int64_t L, int C, int64_t q_lo, int64_t q_hi, const int32_t* orden,
                      const uint16_t* ids_o, int64_t Lv, int32_t* orden_v, uint16_t* ids_v, int64_t* counts,
                      int32_t pad_pos, cudaStream_t s);
size_t shard_merge_workspace(int64_t rows, int nb);
int launch_shard_tails(int64_t rows, int64_t Lc, int nb, int C, int64_t c0, const int32_t* orden_loc,
                       const uint16_t* ids_loc, int32_t* tails, void* ws, cudaStream_t s);
int launch_shard_merge(int64_t rows, int64_t Lc, int nb, int C, int64_t c0, int n_prev, const int32_t* tails_prev,
                       const int32_t* orden_loc, const uint16_t* ids_loc, int64_t Lv, int32_t* orden_v,
                       uint16_t* ids_v, int64_t* row_len, int32_t pad_pos, int* status, void* ws, cudaStream_t s);
size_t ngram_chunk_workspace(int64_t B, int64_t Lc, int n);
int launch_ngram_chunk_sort(const RepetitionArgs& a, uint64_t* keys, void* summary, void* ws, size_t ws_bytes,
                            cudaStream_t s);
int launch_ngram_chunk_finish(const RepetitionArgs& a, int n_prev, const uint64_t* keys_prev, const void* summary_prev,
                              const uint64_t* keys, void* ws, size_t ws_bytes, cudaStream_t s);
int launch_racha(const RepetitionArgs& a, cudaStream_t s);
size_t racha_workspace(int64_t B, int64_t L);
int launch_racha_ws(const RepetitionArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);
int launch_gen_front(const GenFrontArgs& a, bool half, cudaStream_t s);
int launch_gen_gate(const GateArgs& a, bool half, cudaStream_t s);
size_t hawkes_table_bytes(int64_t B, int n, int64_t cap);
int launch_ring_build(int64_t B, int64_t L, int T, int nb, int C, int64_t n_valid, const int32_t* orden,
                      const uint16_t* ids_o, int32_t* ring, int32_t* count, cudaStream_t s);
int launch_hawkes_build(int64_t B, int64_t L, int64_t ld, int n, const float* sig, const double* cv, const double* Bt,
                        const float* la, const float* hawkes, void* table, int64_t cap, int* status, cudaStream_t s);
int launch_gen_attend(const GenArgs& a, const GateArgs& ga, bool half, cudaStream_t s);
int launch_gen_memory(const GenArgs& a, void* table, int64_t hcap, const double* cv, const float* kappa,
                      const double* beta_t, const float* la_t, float* racha_state, uint8_t* vistos, float* hawkes,
                      float* racha, int* status, cudaStream_t s);
int launch_ring_insert(int64_t B, int T, int nb, int C, const int64_t* t_pos, const uint16_t* ids_t, int32_t* ring,
                       int32_t* count, cudaStream_t s);
int launch_clock(const double* beta, double* Bt, int64_t B, int64_t L, cudaStream_t s);
int launch_hash(const HashArgs& a, bool half, cudaStream_t s);
int launch_ids_from_phi(int64_t B, int64_t L, int T, int nb, const float* phi, uint16_t* ids_rows, cudaStream_t s);
size_t bucket_sort_workspace(int64_t rows, int64_t L, int nb);
int launch_bucket_sort(int64_t rows, int64_t L, int nb, const uint16_t* ids_rows, int32_t* orden, uint16_t* ids_o,
                       void* ws, size_t ws_bytes, cudaStream_t s);
int launch_bucket_sort_noalloc(int64_t rows, int64_t L, int nb, const uint16_t* ids_rows, int32_t* orden,
                               uint16_t* ids_o, cudaStream_t s);
int launch_score(const ScoreArgs& a, bool half, cudaStream_t s);
int launch_candidates(int64_t B, int64_t L, int T, int C, int K, const int32_t* orden, const uint16_t* ids_o,
                      const float* sig, int32_t* cand, uint8_t* suffix, cudaStream_t s);
size_t repetition_workspace(int64_t B, int64_t L, int n);
int launch_repetition(const RepetitionArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);
size_t ngram_shared_bytes(int64_t B, int64_t L, int n);
int launch_gate(const GateArgs& a, bool half, cudaStream_t s);
size_t gate_workspace(int64_t M, int d, bool half);
int launch_prepare(const asrn_layer_config& c, const asrn_layer_weights& w, void* prepared, cudaStream_t s);
// 2-D bf16 TMA tensor map, 128-byte swizzle: rows of `inner` elements (row stride in bytes), box inner x outer.
bool make_tmap_f32(void* map /* CUtensorMap */, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                   uint32_t box_inner, uint32_t box_outer);
// The same with the 128-byte shared-memory swizzle (box_inner = 32 fp32).
bool make_tmap_f32_sw128(void* map /* CUtensorMap */, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);
// 3-D maps over row-major (d2, d1, d0) tensors (innermost d0), boxes box0 x box1 x 1, 128-byte swizzle; a box reaching
// outside [0, d1) of its sequence reads zeros there.
bool make_tmap_bf16_3d(void* map /* CUtensorMap */, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                       uint32_t box0, uint32_t box1);
bool make_tmap_f32_3d_sw128(void* map /* CUtensorMap */, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                            uint32_t box0, uint32_t box1);
// Rows of a bf16 matrix for row gathers: box = one row of box_inner elements, swizzle of `swizzle_bytes` (0, 32, 64
// or 128; with a swizzle, box_inner * 2 equals it).
bool make_tmap_rows_bf16(void* map /* CUtensorMap */, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t row_bytes, uint32_t box_inner, int swizzle_bytes);
bool make_tmap_bf16(void* map /* CUtensorMap */, const void* base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);
// GEMM implementation choice: false while the test hook asrn_test_force_cuda_core holds the CUDA-core kernels.
bool tensor_cores_enabled();
int set_force_cuda_core(int on);

}  // namespace asrn
