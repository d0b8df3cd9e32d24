/*
 * asrn_b200.h -- C ABI of libasrn_b200.so: the ASRN layer forward and its O(1) generation step on B200 (sm_100a).
 *
 * Conventions
 *   - Every entry point takes plain device pointers, sizes and a CUDA stream (passed as void*, a cudaStream_t).
 *     The caller allocates every buffer; entry points never allocate, free or synchronise, and are stream-ordered.
 *   - Return value: ASRN_OK (0) or an ASRN_ERR_* status; asrn_status_string() names it. No exception crosses the ABI.
 *   - "act" buffers hold activations in the layer's compute type: bfloat16 when cfg->half (the reference under
 *     torch.autocast(dtype=bfloat16)), float32 otherwise.
 *   - Layouts are row-major: (B, L, d) means index (b * L + t) * d + j. A "row" of a per-table tensor is r = b * T + tau.
 *
 * Reference interfaces replaced (KIROKOWA/ASRN, paths inside that project):
 *   asrn_layer_forward      CapaASRNEstable.forward            asrn/estable.py:407-421
 *   asrn_context            CapaASRNEstable._contexto          asrn/estable.py:153-194 (+ firmas_de_piezas,
 *                                                              asrn/nucleo.py:161-164, and _firma, :634-637)
 *   asrn_clock              Bt = beta.cumsum(1)                asrn/estable.py:418
 *   asrn_hash               CapaASRN._phi_y_valores + _ids     asrn/nucleo.py:644-664
 *   asrn_ids_from_phi       CapaASRN._ids                      asrn/nucleo.py:661-664
 *   asrn_bucket_sort        ids.argsort(dim=-1, stable=True)   asrn/estable.py:220-221
 *   asrn_candidates         the candidate window + _largo_seguido asrn/estable.py:232-265, asrn/nucleo.py:98-108
 *   asrn_score              _acumular after the projection     asrn/estable.py:204-300 (the seam the reference
 *                           (_CasillerosTriton.apply)          fills with asrn/nucleo.py:461-488)
 *   asrn_repetition         CapaASRNEstable._repeticion        asrn/estable.py:304-321 (+ _claves_vistos,
 *                                                              _ordenar_claves, escaneo: asrn/nucleo.py:175-257,
 *                                                              688-701)
 *   asrn_gate               CapaASRNEstable._combinar          asrn/estable.py:376-403
 *   asrn_gen_ring_build     _anillo_desde                      asrn/nucleo.py:1585-1607
 *   asrn_gen_hawkes_build   _MemoriaHawkes.cargar              asrn/nucleo.py:1656-1681
 *   asrn_gen_attend         _candidatos + _atender_cand        asrn/nucleo.py:1621-1631, asrn/estable.py:359-372
 *   asrn_gen_memory         _MemoriaHawkes.paso + _repeticion_o1  asrn/nucleo.py:1683-1714, 953-960
 *   asrn_gen_ring_insert    _anillo_meter                      asrn/nucleo.py:1610-1618
 *   asrn_gen_front          _contexto + _phi_y_valores/_ids (one token)  asrn/estable.py:153-194, nucleo.py:639-664
 *   asrn_shard_tails, asrn_shard_merge, asrn_shard_rows, asrn_score_shard
 *                                        candidate windows / _acumular of one shard of a long sequence
 *                                        (asrn/estable.py:220-300; the reference runs one GPU per sequence)
 *   asrn_gen_gate           _combinar (one token)              asrn/estable.py:376-403
 */
#ifndef ASRN_B200_H
#define ASRN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ASRN_OK = 0,
  ASRN_ERR_ARG = 1,          /* bad shape, null pointer or option out of range */
  ASRN_ERR_UNSUPPORTED = 2,  /* option combination this build does not implement */
  ASRN_ERR_WORKSPACE = 3,    /* workspace / prepared buffer too small or misaligned */
  ASRN_ERR_CUDA = 4,         /* a kernel launch failed (cudaGetLastError) */
  ASRN_ERR_TIMEOUT = 5,      /* a bounded device wait gave up */
  ASRN_ERR_DATA = 6          /* state received from another shard failed validation (recorded in a status word) */
};

/* Layer options (asrn/nucleo.py:585-630) and protections (asrn/estable.py:57-77). */
typedef struct asrn_layer_config {
  int64_t B, L, d;           /* batch, length, width */
  int32_t n_tablas;          /* T, <= 16 */
  int32_t n_bits;            /* bits per table, <= 16 */
  int32_t chunk;             /* C: candidates per table and query, <= 32 */
  int32_t tablas_contexto;   /* context tables (the last ones) */
  int32_t confirmar;         /* cf, <= 32 */
  int32_t sufijo;            /* K, <= 8 */
  int32_t vistos;            /* n-gram orders 1..n, <= 8 */
  int32_t nodos_racha;       /* streak response nodes */
  int32_t hidden;            /* max(8, afin_oculto // 2), <= 128 */
  int32_t half;              /* 1: bfloat16 autocast semantics, 0: float32 */
  float beta_max;            /* +inf: no cap */
  float log_alfa_min;        /* -inf: no floor */
  float mejor_max;           /* +inf: no clamp */
  float tope_puerta;         /* 0: no gate cap */
  float kappa_min;           /* 0: no floor */
  double racha_paso;         /* log1p(racha_max) / (nodos_racha - 1) */
} asrn_layer_config;

/* The layer's parameters as stored by the reference (state_dict names in comments), float32 device pointers. */
typedef struct asrn_layer_weights {
  const float *ln_w, *ln_b;            /* ln_ctx.weight, ln_ctx.bias (d) */
  const float *cq, *ck;                /* cq.weight, ck.weight (cf, d) */
  const float *w_reloj, *b_reloj;      /* w_reloj (2, d), b_reloj (2) */
  const float *pal0_w, *pal0_b;        /* afin_palabra.0.weight (m, d), .bias (m) */
  const float *pal2_w, *pal2_b;        /* afin_palabra.2.weight ((T - Tc) * nb, m), .bias */
  const float *ctx0_w, *ctx0_b;        /* afin_contexto.0.weight (m, 2d), .bias (m) */
  const float *ctx2_w, *ctx2_b;        /* afin_contexto.2.weight (Tc * nb, m), .bias */
  const float *v_w, *o_w;              /* v.weight, o.weight (d, d) */
  const float *g_w, *g_b;              /* g.weight (1, d), g.bias (1) */
  const float *g_conf_w, *g_conf_b;    /* g_conf.weight (1, 4), g_conf.bias (1) */
  const float *w_vistos, *u_hawkes;    /* (n) */
  const float *log_kappa;              /* (n) */
  const float *log_kappa_racha;        /* (1) */
  const float *w_sufijo;               /* (K + 1) */
  const float *gamma;                  /* (T) */
  const float *d_racha;                /* (nodos_racha) */
  const double *c_vistos;              /* buffer c_vistos (n), float64 */
  const float *r_firma;                /* buffer r_firma (d): signatures when no token ids are given */
} asrn_layer_weights;

const char* asrn_status_string(int status);
int asrn_abi_version(void);

/* ---- whole layer ------------------------------------------------------------------------------------------------ */

/* Derived weights (concatenated / rounded projections, W_o @ W_v, decay rates) for a config, computed on the device.
 * Recompute after the parameters change. */
size_t asrn_layer_prepared_bytes(const asrn_layer_config* cfg);
int asrn_layer_prepare(const asrn_layer_config* cfg, const asrn_layer_weights* w, void* prepared, size_t bytes,
                       void* stream);

/* The device status word kept in the prepared buffer: ASRN_OK, or the first error a kernel recorded (for example
 * ASRN_ERR_TIMEOUT from a bounded wait). Synchronises `stream`; reset != 0 clears the word. Returns the status
 * (>= 0), or -ASRN_ERR_* if it could not be read. */
int asrn_layer_status(const asrn_layer_config* cfg, const void* prepared, int reset, void* stream);

size_t asrn_layer_workspace_bytes(const asrn_layer_config* cfg);
/* h_out = layer(E, h, tokens). E, h, h_out: (B, L, d) float32. tokens: (B, L) int64 token ids, or NULL to use the
 * reference's vector signature E . r_firma. h_out may not alias E or h. */
int asrn_layer_forward(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                       const float* E, const float* h, const int64_t* tokens, float* h_out, void* workspace,
                       size_t workspace_bytes, void* stream);

/* The n-gram sort shared by the ASRN layers of a model (the reference sorts the same keys in every layer: its
 * repetition memory depends only on the tokens and on c_vistos, a buffer drawn from a fixed seed and equal in every
 * layer; asrn/nucleo.py:610, :691-701, asrn/estable.py:304-321). asrn_ngram_shared_sort sorts the (B, n) rows of
 * n-gram keys of `tokens` once (workspace: asrn_repetition_workspace_bytes); asrn_layer_forward_ngram is
 * asrn_layer_forward with that sort given (same tokens, same vistos and c_vistos): it runs only the scans. The
 * results equal asrn_layer_forward's bit for bit. */
size_t asrn_ngram_shared_bytes(const asrn_layer_config* cfg);
int asrn_ngram_shared_sort(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                           const int64_t* tokens, void* ngram, size_t ngram_bytes, void* workspace,
                           size_t workspace_bytes, void* stream);
int asrn_layer_forward_ngram(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                             const float* E, const float* h, const int64_t* tokens, const void* ngram,
                             size_t ngram_bytes, float* h_out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- stages (each one seam of the reference; the layer forward runs them in this order) -------------------------- */

/* LN(h) -> Qc, Kc (act, (B, L, cf)), beta (float64), log_alfa (float32); glogit = g(h) (float32); sig (float32). */
int asrn_context(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                 const float* E, const int64_t* tokens, void* Qc, void* Kc, double* beta, float* log_alfa,
                 float* glogit, float* sig, void* stream);

/* Bt = inclusive prefix sum of beta along L, float64, per batch row. */
int asrn_clock(int64_t B, int64_t L, const double* beta, double* Bt, void* stream);

/* E -> Ea (act copy of E, (B, L, d); may equal E when !half), phi (act, (B, L, T * nb)) and the bucket ids per
 * table row, ids_rows (B * T, L) uint16. */
int asrn_hash(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* E,
              void* Ea, void* phi, uint16_t* ids_rows, void* stream);

/* Sign-pack only: phi (B, L, T * nb) float32 -> ids_rows (B * T, L) uint16, bit j = (phi[tau * nb + j] > 0). */
int asrn_ids_from_phi(int64_t B, int64_t L, int32_t T, int32_t nb, const float* phi, uint16_t* ids_rows,
                      void* stream);

/* Stable sort of every row of ids_rows by bucket id (ties by position): orden[r][s] = text position of sorted slot
 * s, ids_o[r][s] = its bucket id. */
size_t asrn_bucket_sort_workspace_bytes(int64_t rows, int64_t L, int32_t nb);
int asrn_bucket_sort(int64_t rows, int64_t L, int32_t nb, const uint16_t* ids_rows, int32_t* orden,
                     uint16_t* ids_o, void* workspace, size_t workspace_bytes, void* stream);

/* Candidate scoring of every (row, sorted slot) against its <= C bucket mates, exact-mask softmax, copy of the next
 * token's value row: acc (B, L, d) += sum over tables and candidates of att * Ea[k + 1] (acc must be zeroed by the
 * caller; apply W_v to acc to get the reference's `salida`). acc is in the compute type: under bfloat16 autocast a
 * bf16 accumulator that the tables add into with bf16 reductions in L2 (the reference's per-table outputs are bf16 as
 * well; the order of the additions is not fixed, so results vary run to run by a few bf16 roundings: about 5e-3 of
 * max|h' - h| at the benchmark shapes), fp32 otherwise (within fp32 rounding). Per-table gate signals in text order,
 * (B, L, T): hay (uint8), mx (float32, -1e9 when no candidate), pk (float32). */
int asrn_score(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
               const int32_t* orden, const uint16_t* ids_o, const void* phi, const void* Qc, const void* Kc,
               const float* sig, const double* Bt, const float* log_alfa, const void* Ea, void* acc,
               uint8_t* sen_hay, float* sen_mx, float* sen_pk, void* stream);

/* ---- local blocks of the model, one generation step (B rows; half: bf16 compute type, else fp32) ---------------
 * The element-wise parts of BloqueLocal (asrn/nucleo.py:969-1014) around its three GEMMs, with the writer's conv
 * buffer (asrn/nucleo.py:1816-1822): asrn_local_in: h = h_prev (+ y_prev, compute type, the previous block's MLP
 * output; may be NULL) -> h_out (may be NULL), LN1(h) rounded to the compute type pushed into the conv window
 * win (B, k, d) (rows shift down in place; 1 <= k <= 16; k = 1 gives a plain LN into win); asrn_local_mid: h1 = h + act(gelu(z))
 * and v_out = act(LN2(h1)); asrn_local_gelu: f = act(gelu(f)) in place (n values). d <= 1024. */
int asrn_local_in(int64_t B, int32_t d, int32_t k, const float* h_prev, const void* y_prev, float* h_out,
                  const float* ln_w, const float* ln_b, float eps, void* win, int32_t half, void* stream);
int asrn_local_mid(int64_t B, int32_t d, const float* h, const void* z, float* h1, const float* ln_w,
                   const float* ln_b, float eps, void* v_out, int32_t half, void* stream);
int asrn_local_gelu(int64_t n, void* f, int32_t half, void* stream);

/* ---- local block of the model over whole sequences, bfloat16 autocast (BloqueLocal.forward, asrn/nucleo.py:969-1014,
 * mezcla='conv') -------------------------------------------------------------------------------------------------------
 * h_out = h1 + bf16(W2 gelu(bf16(W1 LN2(h1) + b1)) + b2), h1 = h + gelu(bf16(bf16(conv_k(pad(LN1(h)))) + b_conv)),
 * with autocast's bf16 operands and roundings. h, h_out: (B, L, d) fp32 (h_out may not alias h). w_conv: bf16
 * (d, k * d), element [o][j * d + c] = conv.weight[o][c][j] (tap j reads position t - (k - 1) + j); w1: bf16 (ff, d);
 * w2: bf16 (d, ff); LayerNorm weights and biases fp32 (biases are rounded to bf16 as autocast does). d a multiple of
 * 128 and at most 1024, ff a multiple of 128 (else ASRN_ERR_UNSUPPORTED). status: device int for the bounded waits
 * (may be null). Workspace: asrn_local_block_workspace_bytes. */
size_t asrn_local_block_workspace_bytes(int64_t B, int64_t L, int32_t d, int32_t ff);
int asrn_local_block(int64_t B, int64_t L, int32_t d, int32_t k, int32_t ff, const float* h, float* h_out,
                     const float* ln1_w, const float* ln1_b, float eps1, const void* w_conv, const float* b_conv,
                     const float* ln2_w, const float* ln2_b, float eps2, const void* w1, const float* b1,
                     const void* w2, const float* b2, void* workspace, size_t workspace_bytes, int* status,
                     void* stream);

/* ---- training: bucket attention and scan, forward and backward ---------------------------------------------------
 * The kernels the reference's training path calls (asrn/nucleo.py:461-537; asrn/estable.py:282-291 in its exact-mask,
 * 64-bit-clock mode), for one table set: phi (B, L, P), Qc / Kc (B, L, CF), V (B, L, D) all fp32 (half = 0) or all
 * bf16 (half = 1); Pf (B, L, K) the K previous signatures (NaN before the start); the clock as fp32 high and low
 * parts Bt_hi, Bt_lo (B, L); log_alfa (B, L); orden / ids_o (B T, L) int32, the positions of each row sorted by
 * bucket and their bucket ids; w_suf (K + 1), gamma (T) fp32. C <= 32, P <= 256, CF <= 32, K <= 8.
 * asrn_bucket_attn_forward: out (B T, L, D) in V's type, per table row in text order (the caller sums the T tables);
 * sen (B T, L, 3) = (any valid key, max valid score or 0, max weight).
 * asrn_bucket_attn_backward: from dout (B, L, D) in V's type, with the scores recomputed, the per-slot gradient
 * buffers of asrn/nucleo.py:491-515 (no atomics): g_phi_q (B T, L, P), g_qc (B T, L, CF), g_b_q (B T, L) fp32;
 * g_phi_k (2, B T, L, P), g_kc (2, B T, L, CF), g_v (2, B T, L, D), g_la (2, B T, L), g_b_k (2, B T, L) fp32 (place
 * 1: the key in its own block, place 0: in the next block's window); partes (B T, ceil(L / C), K + 2) fp32 = per
 * program (sum dS dt, then sum dS per suffix length 0 .. K). Gradient types follow their inputs'. */
int asrn_bucket_attn_forward(int64_t B, int64_t L, int32_t T, int32_t C, int32_t P, int32_t CF, int32_t K, int32_t D,
                             const void* phi, const void* Qc, const void* Kc, const void* V, const float* Pf,
                             const float* Bt_hi, const float* Bt_lo, const float* log_alfa, const int32_t* orden,
                             const int32_t* ids_o, const float* w_suf, const float* gamma, float scale_phi,
                             float scale_c, int32_t half, void* out, float* sen, void* stream);
int asrn_bucket_attn_backward(int64_t B, int64_t L, int32_t T, int32_t C, int32_t P, int32_t CF, int32_t K, int32_t D,
                              const void* phi, const void* Qc, const void* Kc, const void* V, const float* Pf,
                              const float* Bt_hi, const float* Bt_lo, const float* log_alfa, const int32_t* orden,
                              const int32_t* ids_o, const float* w_suf, const float* gamma, float scale_phi,
                              float scale_c, int32_t half, const void* dout, void* g_phi_q, void* g_qc, float* g_b_q,
                              void* g_phi_k, void* g_kc, void* g_v, float* g_la, float* g_b_k, float* partes,
                              void* stream);
/* S_i = a_i S_{i-1} + b_i along each of `rows` rows of L fp32 values (asrn/nucleo.py:188-197), and its backward from
 * g = dL/dS: ga = dL/da, gb = dL/db (either may be NULL) (asrn/nucleo.py:518-537). */
int asrn_scan_forward(int64_t rows, int64_t L, const float* a, const float* b, float* S, void* stream);
int asrn_scan_backward(int64_t rows, int64_t L, const float* a, const float* S, const float* g, float* ga, float* gb,
                       void* stream);

/* ---- sequence-chunk sharding (one long sequence over several GPUs) --------------------------------------------------
 * Shard r of `world` owns positions [c0, c0 + Lc) of every sequence (L = world * Lc). Its sorted rows hold its own
 * slots and, before each bucket's local run, the up to C earlier-chunk slots some local query has as a candidate (the
 * bucket's C most recent earlier positions): the candidates of every local query are then the same as in the full
 * row (asrn/estable.py:220-236, 262-265). Rows are padded with id 0xFFFF, so nb <= 15 here.
 *
 * asrn_shard_tails: from the shard's own sorted chunk (orden_loc, ids_loc: (rows, Lc) from asrn_bucket_sort on the
 * chunk's bucket ids, local positions), per (row, bucket) the bucket's last <= C global positions: tails
 * (rows, 2^nb, C + 1) int32, [0] = count, [1 .. count] ascending. Every shard publishes its tails (all-gather).
 * asrn_shard_merge: the shard's rows from its sorted chunk and the tails of the n_prev = r earlier shards
 * (tails_prev: (n_prev, rows, 2^nb, C + 1), rank order): orden_v / ids_v (rows, Lv), the used length of each row in
 * row_len (rows) int64 (the rest is padding); Lv >= Lc + min(c0, 2^nb * C) bounds every row, so no host round trip
 * is needed. Requires 2+ shards (c0 > 0 or c0 + Lc < L). Both take a workspace of asrn_shard_workspace_bytes.
 * A received tail is used only if its count is in [0, C] and its positions ascend strictly inside its sender's chunk
 * [p Lc, (p + 1) Lc); any other tail is treated as empty and ASRN_ERR_DATA is recorded in *status (a device int, may
 * be NULL), so corrupt state never indexes features out of range.
 * asrn_shard_rows: the same rows from the FULL sorted rows (orden, ids_o: (rows, L) after exchanging all bucket ids);
 * with orden_v == NULL it only writes each row's length to counts (rows) int64; otherwise it writes rows of length Lv
 * (cut at Lv), padded with id 0xFFFF, and the lengths too when counts != NULL. q_lo = c0, q_hi = c0 + Lc.
 * asrn_score_shard is asrn_score over such rows (cfg->L = Lv) with features of L_feat positions per sequence indexed
 * by position, queries = the slots at positions [q_lo, q_hi), outputs (B, q_hi - q_lo, ...); row_len (B*T) int64 or
 * NULL bounds the slots scored in each row (spans past it do no work). */
size_t asrn_shard_workspace_bytes(int64_t rows, int32_t nb);
int asrn_shard_tails(int64_t rows, int64_t Lc, int32_t nb, int32_t C, int64_t c0, const int32_t* orden_loc,
                     const uint16_t* ids_loc, int32_t* tails, void* workspace, size_t workspace_bytes, void* stream);
int asrn_shard_merge(int64_t rows, int64_t Lc, int32_t nb, int32_t C, int64_t c0, int32_t n_prev,
                     const int32_t* tails_prev, const int32_t* orden_loc, const uint16_t* ids_loc, int64_t Lv,
                     int32_t* orden_v, uint16_t* ids_v, int64_t* row_len, int64_t L, void* workspace,
                     size_t workspace_bytes, int* status, void* stream);
int asrn_shard_rows(int64_t rows, int64_t L, int32_t C, int64_t q_lo, int64_t q_hi, const int32_t* orden,
                    const uint16_t* ids_o, int64_t Lv, int32_t* orden_v, uint16_t* ids_v, int64_t* counts,
                    void* stream);
int asrn_score_shard(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, int64_t L_feat,
                     int64_t q_lo, int64_t q_hi, const int32_t* orden, const uint16_t* ids_o, const void* phi,
                     const void* Qc, const void* Kc, const float* sig, const double* Bt, const float* log_alfa,
                     const void* Ea, const int64_t* row_len, void* acc, uint8_t* sen_hay, float* sen_mx,
                     float* sen_pk, void* stream);

/* n-gram memory of one shard's chunk [c0, c0 + cfg->L) of sequences of L_feat positions (asrn/estable.py:304-321
 * carried across chunks; the reference runs whole sequences). sig, Bt, log_alfa: the gathered (B, L_feat) rows.
 * asrn_ngram_chunk_sort: sorts the chunk's (key, position) pairs per (b, order) row and scans them with the chunk
 * alone; writes the sorted keys (B*n, Lc) uint64 (order-preserving images of the fp64 keys) and per group a 32-byte
 * summary (B*n, Lc) at the group's first slot: {fp64 clock of its first and last occurrence, fp32 intensity and
 * decay product at its last slot, fp32 alfa of its last occurrence}. Every shard publishes both (all-gather).
 * asrn_ngram_chunk_finish: with the n_prev = r earlier shards' keys and summaries ((n_prev, B*n, Lc), rank order)
 * and the state the sort left in the workspace (same workspace), vistos (B, Lc, n) uint8 and hawkes (B, Lc, n)
 * float32 of the chunk, equal to the whole-sequence values at its positions.
 * asrn_racha_chunk: the streak of a chunk (cfg->L positions, vistos / beta of the chunk) from the value before it
 * (racha_in (B), NULL = 0) into racha (B, Lc) (may be NULL); racha_map (B, 2) (may be NULL) receives the chunk's map
 * S_last = A * S_before + B0 as (A, B0), from which the next shards' racha_in follow. With a workspace of
 * asrn_racha_workspace_bytes (may be NULL: one block per sequence) few long rows are scanned over all SMs. */
size_t asrn_ngram_chunk_workspace_bytes(const asrn_layer_config* cfg);
int asrn_ngram_chunk_sort(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                          int64_t L_feat, int64_t c0, const float* sig, const double* Bt, const float* log_alfa,
                          uint64_t* keys, void* summary, void* workspace, size_t workspace_bytes, void* stream);
int asrn_ngram_chunk_finish(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                            int64_t L_feat, int64_t c0, int32_t n_prev, const uint64_t* keys_prev,
                            const void* summary_prev, const uint64_t* keys, const double* Bt, const float* log_alfa,
                            uint8_t* vistos, float* hawkes, void* workspace, size_t workspace_bytes, void* stream);
size_t asrn_racha_workspace_bytes(const asrn_layer_config* cfg);
int asrn_racha_chunk(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                     const uint8_t* vistos, const double* beta, const float* racha_in, float* racha, float* racha_map,
                     void* workspace, size_t workspace_bytes, void* stream);

/* The same bucket sort for callers that cannot allocate device memory when they sort (a plug-in inside a host process
 * whose allocator it does not own, a serving loop that keeps a fixed memory footprint after start-up): no workspace
 * argument; rows longer than one tile (8192 positions) use a fixed 32 MiB scratch array inside this library, which
 * every GPU that loads the library keeps until the process exits. Requests whose scratch would exceed 32 MiB
 * (rows * L * 4 + rows * ceil(L / 8192) * 2^nb * 4 bytes, each rounded up to 256) return ASRN_ERR_WORKSPACE.
 * Every call looks up the array's device address in the current context (a host-side query, no stream work), so the
 * entry point stays valid after the context is destroyed and created again. Calls share the array: calls that overlap
 * on the GPU race, so order them on one stream. Empty input (rows or L zero) returns ASRN_OK before any other check,
 * as asrn_bucket_sort does.
 * No counterpart in the reference (its sort is torch.argsort, which allocates through PyTorch). */
int asrn_bucket_sort_noalloc(int64_t rows, int64_t L, int32_t nb, const uint16_t* ids_rows, int32_t* orden,
                             uint16_t* ids_o, void* stream);

/* Candidate windows as the scoring kernel selects them (for verification): cand (B*T, L, C) int32 = text position
 * of the j-th most recent bucket mate of sorted slot s (slot s-1-j), -1 if none; suffix (B*T, L, C) uint8 = its
 * suffix-match length with the query, 0..K (asrn/estable.py:232-236, 251, 262-265; asrn/nucleo.py:98-108). */
int asrn_candidates(int64_t B, int64_t L, int32_t T, int32_t C, int32_t K, const int32_t* orden,
                    const uint16_t* ids_o, const float* sig, int32_t* cand, uint8_t* suffix, void* stream);

/* n-gram repetition memory: vistos (B, L, n) uint8, hawkes (B, L, n) float32, racha (B, L) float32.
 * Optional debug outputs (NULL to skip): keys (B, L, n) float64, orden_ng (B, n, L) int32 (stable argsort of the
 * keys, NaN last), repetido (B, n, L) uint8. */
size_t asrn_repetition_workspace_bytes(const asrn_layer_config* cfg);
int asrn_repetition(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const float* sig, const double* beta, const double* Bt, const float* log_alfa, uint8_t* vistos,
                    float* hawkes, float* racha, double* keys, int32_t* orden_ng, uint8_t* repetido,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Gate and output projection: h_out = h + sigmoid(logit) * (W_o W_v)(acc / max(1, tables with candidates)), acc in
 * the compute type (as asrn_score leaves it). The bf16 tensor-core path needs a workspace of
 * asrn_gate_workspace_bytes(cfg) (the per-token gate values; 0 when it is not used). */
size_t asrn_gate_workspace_bytes(const asrn_layer_config* cfg);
int asrn_gate(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
              const float* glogit, const void* acc, const uint8_t* sen_hay, const float* sen_mx,
              const float* sen_pk, const uint8_t* vistos, const float* hawkes, const float* racha, float* h_out,
              void* workspace, size_t workspace_bytes, void* stream);

/* ---- O(1) generation step (the writer's per-token work of one ASRN layer) ------------------------------------------
 * Per layer the caller keeps: rings (B, T, 2^nb, C) int32 and counts (B, T, 2^nb) int32; a Hawkes table of
 * asrn_gen_hawkes_table_bytes(B, n, hcap) bytes (hcap a power of two, at least twice the positions a sequence will
 * hold); per sequence caches of `cap` positions: signatures f32, clock f64, log_alfa f32, phi (P) and Kc (cf) in the
 * compute type; and, shared by every layer, the rows of E in the compute type (the value of position k is row k+1).
 * The step entry points read the new token's position from device memory (t_pos, one int64), so a step is a fixed
 * sequence of launches that a CUDA graph can capture and replay; a position outside [1, cap) makes the kernels write
 * nothing and set ASRN_ERR_ARG in the layer's status word (asrn_layer_status). */

/* Rings of the prompt from its bucket sort (asrn_bucket_sort of the (B*T, L) ids): positions < n_valid, the C most
 * recent of each bucket in slot rank % C, -1 for empty slots; count = positions per bucket. */
int asrn_gen_ring_build(int64_t B, int64_t L, int32_t T, int32_t nb, int32_t C, int64_t n_valid, const int32_t* orden,
                        const uint16_t* ids_o, int32_t* ring, int32_t* count, void* stream);

size_t asrn_gen_hawkes_table_bytes(int64_t B, int32_t n, int64_t cap);
/* Hawkes table at the end of the prompt (cfg->B sequences of L positions; caches with leading dimension ld): for each
 * n-gram key its last occurrence p gives (B_u, A) = (Bt[p], hawkes[p] + exp(log_alfa[p])). hawkes: (B, L, n). */
int asrn_gen_hawkes_build(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, int64_t L,
                          int64_t ld, const float* sig, const double* Bt, const float* log_alfa, const float* hawkes,
                          void* table, int64_t cap, void* stream);

/* Context stage and sign-hash projection of one new token per sequence (cfg->B sequences, cfg->L = 1), with the
 * whole-sequence stages' semantics (asrn_context, asrn_hash) for a token at t >= 1: h, e_t, e_prev (B, d) fp32 (the
 * state, E of the token and of the previous token), tokens (B) int64 -> Qc, Kc (B, cf) in the compute type, beta (B)
 * f64, log_alfa, glogit, sig (B) f32, phi (B, P) in the compute type, ids (B, T) uint16. With scratch (B, 2 *
 * confirmar + 3 + 3 * hidden) float32 the projections are split over (sequence, slice of 32 weight rows) blocks and
 * a second kernel finishes each sequence; with scratch NULL one block per sequence does all of it (the weights read
 * by every block; they stay in L2). Both give the same bits. */
int asrn_gen_front(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                   const float* e_t, const float* e_prev, const int64_t* tokens, void* Qc, void* Kc, double* beta,
                   float* log_alfa, float* glogit, float* sig, void* phi, uint16_t* ids, float* scratch,
                   void* stream);
/* asrn_gen_front on h + y, where y (act, (B, d)) is the previous local block's MLP output that the model adds to the
 * residual stream before the ASRN layer (asrn/nucleo.py:1816-1822): the sum is formed in the kernel that reads h and
 * written to h_sum (float32 (B, d), the gate's residual input), so the step needs no separate add. */
int asrn_gen_front_residual(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                            const float* h, const void* y, float* h_sum, const float* e_t, const float* e_prev,
                            const int64_t* tokens, void* Qc, void* Kc, double* beta, float* log_alfa, float* glogit,
                            float* sig, void* phi, uint16_t* ids, float* scratch, void* stream);

/* Gate of the new tokens (asrn_gate's semantics for cfg->B * cfg->L rows, no workspace): W_ov is spread over d / 32
 * blocks. cbuf / sigma (both or neither; bf16 mode): the operand and gate values asrn_gen_attend precomputed. */
int asrn_gen_gate(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                  const float* glogit, const float* acc, const uint8_t* sen_hay, const float* sen_mx,
                  const float* sen_pk, const uint8_t* vistos, const float* hawkes, const float* racha, float* h_out,
                  const void* cbuf, const float* sigma, void* stream);

/* n-gram memory of the new token at position *t_pos (its signature already in sig_cache): appends its clock
 * Bt[t] = Bt[t-1] + beta_t and log_alfa_t to the caches, then vistos (B, n), hawkes (B, n) from the Hawkes table
 * (updated in place), and the streak racha (B) from racha_state (updated in place). Runs before asrn_gen_attend. */
int asrn_gen_memory(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const int64_t* t_pos, int64_t cap, const float* sig_cache, double* bt_cache, float* la_cache,
                    const double* beta_t, const float* log_alfa_t, void* table, int64_t hcap, float* racha_state,
                    uint8_t* vistos, float* hawkes, float* racha, void* stream);

/* The new token at position *t_pos (phi_t, Qc_t, Kc_t, ids_t; its clock / log_alfa already appended by
 * asrn_gen_memory) against the C candidates of each table from the rings: acc (B, d) = sum over tables of
 * att * E[k + 1] (summed in a fixed order: deterministic); per-table signals (B, T). Appends phi_t and Kc_t to the
 * caches. bf16 mode, optional (all six or none): given g(h) glogit (B), vistos (B, n), hawkes (B, n), racha (B) of
 * the new token, it also writes the gate's operand cbuf (B, d) bf16 = bf16(acc / max(1, pt)) and gate values sigma
 * (B), for asrn_gen_gate. */
int asrn_gen_attend(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const int64_t* t_pos, int64_t cap, const uint16_t* ids_t, const void* phi_t, const void* qc_t,
                    const void* kc_t, const int32_t* ring, const float* sig_cache, const double* bt_cache,
                    const float* la_cache, void* phi_cache, void* kc_cache, const void* ea_cache, float* acc,
                    uint8_t* sen_hay, float* sen_mx, float* sen_pk, const float* glogit, const uint8_t* vistos,
                    const float* hawkes, const float* racha, void* cbuf, float* sigma, void* stream);

/* Put position *t_pos into the ring of its bucket in every table. */
int asrn_gen_ring_insert(int64_t B, int32_t T, int32_t nb, int32_t C, const int64_t* t_pos, const uint16_t* ids_t,
                         int32_t* ring, int32_t* count, void* stream);

/* ---- device sampling with the reference's random numbers ----------------------------------------------------------
 * Replaces the host draw torch.multinomial(prob.cpu(), 1, generator=g) of asrn/nucleo.py:1962 on the CPU generator
 * g = torch.Generator('cpu').manual_seed(semilla) of asrn/nucleo.py:1996. For one sample torch takes, per row, the
 * argmax of prob / q with q an Exp(1) draw per element of prob (one MT19937 64-bit value each, in memory order), so
 * step k of a call on a (B, V) matrix reads the generator's 32-bit outputs [2 B V k, 2 B V (k + 1)).
 * asrn_sampler_seed_state (host): the 624-word MT19937 array manual_seed(seed) starts from (uses seed mod 2^32).
 * asrn_sampler_jump_poly (host): x^distance modulo the generator's characteristic polynomial, 624 words (bit b of word
 *   w = coefficient 32 w + b); the polynomial is found once per process (Berlekamp-Massey, tens of ms) and each
 *   distance is cached. Returns ASRN_ERR_UNSUPPORTED if the polynomial could not be found.
 * asrn_sampler_fill (device): for k < steps, q[k * draws + i] = the i-th Exp(1) draw of the k-th draws-element tensor
 *   made after `state` (624 device words: the window of untempered words the next draw starts from; the seed state
 *   before any draw); polys = levels device polynomials, polys[l] = x^(2^l * 2 * draws) mod phi; steps <= 2^levels.
 *   end_state (device, may be null) receives the window after steps * draws draws. One block per step. q matches
 *   torch's CPU exponential_ bit for bit except where CUDA's double log1p and the host's differ by an ulp at a float
 *   rounding boundary (about 2^-29 of the draws; such a q moves by one float ulp).
 * asrn_sample_argmax (device): out[r] = argmax_j prob[r, j] / q[r, j] (IEEE float division; NaN wins; ties keep the
 *   lower index), torch.multinomial's one-sample rule. A row with an element that is negative, infinite or NaN, or
 *   whose elements are all zero, records ASRN_ERR_DATA in *status (device int, may be null; torch raises there). */
int asrn_sampler_seed_state(uint64_t seed, uint32_t* state);
int asrn_sampler_jump_poly(uint64_t distance, uint32_t* poly);
int asrn_sampler_fill(int64_t draws, int64_t steps, int32_t levels, const uint32_t* state, const uint32_t* polys,
                      float* q, uint32_t* end_state, void* stream);
int asrn_sample_argmax(int64_t rows, int64_t V, const float* prob, const float* q, int64_t* out, int* status,
                       void* stream);
/* out[r] = argmax_j x[r, j] (device), torch.argmax's rule (NaN wins; equal values keep the lower index): the greedy
 * token of a generation step. x (rows, V) fp32 (dtype 0) or bf16 (dtype 1, 16-byte aligned). */
int asrn_argmax_rows(int64_t rows, int64_t V, const void* x, int32_t dtype, int64_t* out, void* stream);

/* ---- test hooks (no counterpart in the reference; the layer forward never calls them) ------------------------------
 * asrn_test_force_cuda_core: 1 routes the bfloat16 work of later calls to the CUDA-core kernels (the fp32 path's), so
 * tests can compare them with the tensor-core kernels; 0 restores the default; a negative value only queries. Returns
 * the previous setting.
 * asrn_test_bounded_wait: one kernel holding TMEM waits, with the limit limit_ns, on an mbarrier that nothing arrives
 * on, through the same bounded wait every tcgen05 kernel uses; the wait gives up, records ASRN_ERR_TIMEOUT in *status
 * (device int, ASRN_OK before) and the kernel frees its TMEM and returns; *result (device int) = 1 if the wait had
 * completed, 0 if it gave up. */
int asrn_test_force_cuda_core(int on);
int asrn_test_bounded_wait(uint64_t limit_ns, int* status, int* result, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ASRN_B200_H */
