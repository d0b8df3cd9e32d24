// extern "C" entry points of libasrn_b200.so (declared in include/asrn_b200.h).
#include "common.cuh"
#include "layout.h"

using namespace asrn;

namespace {

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int check_config(const asrn_layer_config* c) {
  if (!c) return ASRN_ERR_ARG;
  if (c->B < 0 || c->L < 0 || c->d < 1 || c->d > 1024) return ASRN_ERR_ARG;
  if (c->n_tablas < 2 || c->n_tablas > kMaxTables) return ASRN_ERR_ARG;
  if (c->n_bits < 1 || c->n_bits > kMaxBits) return ASRN_ERR_ARG;
  if ((int64_t)c->n_tablas * c->n_bits > kMaxPhi) return ASRN_ERR_UNSUPPORTED;
  if (c->chunk < 1 || c->chunk > 32) return ASRN_ERR_UNSUPPORTED;
  if (c->tablas_contexto < 1 || c->tablas_contexto >= c->n_tablas) return ASRN_ERR_ARG;
  if (c->confirmar < 1 || c->confirmar > kMaxConfirm) return ASRN_ERR_UNSUPPORTED;
  if (c->sufijo < 1 || c->sufijo > kMaxSuffix) return ASRN_ERR_UNSUPPORTED;
  if (c->vistos < 1 || c->vistos > kMaxSeen) return ASRN_ERR_UNSUPPORTED;
  if (c->nodos_racha < 2) return ASRN_ERR_ARG;
  if (c->hidden < 1 || c->hidden > kMaxHidden) return ASRN_ERR_UNSUPPORTED;
  if (c->half != 0 && c->half != 1) return ASRN_ERR_ARG;
  if (c->L > (int64_t)1 << 30) return ASRN_ERR_UNSUPPORTED;
  return ASRN_OK;
}

int check_weights(const asrn_layer_weights* w) {
  if (!w) return ASRN_ERR_ARG;
  const void* ps[] = {w->ln_w, w->ln_b, w->cq, w->ck, w->w_reloj, w->b_reloj, w->pal0_w, w->pal0_b, w->pal2_w,
                      w->pal2_b, w->ctx0_w, w->ctx0_b, w->ctx2_w, w->ctx2_b, w->v_w, w->o_w, w->g_w, w->g_b,
                      w->g_conf_w, w->g_conf_b, w->w_vistos, w->u_hawkes, w->log_kappa, w->log_kappa_racha,
                      w->w_sufijo, w->gamma, w->d_racha, w->c_vistos, w->r_firma};
  for (const void* p : ps)
    if (!p) return ASRN_ERR_ARG;
  return ASRN_OK;
}

// Workspace of one layer forward, in order of use.
struct Workspace {
  size_t sig, qc, kc, beta, bt, la, glogit, ea, phi, ids_rows, orden, ids_o, acc, hay, mx, pk, vistos, hawkes,
      racha, sort, sigma, rep, total;
  size_t sort_bytes;
};

Workspace workspace_layout(const asrn_layer_config& c) {
  const size_t M = (size_t)c.B * c.L, es = c.half ? 2 : 4, d = c.d, T = c.n_tablas, n = c.vistos;
  const size_t P = T * c.n_bits;
  Workspace w;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes); return at; };
  w.sig = take(M * 4);
  w.qc = take(M * c.confirmar * es);
  w.kc = take(M * c.confirmar * es);
  w.beta = take(M * 8);
  w.bt = take(M * 8);
  w.la = take(M * 4);
  w.glogit = take(M * 4);
  w.ea = take(c.half ? M * d * es : 0);
  w.phi = take(M * P * es);
  w.ids_rows = take(M * T * 2);
  w.orden = take(M * T * 4);
  w.ids_o = take(M * T * 2);
  w.acc = take(M * d * (c.half ? 2 : 4));      // bf16 accumulator under autocast
  w.hay = take(M * T);
  w.mx = take(M * T * 4);
  w.pk = take(M * T * 4);
  w.vistos = take(M * n);
  w.hawkes = take(M * n * 4);
  w.racha = take(M * 4);
  w.sort_bytes = bucket_sort_workspace((int64_t)c.B * T, c.L, c.n_bits);
  w.sort = take(w.sort_bytes);
  w.sigma = take(M * 8);                       // gate values and 1 / max(1, pt) (tensor-core gate)
  w.rep = take(repetition_workspace(c.B, c.L, c.vistos));
  w.total = o;
  return w;
}

ContextArgs context_args(const asrn_layer_config& c, const asrn_layer_weights& w, const char* prep, const float* h,
                         const float* E, const int64_t* tokens) {
  const PreparedLayout pl = prepared_layout(c);
  ContextArgs a{};
  a.B = c.B; a.L = c.L; a.d = (int)c.d; a.cf = c.confirmar;
  a.h = h; a.E = E; a.tokens = tokens;
  a.ln_w = w.ln_w; a.ln_b = w.ln_b; a.w_reloj = w.w_reloj; a.b_reloj = w.b_reloj;
  a.g_w = w.g_w; a.g_b = w.g_b; a.r_firma = w.r_firma;
  a.wctx = prep + pl.wctx;
  a.beta_max = c.beta_max; a.log_alfa_min = c.log_alfa_min;
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  return a;
}

HashArgs hash_args(const asrn_layer_config& c, const char* prep, const float* E, void* Ea, void* phi,
                   uint16_t* ids_rows) {
  const PreparedLayout pl = prepared_layout(c);
  HashArgs a{};
  a.B = c.B; a.L = c.L; a.d = (int)c.d; a.m = c.hidden; a.T = c.n_tablas; a.Tw = c.n_tablas - c.tablas_contexto;
  a.nb = c.n_bits; a.P = c.n_tablas * c.n_bits;
  a.E = E; a.Ea = Ea;
  a.w1 = prep + pl.w1; a.b1 = reinterpret_cast<const float*>(prep + pl.b1);
  a.w2 = prep + pl.w2; a.b2 = reinterpret_cast<const float*>(prep + pl.b2);
  a.w2bd = prep + pl.w2bd;
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  a.phi = phi; a.ids_rows = ids_rows;
  return a;
}

ScoreArgs score_args(const asrn_layer_config& c, const asrn_layer_weights& w, const char* prep) {
  const PreparedLayout pl = prepared_layout(c);
  ScoreArgs a{};
  a.B = c.B; a.L = c.L; a.d = (int)c.d; a.T = c.n_tablas; a.nb = c.n_bits; a.P = c.n_tablas * c.n_bits;
  a.Lf = c.L; a.q_lo = 0; a.q_hi = c.L;
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  a.C = c.chunk; a.cf = c.confirmar; a.K = c.sufijo;
  a.inv_temp_div = (float)sqrt((double)a.P);
  a.esc_c = (float)pow((double)c.confirmar, -0.5);
  a.w_suf = w.w_sufijo;
  a.tasa = reinterpret_cast<const float*>(prep + pl.tasa);
  return a;
}

RepetitionArgs repetition_args(const asrn_layer_config& c, const asrn_layer_weights& w, const char* prep) {
  const PreparedLayout pl = prepared_layout(c);
  RepetitionArgs a{};
  a.B = c.B; a.L = c.L; a.n = c.vistos;
  a.Lf = c.L; a.pos0 = 0;
  a.c = w.c_vistos;
  a.kappa = reinterpret_cast<const float*>(prep + pl.kappa);
  return a;
}

GateArgs gate_args(const asrn_layer_config& c, const asrn_layer_weights& w, const char* prep) {
  const PreparedLayout pl = prepared_layout(c);
  GateArgs a{};
  a.B = c.B; a.L = c.L; a.d = (int)c.d; a.T = c.n_tablas; a.Tc = c.tablas_contexto; a.n = c.vistos;
  a.nodes = c.nodos_racha;
  a.mejor_max = c.mejor_max; a.tope = c.tope_puerta; a.racha_paso = (float)c.racha_paso;
  a.wov = prep + pl.wov;
  a.gconf = reinterpret_cast<const float*>(prep + pl.gconf);
  a.w_vistos = w.w_vistos; a.u_hawkes = w.u_hawkes; a.d_racha = w.d_racha;
  a.u_racha = reinterpret_cast<const float*>(prep + pl.u_racha);
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  return a;
}

}  // namespace

extern "C" {

const char* asrn_status_string(int status) {
  switch (status) {
    case ASRN_OK: return "ok";
    case ASRN_ERR_ARG: return "invalid argument (shape, null pointer or option out of range)";
    case ASRN_ERR_UNSUPPORTED: return "option combination not supported by this build";
    case ASRN_ERR_WORKSPACE: return "workspace or prepared buffer too small";
    case ASRN_ERR_CUDA: return "CUDA kernel launch failed";
    case ASRN_ERR_DATA: return "state received from another shard failed validation (corrupt or from a faulty rank)";
    case ASRN_ERR_TIMEOUT: return "bounded device wait timed out";
    default: return "unknown status";
  }
}

int asrn_abi_version(void) { return 4; }

size_t asrn_layer_prepared_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return prepared_layout(*cfg).total;
}

int asrn_layer_prepare(const asrn_layer_config* cfg, const asrn_layer_weights* w, void* prepared, size_t bytes,
                       void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || bytes < prepared_layout(*cfg).total) return ASRN_ERR_WORKSPACE;
  return launch_prepare(*cfg, *w, prepared, as_stream(stream));
}

int asrn_layer_status(const asrn_layer_config* cfg, const void* prepared, int reset, void* stream) {
  int st = check_config(cfg);
  if (st) return -st;
  if (!prepared) return -ASRN_ERR_ARG;
  const PreparedLayout pl = prepared_layout(*cfg);
  int* dev = reinterpret_cast<int*>(const_cast<char*>(reinterpret_cast<const char*>(prepared)) + pl.status);
  int host = 0;
  cudaStream_t s = as_stream(stream);
  if (cudaMemcpyAsync(&host, dev, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return -ASRN_ERR_CUDA;
  if (reset && cudaMemsetAsync(dev, 0, sizeof(int), s) != cudaSuccess) return -ASRN_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return -ASRN_ERR_CUDA;
  return host;
}

size_t asrn_layer_workspace_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return workspace_layout(*cfg).total;
}

}  // extern "C"

// The layer forward; with `ngram` (asrn_ngram_shared_sort's output for the same tokens) the repetition stage runs
// only its scans.
static int layer_forward(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                         const float* E, const float* h, const int64_t* tokens, const void* ngram, size_t ngram_bytes,
                         float* h_out, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  const asrn_layer_config& c = *cfg;
  if ((int64_t)c.B * c.L == 0) return ASRN_OK;
  if (!E || !h || !h_out || !prepared) return ASRN_ERR_ARG;
  if (ngram && (!tokens || ngram_bytes < ngram_shared_bytes(c.B, c.L, c.vistos))) return ASRN_ERR_ARG;
  const Workspace ws = workspace_layout(c);
  if (!workspace || workspace_bytes < ws.total) return ASRN_ERR_WORKSPACE;
  cudaStream_t s = as_stream(stream);
  char* base = reinterpret_cast<char*>(workspace);
  const char* prep = reinterpret_cast<const char*>(prepared);
  const int64_t M = c.B * c.L;
  float* sig = reinterpret_cast<float*>(base + ws.sig);
  double* beta = reinterpret_cast<double*>(base + ws.beta);
  double* Bt = reinterpret_cast<double*>(base + ws.bt);
  float* la = reinterpret_cast<float*>(base + ws.la);
  float* glogit = reinterpret_cast<float*>(base + ws.glogit);
  void* Ea = c.half ? (void*)(base + ws.ea) : (void*)E;
  void* phi = base + ws.phi;
  uint16_t* ids_rows = reinterpret_cast<uint16_t*>(base + ws.ids_rows);
  int32_t* orden = reinterpret_cast<int32_t*>(base + ws.orden);
  uint16_t* ids_o = reinterpret_cast<uint16_t*>(base + ws.ids_o);
  void* acc = base + ws.acc;
  uint8_t* hay = reinterpret_cast<uint8_t*>(base + ws.hay);
  float* mx = reinterpret_cast<float*>(base + ws.mx);
  float* pk = reinterpret_cast<float*>(base + ws.pk);
  uint8_t* vistos = reinterpret_cast<uint8_t*>(base + ws.vistos);
  float* hawkes = reinterpret_cast<float*>(base + ws.hawkes);
  float* racha = reinterpret_cast<float*>(base + ws.racha);

  ContextArgs ca = context_args(c, *w, prep, h, E, tokens);
  ca.Qc = base + ws.qc; ca.Kc = base + ws.kc; ca.beta = beta; ca.log_alfa = la; ca.glogit = glogit; ca.sig = sig;
  if ((st = launch_context(ca, c.half, s))) return st;
  if ((st = launch_clock(beta, Bt, c.B, c.L, s))) return st;
  HashArgs ha = hash_args(c, prep, E, Ea, phi, ids_rows);
  if ((st = launch_hash(ha, c.half, s))) return st;
  if ((st = launch_bucket_sort(c.B * c.n_tablas, c.L, c.n_bits, ids_rows, orden, ids_o, base + ws.sort,
                               ws.sort_bytes, s)))
    return st;
  if (cudaMemsetAsync(acc, 0, (size_t)M * c.d * (c.half ? 2 : 4), s) != cudaSuccess) return ASRN_ERR_CUDA;
  ScoreArgs sa = score_args(c, *w, prep);
  sa.orden = orden; sa.ids_o = ids_o; sa.phi = phi; sa.Qc = base + ws.qc; sa.Kc = base + ws.kc; sa.sig = sig;
  sa.Bt = Bt; sa.log_alfa = la; sa.Ea = Ea; sa.acc = acc; sa.sen_hay = hay; sa.sen_mx = mx; sa.sen_pk = pk;
  if ((st = launch_score(sa, c.half, s))) return st;
  RepetitionArgs ra = repetition_args(c, *w, prep);
  ra.sig = sig; ra.beta = beta; ra.Bt = Bt; ra.log_alfa = la; ra.vistos = vistos; ra.hawkes = hawkes;
  ra.racha = racha;
  if (ngram) {
    char* ng = const_cast<char*>(reinterpret_cast<const char*>(ngram));
    ra.ng_mode = kNgScanOnly;
    ra.ng_keys = reinterpret_cast<uint64_t*>(ng);
    ra.ng_pos = reinterpret_cast<uint32_t*>(ng + align_up((size_t)c.B * c.vistos * c.L * 8));
  }
  if ((st = launch_repetition(ra, base + ws.rep, repetition_workspace(c.B, c.L, c.vistos), s))) return st;
  GateArgs ga = gate_args(c, *w, prep);
  ga.h = h; ga.glogit = glogit; ga.sen_hay = hay; ga.sen_mx = mx; ga.sen_pk = pk;
  ga.vistos = vistos; ga.hawkes = hawkes; ga.racha = racha; ga.out = h_out;
  if (c.half) {
    ga.acc16 = reinterpret_cast<const __nv_bfloat16*>(acc);
    ga.sigma = reinterpret_cast<float*>(base + ws.sigma);
    ga.rpt = ga.sigma + M;
  } else {
    ga.acc = reinterpret_cast<const float*>(acc);
  }
  return launch_gate(ga, c.half, s);
}

extern "C" {

int asrn_layer_forward(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                       const float* E, const float* h, const int64_t* tokens, float* h_out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return layer_forward(cfg, w, prepared, E, h, tokens, nullptr, 0, h_out, workspace, workspace_bytes, stream);
}

size_t asrn_ngram_shared_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return ngram_shared_bytes(cfg->B, cfg->L, cfg->vistos);
}

int asrn_ngram_shared_sort(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                           const int64_t* tokens, void* ngram, size_t ngram_bytes, void* workspace,
                           size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  const asrn_layer_config& c = *cfg;
  if ((int64_t)c.B * c.L == 0) return ASRN_OK;
  if (!prepared || !tokens || !ngram || ngram_bytes < ngram_shared_bytes(c.B, c.L, c.vistos)) return ASRN_ERR_ARG;
  RepetitionArgs ra = repetition_args(c, *w, reinterpret_cast<const char*>(prepared));
  char* ng = reinterpret_cast<char*>(ngram);
  ra.tok = tokens;
  ra.ng_mode = kNgSortOnly;
  ra.ng_keys = reinterpret_cast<uint64_t*>(ng);
  ra.ng_pos = reinterpret_cast<uint32_t*>(ng + align_up((size_t)c.B * c.vistos * c.L * 8));
  return launch_repetition(ra, workspace, workspace_bytes, as_stream(stream));
}

int asrn_layer_forward_ngram(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                             const float* E, const float* h, const int64_t* tokens, const void* ngram,
                             size_t ngram_bytes, float* h_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ngram) return ASRN_ERR_ARG;
  return layer_forward(cfg, w, prepared, E, h, tokens, ngram, ngram_bytes, h_out, workspace, workspace_bytes, stream);
}

int asrn_context(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                 const float* E, const int64_t* tokens, void* Qc, void* Kc, double* beta, float* log_alfa,
                 float* glogit, float* sig, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!h || !prepared || !Qc || !Kc || !beta || !log_alfa || !glogit || !sig || (!tokens && !E)) return ASRN_ERR_ARG;
  ContextArgs a = context_args(*cfg, *w, reinterpret_cast<const char*>(prepared), h, E, tokens);
  a.Qc = Qc; a.Kc = Kc; a.beta = beta; a.log_alfa = log_alfa; a.glogit = glogit; a.sig = sig;
  return launch_context(a, cfg->half, as_stream(stream));
}

int asrn_clock(int64_t B, int64_t L, const double* beta, double* Bt, void* stream) {
  if (B < 0 || L < 0 || (B * L > 0 && (!beta || !Bt))) return ASRN_ERR_ARG;
  return launch_clock(beta, Bt, B, L, as_stream(stream));
}

int asrn_hash(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* E,
              void* Ea, void* phi, uint16_t* ids_rows, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if (!prepared || !E || !phi || !ids_rows || (cfg->half && !Ea)) return ASRN_ERR_ARG;
  (void)w;
  HashArgs a = hash_args(*cfg, reinterpret_cast<const char*>(prepared), E, Ea, phi, ids_rows);
  return launch_hash(a, cfg->half, as_stream(stream));
}

int asrn_ids_from_phi(int64_t B, int64_t L, int32_t T, int32_t nb, const float* phi, uint16_t* ids_rows,
                      void* stream) {
  if (B < 0 || L < 0 || T < 1 || nb < 1 || nb > 16 || (B * L > 0 && (!phi || !ids_rows))) return ASRN_ERR_ARG;
  return launch_ids_from_phi(B, L, T, nb, phi, ids_rows, as_stream(stream));
}

size_t asrn_bucket_sort_workspace_bytes(int64_t rows, int64_t L, int32_t nb) {
  return bucket_sort_workspace(rows, L, nb);
}

int asrn_bucket_sort(int64_t rows, int64_t L, int32_t nb, const uint16_t* ids_rows, int32_t* orden,
                     uint16_t* ids_o, void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || L < 0 || (rows * L > 0 && (!ids_rows || !orden || !ids_o))) return ASRN_ERR_ARG;
  return launch_bucket_sort(rows, L, nb, ids_rows, orden, ids_o, workspace, workspace_bytes, as_stream(stream));
}

int asrn_score(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
               const int32_t* orden, const uint16_t* ids_o, const void* phi, const void* Qc, const void* Kc,
               const float* sig, const double* Bt, const float* log_alfa, const void* Ea, void* acc,
               uint8_t* sen_hay, float* sen_mx, float* sen_pk, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !orden || !ids_o || !phi || !Qc || !Kc || !sig || !Bt || !log_alfa || !Ea || !acc || !sen_hay ||
      !sen_mx || !sen_pk)
    return ASRN_ERR_ARG;
  ScoreArgs a = score_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.orden = orden; a.ids_o = ids_o; a.phi = phi; a.Qc = Qc; a.Kc = Kc; a.sig = sig; a.Bt = Bt; a.log_alfa = log_alfa;
  a.Ea = Ea; a.acc = acc; a.sen_hay = sen_hay; a.sen_mx = sen_mx; a.sen_pk = sen_pk;
  return launch_score(a, cfg->half, as_stream(stream));
}

int asrn_shard_rows(int64_t rows, int64_t L, int32_t C, int64_t q_lo, int64_t q_hi, const int32_t* orden,
                    const uint16_t* ids_o, int64_t Lv, int32_t* orden_v, uint16_t* ids_v, int64_t* counts,
                    void* stream) {
  if (rows < 0 || L < 0 || C < 1 || C > 32 || q_lo < 0 || q_hi <= q_lo || q_hi > L || L >= ((int64_t)1 << 31) ||
      (q_lo == 0 && q_hi == L) || (rows * L > 0 && (!orden || !ids_o)))
    return ASRN_ERR_ARG;
  if (orden_v ? (!ids_v || Lv < 1) : !counts) return ASRN_ERR_ARG;   // counts is optional when compacting
  const int32_t pad_pos = (int32_t)(q_lo > 0 ? 0 : q_hi);
  return launch_shard_rows(rows, L, C, q_lo, q_hi, orden, ids_o, Lv, orden_v, ids_v, counts, pad_pos,
                           as_stream(stream));
}

size_t asrn_shard_workspace_bytes(int64_t rows, int32_t nb) {
  if (rows < 0 || nb < 1 || nb > 15) return 0;
  return shard_merge_workspace(rows, nb);
}

int asrn_shard_tails(int64_t rows, int64_t Lc, int32_t nb, int32_t C, int64_t c0, const int32_t* orden_loc,
                     const uint16_t* ids_loc, int32_t* tails, void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || Lc < 0 || nb < 1 || nb > 15 || C < 1 || C > 32 || c0 < 0 || c0 + Lc >= ((int64_t)1 << 31) ||
      (rows * Lc > 0 && (!orden_loc || !ids_loc)) || (rows > 0 && !tails))
    return ASRN_ERR_ARG;
  if (rows == 0) return ASRN_OK;
  if (!workspace || workspace_bytes < shard_merge_workspace(rows, nb)) return ASRN_ERR_WORKSPACE;
  return launch_shard_tails(rows, Lc, nb, C, c0, orden_loc, ids_loc, tails, workspace, as_stream(stream));
}

int asrn_shard_merge(int64_t rows, int64_t Lc, int32_t nb, int32_t C, int64_t c0, int32_t n_prev,
                     const int32_t* tails_prev, const int32_t* orden_loc, const uint16_t* ids_loc, int64_t Lv,
                     int32_t* orden_v, uint16_t* ids_v, int64_t* row_len, int64_t L, void* workspace,
                     size_t workspace_bytes, int* status, void* stream) {
  if (rows < 0 || Lc < 1 || nb < 1 || nb > 15 || C < 1 || C > 32 || c0 < 0 || n_prev < 0 || L < c0 + Lc ||
      L >= ((int64_t)1 << 31) || (c0 == 0 && c0 + Lc == L) || (n_prev > 0 && !tails_prev) ||
      (rows > 0 && (!orden_loc || !ids_loc || !orden_v || !ids_v || !row_len)))
    return ASRN_ERR_ARG;
  const int64_t ring_max = ((int64_t)1 << nb) * C;
  if (Lv < Lc + (c0 < ring_max ? c0 : ring_max)) return ASRN_ERR_ARG;
  if (rows == 0) return ASRN_OK;
  if (!workspace || workspace_bytes < shard_merge_workspace(rows, nb)) return ASRN_ERR_WORKSPACE;
  const int32_t pad_pos = (int32_t)(c0 > 0 ? 0 : c0 + Lc);
  return launch_shard_merge(rows, Lc, nb, C, c0, n_prev, tails_prev, orden_loc, ids_loc, Lv, orden_v, ids_v, row_len,
                            pad_pos, status, workspace, as_stream(stream));
}

int asrn_score_shard(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, int64_t L_feat,
                     int64_t q_lo, int64_t q_hi, const int32_t* orden, const uint16_t* ids_o, const void* phi,
                     const void* Qc, const void* Kc, const float* sig, const double* Bt, const float* log_alfa,
                     const void* Ea, const int64_t* row_len, void* acc, uint8_t* sen_hay, float* sen_mx,
                     float* sen_pk, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !orden || !ids_o || !phi || !Qc || !Kc || !sig || !Bt || !log_alfa || !Ea || !acc || !sen_hay ||
      !sen_mx || !sen_pk || q_lo < 0 || q_hi <= q_lo || q_hi > L_feat || L_feat >= ((int64_t)1 << 31))
    return ASRN_ERR_ARG;
  ScoreArgs a = score_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.Lf = L_feat; a.q_lo = q_lo; a.q_hi = q_hi;
  a.orden = orden; a.ids_o = ids_o; a.phi = phi; a.Qc = Qc; a.Kc = Kc; a.sig = sig; a.Bt = Bt; a.log_alfa = log_alfa;
  a.Ea = Ea; a.row_len = row_len; a.acc = acc; a.sen_hay = sen_hay; a.sen_mx = sen_mx; a.sen_pk = sen_pk;
  return launch_score(a, cfg->half, as_stream(stream));
}

int asrn_bucket_sort_noalloc(int64_t rows, int64_t L, int32_t nb, const uint16_t* ids_rows, int32_t* orden,
                             uint16_t* ids_o, void* stream) {
  if (rows < 0 || L < 0 || (rows * L > 0 && (!ids_rows || !orden || !ids_o))) return ASRN_ERR_ARG;
  return launch_bucket_sort_noalloc(rows, L, nb, ids_rows, orden, ids_o, as_stream(stream));
}

int asrn_candidates(int64_t B, int64_t L, int32_t T, int32_t C, int32_t K, const int32_t* orden,
                    const uint16_t* ids_o, const float* sig, int32_t* cand, uint8_t* suffix, void* stream) {
  if (B < 0 || L < 0 || T < 1 || (B * L > 0 && (!orden || !ids_o || !sig || !cand || !suffix))) return ASRN_ERR_ARG;
  return launch_candidates(B, L, T, C, K, orden, ids_o, sig, cand, suffix, as_stream(stream));
}

size_t asrn_repetition_workspace_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return repetition_workspace(cfg->B, cfg->L, cfg->vistos);
}

int asrn_repetition(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const float* sig, const double* beta, const double* Bt, const float* log_alfa, uint8_t* vistos,
                    float* hawkes, float* racha, double* keys, int32_t* orden_ng, uint8_t* repetido,
                    void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !sig || !beta || !Bt || !log_alfa || !vistos || !hawkes || !racha) return ASRN_ERR_ARG;
  RepetitionArgs a = repetition_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.sig = sig; a.beta = beta; a.Bt = Bt; a.log_alfa = log_alfa; a.vistos = vistos; a.hawkes = hawkes; a.racha = racha;
  a.keys = keys; a.orden_ng = orden_ng; a.repetido = repetido;
  return launch_repetition(a, workspace, workspace_bytes, as_stream(stream));
}

size_t asrn_ngram_chunk_workspace_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return ngram_chunk_workspace(cfg->B, cfg->L, cfg->vistos);
}

int asrn_ngram_chunk_sort(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                          int64_t L_feat, int64_t c0, const float* sig, const double* Bt, const float* log_alfa,
                          uint64_t* keys, void* summary, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !sig || !Bt || !log_alfa || !keys || !summary || c0 < 0 || c0 + cfg->L > L_feat ||
      L_feat >= ((int64_t)1 << 31))
    return ASRN_ERR_ARG;
  RepetitionArgs a = repetition_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.Lf = L_feat; a.pos0 = c0;
  a.sig = sig; a.Bt = Bt; a.log_alfa = log_alfa;
  return launch_ngram_chunk_sort(a, keys, summary, workspace, workspace_bytes, as_stream(stream));
}

int asrn_ngram_chunk_finish(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                            int64_t L_feat, int64_t c0, int32_t n_prev, const uint64_t* keys_prev,
                            const void* summary_prev, const uint64_t* keys, const double* Bt, const float* log_alfa,
                            uint8_t* vistos, float* hawkes, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !keys || !Bt || !log_alfa || !vistos || !hawkes || n_prev < 0 ||
      (n_prev > 0 && (!keys_prev || !summary_prev)) || c0 < 0 || c0 + cfg->L > L_feat ||
      L_feat >= ((int64_t)1 << 31))
    return ASRN_ERR_ARG;
  RepetitionArgs a = repetition_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.Lf = L_feat; a.pos0 = c0;
  a.Bt = Bt; a.log_alfa = log_alfa; a.vistos = vistos; a.hawkes = hawkes;
  return launch_ngram_chunk_finish(a, n_prev, keys_prev, summary_prev, keys, workspace, workspace_bytes,
                                   as_stream(stream));
}

size_t asrn_racha_workspace_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return racha_workspace(cfg->B, cfg->L);
}

int asrn_racha_chunk(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                     const uint8_t* vistos, const double* beta, const float* racha_in, float* racha, float* racha_map,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !vistos || !beta || (!racha && !racha_map)) return ASRN_ERR_ARG;
  RepetitionArgs a = repetition_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.vistos = const_cast<uint8_t*>(vistos); a.beta = beta; a.racha = racha;
  a.racha_in = racha_in; a.racha_map = racha_map;
  return launch_racha_ws(a, workspace, workspace_bytes, as_stream(stream));
}

size_t asrn_gate_workspace_bytes(const asrn_layer_config* cfg) {
  if (check_config(cfg) != ASRN_OK) return 0;
  return gate_workspace(cfg->B * cfg->L, (int)cfg->d, cfg->half != 0);
}

int asrn_gate(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
              const float* glogit, const void* acc, const uint8_t* sen_hay, const float* sen_mx,
              const float* sen_pk, const uint8_t* vistos, const float* hawkes, const float* racha, float* h_out,
              void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !h || !glogit || !acc || !sen_hay || !sen_mx || !sen_pk || !vistos || !hawkes || !racha || !h_out)
    return ASRN_ERR_ARG;
  GateArgs a = gate_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.h = h; a.glogit = glogit; a.sen_hay = sen_hay; a.sen_mx = sen_mx; a.sen_pk = sen_pk;
  a.vistos = vistos; a.hawkes = hawkes; a.racha = racha; a.out = h_out;
  if (cfg->half) a.acc16 = reinterpret_cast<const __nv_bfloat16*>(acc);
  else a.acc = reinterpret_cast<const float*>(acc);
  const size_t need = gate_workspace(cfg->B * cfg->L, (int)cfg->d, cfg->half != 0);
  if (need > 0) {
    if (!workspace || workspace_bytes < need) return ASRN_ERR_WORKSPACE;
    a.sigma = reinterpret_cast<float*>(workspace);
    a.rpt = a.sigma + cfg->B * cfg->L;
  }
  return launch_gate(a, cfg->half, as_stream(stream));
}

// ---- generation step ---------------------------------------------------------------------------------------------

int asrn_gen_ring_build(int64_t B, int64_t L, int32_t T, int32_t nb, int32_t C, int64_t n_valid, const int32_t* orden,
                        const uint16_t* ids_o, int32_t* ring, int32_t* count, void* stream) {
  if (B < 0 || L < 0 || T < 1 || nb < 1 || nb > 16 || C < 1 || C > 32 || !ring || !count ||
      (B * L > 0 && (!orden || !ids_o)))
    return ASRN_ERR_ARG;
  return launch_ring_build(B, L, T, nb, C, n_valid, orden, ids_o, ring, count, as_stream(stream));
}

size_t asrn_gen_hawkes_table_bytes(int64_t B, int32_t n, int64_t cap) { return hawkes_table_bytes(B, n, cap); }

int asrn_gen_hawkes_build(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, int64_t L,
                          int64_t ld, const float* sig, const double* Bt, const float* log_alfa, const float* hawkes,
                          void* table, int64_t cap, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !table || (cfg->B * L > 0 && (!sig || !Bt || !log_alfa || !hawkes)) || ld < L) return ASRN_ERR_ARG;
  const PreparedLayout pl = prepared_layout(*cfg);
  int* status = reinterpret_cast<int*>(const_cast<char*>(reinterpret_cast<const char*>(prepared)) + pl.status);
  return launch_hawkes_build(cfg->B, L, ld, cfg->vistos, sig, w->c_vistos, Bt, log_alfa, hawkes, table, cap, status,
                             as_stream(stream));
}

static GenArgs gen_args(const asrn_layer_config& c, const asrn_layer_weights& w, const char* prep,
                        const int64_t* t_pos, int64_t cap) {
  const PreparedLayout pl = prepared_layout(c);
  GenArgs a{};
  a.B = c.B; a.t_pos = t_pos; a.cap = cap;
  a.d = (int)c.d; a.T = c.n_tablas; a.nb = c.n_bits; a.P = c.n_tablas * c.n_bits; a.C = c.chunk; a.cf = c.confirmar;
  a.K = c.sufijo; a.n = c.vistos;
  a.inv_temp_div = (float)sqrt((double)a.P);
  a.esc_c = (float)pow((double)c.confirmar, -0.5);
  a.w_suf = w.w_sufijo;
  a.tasa = reinterpret_cast<const float*>(prep + pl.tasa);
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  return a;
}

int asrn_gen_attend(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const int64_t* t_pos, int64_t cap, const uint16_t* ids_t, const void* phi_t, const void* qc_t,
                    const void* kc_t, const int32_t* ring, const float* sig_cache, const double* bt_cache,
                    const float* la_cache, void* phi_cache, void* kc_cache, const void* ea_cache, float* acc,
                    uint8_t* sen_hay, float* sen_mx, float* sen_pk, const float* glogit, const uint8_t* vistos,
                    const float* hawkes, const float* racha, void* cbuf, float* sigma, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !t_pos || !ids_t || !phi_t || !qc_t || !kc_t || !ring || !sig_cache || !bt_cache || !la_cache ||
      !phi_cache || !kc_cache || !ea_cache || !acc || !sen_hay || !sen_mx || !sen_pk || cap < 2)
    return ASRN_ERR_ARG;
  // optional gate precomputation (bf16 mode): all of glogit, vistos, hawkes, racha, cbuf, sigma, or none
  const bool pre = cbuf || sigma;
  if (pre && (!cfg->half || !cbuf || !sigma || !glogit || !vistos || !hawkes || !racha)) return ASRN_ERR_ARG;
  GateArgs ga = gate_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  if (pre) {
    ga.glogit = glogit; ga.vistos = vistos; ga.hawkes = hawkes; ga.racha = racha;
    ga.cbuf = reinterpret_cast<__nv_bfloat16*>(cbuf); ga.sigma = sigma;
  }
  GenArgs a = gen_args(*cfg, *w, reinterpret_cast<const char*>(prepared), t_pos, cap);
  a.ids_t = ids_t; a.phi_t = phi_t; a.qc_t = qc_t; a.kc_t = kc_t; a.ring = ring; a.sig_cache = sig_cache;
  a.bt_cache = bt_cache; a.la_cache = la_cache; a.phi_cache = phi_cache; a.kc_cache = kc_cache;
  a.phi_cache_w = phi_cache; a.kc_cache_w = kc_cache; a.ea_cache = ea_cache; a.acc = acc;
  a.sen_hay = sen_hay; a.sen_mx = sen_mx; a.sen_pk = sen_pk;
  return launch_gen_attend(a, ga, cfg->half != 0, as_stream(stream));
}

int asrn_gen_memory(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                    const int64_t* t_pos, int64_t cap, const float* sig_cache, double* bt_cache, float* la_cache,
                    const double* beta_t, const float* log_alfa_t, void* table, int64_t hcap, float* racha_state,
                    uint8_t* vistos, float* hawkes, float* racha, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (!prepared || !t_pos || !sig_cache || !bt_cache || !la_cache || !beta_t || !log_alfa_t || !table ||
      !racha_state || !vistos || !hawkes || !racha || cap < 2)
    return ASRN_ERR_ARG;
  const char* prep = reinterpret_cast<const char*>(prepared);
  const PreparedLayout pl = prepared_layout(*cfg);
  GenArgs a = gen_args(*cfg, *w, prep, t_pos, cap);
  a.sig_cache = sig_cache; a.bt_cache = bt_cache; a.bt_w = bt_cache; a.la_cache = la_cache; a.la_w = la_cache;
  return launch_gen_memory(a, table, hcap, w->c_vistos, reinterpret_cast<const float*>(prep + pl.kappa), beta_t,
                           log_alfa_t, racha_state, vistos, hawkes, racha, a.status, as_stream(stream));
}

int asrn_gen_ring_insert(int64_t B, int32_t T, int32_t nb, int32_t C, const int64_t* t_pos, const uint16_t* ids_t,
                         int32_t* ring, int32_t* count, void* stream) {
  if (B < 0 || T < 1 || nb < 1 || nb > 16 || C < 1 || C > 32 || (B > 0 && (!t_pos || !ids_t || !ring || !count)))
    return ASRN_ERR_ARG;
  return launch_ring_insert(B, T, nb, C, t_pos, ids_t, ring, count, as_stream(stream));
}

static int gen_front(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                     const void* y, float* h_sum, const float* e_t, const float* e_prev, const int64_t* tokens,
                     void* Qc, void* Kc, double* beta, float* log_alfa, float* glogit, float* sig, void* phi,
                     uint16_t* ids, float* scratch, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (cfg->B > 0 && (!prepared || !h || !e_t || !e_prev || !tokens || !Qc || !Kc || !beta || !log_alfa || !glogit ||
                     !sig || !phi || !ids))
    return ASRN_ERR_ARG;
  const char* prep = reinterpret_cast<const char*>(prepared);
  const PreparedLayout pl = prepared_layout(*cfg);
  GenFrontArgs a{};
  a.B = cfg->B; a.d = (int)cfg->d; a.cf = cfg->confirmar; a.m = cfg->hidden; a.T = cfg->n_tablas;
  a.Tw = cfg->n_tablas - cfg->tablas_contexto; a.nb = cfg->n_bits; a.P = cfg->n_tablas * cfg->n_bits;
  a.h = h; a.e_t = e_t; a.e_prev = e_prev; a.tokens = tokens;
  a.ln_w = w->ln_w; a.ln_b = w->ln_b; a.w_reloj = w->w_reloj; a.b_reloj = w->b_reloj; a.g_w = w->g_w; a.g_b = w->g_b;
  a.wctx = prep + pl.wctx; a.w1 = prep + pl.w1; a.b1 = reinterpret_cast<const float*>(prep + pl.b1);
  a.w2 = prep + pl.w2; a.b2 = reinterpret_cast<const float*>(prep + pl.b2);
  a.beta_max = cfg->beta_max; a.log_alfa_min = cfg->log_alfa_min;
  a.Qc = Qc; a.Kc = Kc; a.beta = beta; a.log_alfa = log_alfa; a.glogit = glogit; a.sig = sig; a.phi = phi; a.ids = ids;
  a.dots = scratch;
  a.status = reinterpret_cast<int*>(const_cast<char*>(prep) + pl.status);
  a.y = y;
  a.h_sum = h_sum;
  return launch_gen_front(a, cfg->half != 0, as_stream(stream));
}

int asrn_gen_front(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                   const float* e_t, const float* e_prev, const int64_t* tokens, void* Qc, void* Kc, double* beta,
                   float* log_alfa, float* glogit, float* sig, void* phi, uint16_t* ids, float* scratch,
                   void* stream) {
  return gen_front(cfg, w, prepared, h, nullptr, nullptr, e_t, e_prev, tokens, Qc, Kc, beta, log_alfa, glogit, sig,
                   phi, ids, scratch, stream);
}

int asrn_gen_front_residual(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared,
                            const float* h, const void* y, float* h_sum, const float* e_t, const float* e_prev,
                            const int64_t* tokens, void* Qc, void* Kc, double* beta, float* log_alfa, float* glogit,
                            float* sig, void* phi, uint16_t* ids, float* scratch, void* stream) {
  if (cfg && cfg->B > 0 && (!y || !h_sum)) return ASRN_ERR_ARG;
  return gen_front(cfg, w, prepared, h, y, h_sum, e_t, e_prev, tokens, Qc, Kc, beta, log_alfa, glogit, sig, phi, ids,
                   scratch, stream);
}

int asrn_gen_gate(const asrn_layer_config* cfg, const asrn_layer_weights* w, const void* prepared, const float* h,
                  const float* glogit, const float* acc, const uint8_t* sen_hay, const float* sen_mx,
                  const float* sen_pk, const uint8_t* vistos, const float* hawkes, const float* racha, float* h_out,
                  const void* cbuf, const float* sigma, void* stream) {
  int st = check_config(cfg);
  if (st) return st;
  if ((st = check_weights(w))) return st;
  if (cfg->B * cfg->L > 0 && (!prepared || !h || !glogit || !acc || !sen_hay || !sen_mx || !sen_pk || !vistos ||
                              !hawkes || !racha || !h_out))
    return ASRN_ERR_ARG;
  GateArgs a = gate_args(*cfg, *w, reinterpret_cast<const char*>(prepared));
  a.h = h; a.glogit = glogit; a.acc = acc; a.sen_hay = sen_hay; a.sen_mx = sen_mx; a.sen_pk = sen_pk;
  a.vistos = vistos; a.hawkes = hawkes; a.racha = racha; a.out = h_out;
  if ((cbuf != nullptr) != (sigma != nullptr) || (cbuf && !cfg->half)) return ASRN_ERR_ARG;
  a.cbuf = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(cbuf));
  a.sigma = const_cast<float*>(sigma);
  return launch_gen_gate(a, cfg->half != 0, as_stream(stream));
}

int asrn_local_in(int64_t B, int32_t d, int32_t k, const float* h_prev, const void* y_prev, float* h_out,
                  const float* ln_w, const float* ln_b, float eps, void* win, int32_t half, void* stream) {
  if (B < 0 || d < 1 || k < 1 || k > 16 || (B > 0 && (!h_prev || !ln_w || !ln_b || !win))) return ASRN_ERR_ARG;
  return launch_local_in(B, d, k, h_prev, y_prev, h_out, ln_w, ln_b, eps, win, half != 0, as_stream(stream));
}

int asrn_local_mid(int64_t B, int32_t d, const float* h, const void* z, float* h1, const float* ln_w,
                   const float* ln_b, float eps, void* v_out, int32_t half, void* stream) {
  if (B < 0 || d < 1 || (B > 0 && (!h || !z || !h1 || !ln_w || !ln_b || !v_out))) return ASRN_ERR_ARG;
  return launch_local_mid(B, d, h, z, h1, ln_w, ln_b, eps, v_out, half != 0, as_stream(stream));
}

int asrn_local_gelu(int64_t n, void* f, int32_t half, void* stream) {
  if (n < 0 || (n > 0 && !f)) return ASRN_ERR_ARG;
  return launch_local_gelu(n, f, half != 0, as_stream(stream));
}

}  // extern "C"
