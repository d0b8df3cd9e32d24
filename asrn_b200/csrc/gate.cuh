// Gate scalars of one token, shared by the whole-sequence gate (gate.cu) and the generation step (writer.cu).
// Reference: CapaASRNEstable._combinar (asrn/estable.py:376-403), _senales (asrn/estable.py:294-300),
// _respuesta_racha (asrn/nucleo.py:865-878). The per-table signals, g(h), vistos, Hawkes and streak of token g are read
// through the GateArgs pointers (global or shared memory).
#pragma once
#include "common.cuh"
#include "layout.h"

namespace asrn {

// Gate of one token (sigmoid(logit), rounded to the compute type) and max(1, pt).
template <bool Half>
__device__ __forceinline__ void gate_of_token(const GateArgs& a, int64_t g, float* sigma, float* ptc) {
  const int T = a.T;
  float pt = 0.f, mejor = kProhibido, pico = 0.f, pctx = 0.f;
  for (int tau = 0; tau < T; ++tau) {
    const float hay = (float)a.sen_hay[g * T + tau];
    pt = __fadd_rn(pt, hay);
    if (hay > 0.f) mejor = fmaxf(mejor, a.sen_mx[g * T + tau]);
    pico = __fadd_rn(pico, __fmul_rn(a.sen_pk[g * T + tau], hay));
    if (tau >= T - a.Tc) pctx = __fadd_rn(pctx, hay);
  }
  mejor = fmaxf(mejor, kProhibido);
  mejor = (pt > 0.f) ? mejor : 0.f;
  mejor = fminf(fmaxf(mejor, -a.mejor_max), a.mejor_max);
  const float pt1 = fmaxf(pt, 1.f);
  float s[4] = {__fdiv_rn(pt, (float)T), mejor, __fdiv_rn(pico, pt1), __fdiv_rn(pctx, (float)a.Tc)};
  float gc = 0.f;
  for (int i = 0; i < 4; ++i) gc = fmaf(act<Half>(s[i]), a.gconf[i], gc);
  gc = act<Half>(__fadd_rn(gc, a.gconf[4]));
  float logit = __fadd_rn(a.glogit[g], gc);
  float sv = 0.f;
  for (int j = 0; j < a.n; ++j) sv = __fadd_rn(sv, __fmul_rn((float)a.vistos[g * a.n + j], a.w_vistos[j]));
  logit = __fadd_rn(logit, sv);
  float sh = 0.f;
  for (int j = 0; j < a.n; ++j) sh = __fadd_rn(sh, __fmul_rn(log1pf(a.hawkes[g * a.n + j]), a.u_hawkes[j]));
  logit = __fadd_rn(logit, sh);
  // response to the streak: linear interpolation of u_racha on x = log1p(racha) / paso, flat past the last node
  float x = __fdiv_rn(log1pf(a.racha[g]), a.racha_paso);
  x = fminf(x, (float)(a.nodes - 1));
  const float xf = (x != x) ? 0.f : x;
  int i = (int)floorf(xf);
  i = min(max(i, 0), a.nodes - 2);
  const float resp = __fadd_rn(a.u_racha[i], __fmul_rn(__fsub_rn(x, (float)i), a.d_racha[i + 1]));
  logit = __fadd_rn(logit, resp);
  if (a.tope > 0.f) logit = __fmul_rn(a.tope, tanhf(__fdiv_rn(logit, a.tope)));
  *sigma = act<Half>(1.f / (1.f + expf(-logit)));
  *ptc = pt1;
}

}  // namespace asrn
