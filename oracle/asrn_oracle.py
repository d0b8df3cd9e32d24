"""CPU oracle for the ASRN layer forward and its O(1) generation step -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's own algorithm (KIROKOWA/ASRN, `asrn/estable.py` + `asrn/nucleo.py`), used as
the checker by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg. The product path
(asrn_b200/) never imports this module: it runs the CUDA kernels of libasrn_b200.so or fails.

Parity of this restatement is pinned against the reference itself: tests/golden/*.npz hold the reference's
intermediates and outputs on seeded inputs (made by tests/golden/make_golden.py, which imports the reference), and
tests/test_oracle_golden.py checks this module against every one of them.

Precision modes
  bf16=False  every tensor op in fp32 (fp64 for the clock and the n-gram keys), as the reference without autocast.
  bf16=True   emulates torch.autocast(dtype=bfloat16) on the CPU: the inputs of F.linear / bmm / einsum are rounded
              to bfloat16, products accumulate in fp32 and the result is rounded to bfloat16; element-wise ops on
              bf16 tensors round their result to bf16; mixing a bf16 and an fp32 tensor promotes to fp32.
"""
import math

import numpy as np

try:
    from scipy.special import erf as _erf
except ImportError:                                   # pragma: no cover - scipy is in the image
    _erf = np.vectorize(math.erf, otypes=[np.float64])

PROHIBIDO = -1e9                                      # asrn/nucleo.py:86


# --------------------------------------------------------------------------------------------------------------------
# bfloat16 emulation
# --------------------------------------------------------------------------------------------------------------------

def bf16(x):
    """Round to the nearest bfloat16 (ties to even), returned as float32 (the rounding torch's .to(bfloat16) does)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = u + np.uint32(0x7FFF)
    r += (u >> np.uint32(16)) & np.uint32(1)
    r &= np.uint32(0xFFFF0000)
    out = r.view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, x, out)
    return out


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def linear(x, W, b=None, half=False):
    """F.linear(x, W, b). half: autocast bf16 (inputs and bias to bf16, fp32 accumulation, bf16 output)."""
    if half:
        x, W = bf16(x), bf16(W)
        b = None if b is None else bf16(b)
    y = np.matmul(x.astype(np.float64), W.astype(np.float64).T)
    if b is not None:
        y = y + b.astype(np.float64)
    y = y.astype(np.float32)
    return bf16(y) if half else y


def softplus(x):
    """torch.nn.functional.softplus (beta=1, threshold=20)."""
    x = _f32(x)
    with np.errstate(over='ignore'):
        return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))).astype(np.float32)


def logsigmoid(x):
    x = _f32(x)
    return (np.minimum(x, 0) - np.log1p(np.exp(-np.abs(x)))).astype(np.float32)


def gelu(x, half=False):
    y = (0.5 * x.astype(np.float64) * (1.0 + _erf(x.astype(np.float64) / math.sqrt(2.0)))).astype(np.float32)
    return bf16(y) if half else y


def layer_norm(x, w, b, eps=1e-5):
    x64 = x.astype(np.float64)
    mu = x64.mean(-1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(-1, keepdims=True)
    return ((x64 - mu) / np.sqrt(var + eps) * w + b).astype(np.float32)


# --------------------------------------------------------------------------------------------------------------------
# Layer options and parameters
# --------------------------------------------------------------------------------------------------------------------

class Layer:
    """Parameters (state_dict names of asrn.estable.CapaASRNEstable) + options (asrn/nucleo.py:585-630,
    asrn/estable.py:57-77)."""

    def __init__(self, params, d, n_tablas=8, n_bits=14, afin_oculto=128, chunk=32, tablas_contexto=4, confirmar=16,
                 sufijo=4, vistos=4, nodos_racha=16, racha_max=256, mascara_exacta=True, reloj_64=True,
                 beta_max=1e4, log_alfa_min=-30.0, mejor_max=1e4, tope_puerta=None, kappa_min=None, **_):
        self.p = {k: np.asarray(v) for k, v in params.items()}
        self.d, self.T, self.nb, self.C = d, n_tablas, n_bits, chunk
        self.Tc, self.cf, self.K, self.n = tablas_contexto, confirmar, sufijo, vistos
        self.m = max(8, afin_oculto // 2)
        self.temperatura = (n_tablas * n_bits) ** 0.5
        self.racha_paso = math.log1p(racha_max) / (nodos_racha - 1)
        self.mascara_exacta, self.reloj_64 = mascara_exacta, reloj_64
        self.beta_max, self.log_alfa_min, self.mejor_max = beta_max, log_alfa_min, mejor_max
        self.tope_puerta, self.kappa_min = tope_puerta, kappa_min
        if not (mascara_exacta and reloj_64):
            raise NotImplementedError('the oracle restates the default protections (group A): exact mask, 64-bit clock')

    def __getitem__(self, k):
        return self.p[k]

    def kappas(self):
        """asrn/estable.py:196-200."""
        k = np.exp(self['log_kappa'].astype(np.float32))
        kr = np.exp(self['log_kappa_racha'].astype(np.float32))
        if self.kappa_min is not None:
            k, kr = np.maximum(k, np.float32(self.kappa_min)), np.maximum(kr, np.float32(self.kappa_min))
        return k.astype(np.float32), kr.astype(np.float32)


def firmas_de_piezas(tokens):
    """asrn/nucleo.py:161-164: token id -> fp32 signature."""
    return np.asarray(tokens).astype(np.float32)


def anteriores(sig, n, desde=1):
    """asrn/nucleo.py:167-172: (B, L, n) signatures of t-desde, t-desde-1, ... (NaN before the start)."""
    B, L = sig.shape
    out = np.full((B, L, n), np.nan, dtype=sig.dtype)
    for j in range(n):
        s = desde + j
        if s < L:
            out[:, s:, j] = sig[:, :L - s]
    return out


def largo_seguido(a, b):
    """asrn/nucleo.py:98-108: number of leading positions where a == b (NaN never matches)."""
    sigue = a[..., 0] == b[..., 0]
    largo = sigue.astype(np.int32)
    for j in range(1, a.shape[-1]):
        sigue = sigue & (a[..., j] == b[..., j])
        largo = largo + sigue
    return largo


# --------------------------------------------------------------------------------------------------------------------
# The layer forward, part by part
# --------------------------------------------------------------------------------------------------------------------

def contexto(lay, h, half):
    """asrn/estable.py:153-194 (CPU branches): LN(h) -> Qc, Kc, beta (fp64), log_alfa."""
    cf = lay.cf
    hh32 = layer_norm(h, lay['ln_ctx.weight'], lay['ln_ctx.bias'])
    if half:
        y = linear(hh32, np.concatenate([lay['cq.weight'], lay['ck.weight']]), half=True)
        u = linear(hh32, lay['w_reloj'], lay['b_reloj'])
        Qc, Kc = y[..., :cf], y[..., cf:]
    else:
        W = np.concatenate([lay['cq.weight'], lay['ck.weight'], lay['w_reloj']])
        b = np.concatenate([np.zeros(2 * cf, np.float32), lay['b_reloj']])
        y = linear(hh32, W, b)
        Qc, Kc, u = y[..., :cf], y[..., cf:2 * cf], y[..., 2 * cf:]
    beta = softplus(u[..., 0])
    log_alfa = (logsigmoid(u[..., 1]) + np.float32(math.log(2))).astype(np.float32)
    if lay.beta_max is not None:
        beta = np.minimum(beta, np.float32(lay.beta_max))
    if lay.log_alfa_min is not None:
        log_alfa = np.maximum(log_alfa, np.float32(lay.log_alfa_min))
    return Qc, Kc, beta.astype(np.float64), log_alfa


def phi_y_valores(lay, E, half):
    """asrn/nucleo.py:644-659: phi (B, L, T*nb) [word tables, then context tables] and V_t = v(E_{t+1})."""
    d, L, m = lay.d, E.shape[1], lay.m
    Ea = bf16(E) if half else E.astype(np.float32)
    y = linear(Ea, np.concatenate([lay['afin_palabra.0.weight'], lay['v.weight']]),
               np.concatenate([lay['afin_palabra.0.bias'], np.zeros(d, np.float32)]), half)
    hp, v = y[..., :m], y[..., m:]
    prev = np.zeros_like(Ea)
    prev[:, 1:] = Ea[:, :-1]
    llave = np.concatenate([Ea, prev], -1)
    c0 = linear(llave, lay['afin_contexto.0.weight'], lay['afin_contexto.0.bias'], half)
    phi_w = linear(gelu(hp, half), lay['afin_palabra.2.weight'], lay['afin_palabra.2.bias'], half)
    phi_c = linear(gelu(c0, half), lay['afin_contexto.2.weight'], lay['afin_contexto.2.bias'], half)
    phi = np.concatenate([phi_w, phi_c], -1)
    V = np.zeros_like(v)
    V[:, :-1] = v[:, 1:]
    return phi, V


def ids_de(phi, T, nb):
    """asrn/nucleo.py:661-664: bucket of each table = the signs of its nb outputs read as a number (bit j = col j)."""
    bits = phi.reshape(*phi.shape[:-1], T, nb) > 0
    return (bits.astype(np.int64) << np.arange(nb)).sum(-1).astype(np.int32)


def bucket_sort(ids):
    """asrn/estable.py:220-221: per row b*T + tau, the stable argsort of the bucket ids (ties by position)."""
    B, L, T = ids.shape
    rows = ids.transpose(0, 2, 1).reshape(B * T, L)
    orden = np.argsort(rows, axis=-1, kind='stable').astype(np.int32)
    return orden, np.take_along_axis(rows, orden, -1)


def candidatos_filas(ids_o_row, C):
    """asrn/estable.py:232-236, 262-265: for each sorted slot s, the candidate slots [max(0, s-C), s) with the same
    id (the previous block + current block window restricted to the C slots before the query). Returns lo (L,):
    the candidates of s are the slots lo[s] .. s-1."""
    L = ids_o_row.shape[0]
    lo = np.empty(L, np.int64)
    start = 0
    for s in range(L):
        if s == 0 or ids_o_row[s] != ids_o_row[s - 1]:
            start = s
        lo[s] = max(start, s - C)
    return lo


def acumular(lay, E, Qc, Kc, Bt, log_alfa, sig, half, want_detail=False, ids_override=None):
    """asrn/estable.py:204-300 restated per query: each (row, sorted slot) scores its candidates with
      s = <phi_q, phi_k>/sqrt(P) + <Qc_q, Kc_k> cf^-1/2 + w_suf[suffix length] + log_alfa_k + (gamma_tau / C)(B_k - B_q)
    (clock difference in fp64, then fp32), exact-mask softmax (asrn/estable.py:121-138), copies the next token's value
    and sums the T tables in text order; the gate signals come from _senales (asrn/estable.py:294-300)."""
    B, L, d = E.shape
    T, C, K = lay.T, lay.C, lay.K
    phi, V = phi_y_valores(lay, E, half)
    ids = ids_de(phi, T, lay.nb) if ids_override is None else np.asarray(ids_override, np.int32)
    orden, ids_o = bucket_sort(ids)
    Pf = anteriores(sig, K)
    tasa = (lay['gamma'].astype(np.float32) / np.float32(C)).astype(np.float32)
    w_suf = lay['w_sufijo'].astype(np.float32)
    inv_t = np.float32(lay.temperatura)
    esc_c = np.float32(lay.cf ** -0.5)
    out_t = np.zeros((B, T, L, d), np.float32)
    senal = np.zeros((B, T, L, 3), np.float32)
    detail = {'lo': np.zeros((B * T, L), np.int64), 'largo': {}}
    for b in range(B):
        for tau in range(T):
            r = b * T + tau
            lo = candidatos_filas(ids_o[r], C)
            detail['lo'][r] = lo
            for s in range(L):
                q = orden[r, s]
                ks = orden[r, lo[s]:s]
                if ks.size == 0:
                    senal[b, tau, q] = (0.0, PROHIBIDO, 0.0)
                    continue
                dphi = phi[b, ks].astype(np.float64) @ phi[b, q].astype(np.float64)
                dqk = Kc[b, ks].astype(np.float64) @ Qc[b, q].astype(np.float64)
                if half:
                    s1 = bf16(bf16(dphi.astype(np.float32)) / inv_t)
                    s2 = bf16(bf16(dqk.astype(np.float32)) * esc_c)
                    sc = bf16(s1 + s2)
                else:
                    sc = (dphi.astype(np.float32) / inv_t) + (dqk.astype(np.float32) * esc_c)
                ln = largo_seguido(np.broadcast_to(Pf[b, q], (ks.size, K)), Pf[b, ks])
                if want_detail:
                    detail['largo'][(r, s)] = ln
                sc = (sc + w_suf[ln]).astype(np.float32)
                sc = (sc + log_alfa[b, ks]).astype(np.float32)
                dt = (Bt[b, ks] - Bt[b, q]).astype(np.float32)
                sc = (sc + dt * tasa[tau]).astype(np.float32)
                mx = sc.max()
                e = np.exp((sc - mx).astype(np.float32)).astype(np.float32)
                att = (e / e.sum(dtype=np.float32)).astype(np.float32)
                vk = V[b, ks + 0]
                if half:
                    o = bf16((bf16(att).astype(np.float64) @ vk.astype(np.float64)).astype(np.float32))
                else:
                    o = (att.astype(np.float64) @ vk.astype(np.float64)).astype(np.float32)
                out_t[b, tau, q] = o
                senal[b, tau, q] = (1.0, mx, att.max())
    salida = out_t.sum(1, dtype=np.float32)
    if half:
        salida = bf16(salida)
    hay = senal[..., 0:1]
    mejor = np.where(hay > 0, senal[..., 1:2], PROHIBIDO).max(1)
    mejor = np.maximum(mejor, PROHIBIDO).astype(np.float32)
    acc = {'salida': salida, 'peso_total': hay.sum(1), 'mejor': mejor,
           'pico': (senal[..., 2:3] * hay).sum(1), 'peso_ctx': hay[:, T - lay.Tc:].sum(1), 'senal': senal,
           'phi': phi, 'V': V, 'ids': ids, 'orden': orden, 'ids_o': ids_o}
    if want_detail:
        acc['detail'] = detail
    return acc


def claves_de(sig, c, n):
    """asrn/nucleo.py:175-185: fp64 keys of the 1..n-token groups ending at t, summed in the order j = 0..n-1."""
    prev = anteriores(sig.astype(np.float64), n, desde=0)
    clave = np.zeros(prev.shape[:-1], np.float64)
    out = []
    for k in range(n):
        clave = clave + prev[..., k] * c[k]
        out.append(clave)
    return np.stack(out, -1)


def ordenar_claves(claves):
    """asrn/nucleo.py:693-701: per (b, n) row, stable argsort of the keys (NaN last) and repetido_i = key_i == key_{i-1}."""
    k = claves.transpose(0, 2, 1)
    orden = np.argsort(k, axis=-1, kind='stable')
    ks = np.take_along_axis(k, orden, -1)
    rep = np.zeros(ks.shape, bool)
    rep[..., 1:] = ks[..., 1:] == ks[..., :-1]
    return orden.astype(np.int32), rep


def escaneo(a, b):
    """asrn/nucleo.py:188-196 (S_i = a_i S_{i-1} + b_i along the last axis, S_{-1} = 0), sequential, accumulated in
    fp64 and returned as fp32."""
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    S = np.zeros_like(a64)
    acc = np.zeros(a64.shape[:-1])
    for i in range(a64.shape[-1]):
        acc = a64[..., i] * acc + b64[..., i]
        S[..., i] = acc
    return S.astype(np.float32)


def repeticion(lay, sig, beta, Bt, log_alfa):
    """asrn/estable.py:304-321: vistos (B, L, n), Hawkes intensity (B, L, n) and streak (B, L)."""
    n = lay.n
    kappa, kappa_r = lay.kappas()
    claves = claves_de(sig, lay['c_vistos'].astype(np.float64), n)
    orden, rep = ordenar_claves(claves)
    B, _, L = orden.shape
    vistos = np.zeros((B, n, L), bool)
    np.put_along_axis(vistos, orden, rep, -1)
    B_o = np.take_along_axis(np.broadcast_to(Bt[:, None, :], (B, n, L)), orden, -1)
    alfa_o = np.take_along_axis(np.broadcast_to(np.exp(log_alfa.astype(np.float32))[:, None, :], (B, n, L)), orden, -1)
    dB = np.zeros((B, n, L), np.float32)
    dB[..., 1:] = np.maximum(B_o[..., 1:] - B_o[..., :-1], 0).astype(np.float32)
    a = (rep * np.exp((-kappa[None, :, None] * dB).astype(np.float32))).astype(np.float32)
    alfa_prev = np.zeros((B, n, L), np.float32)
    alfa_prev[..., 1:] = alfa_o[..., :-1]
    lam = escaneo(a, (a * alfa_prev).astype(np.float32))
    hawkes = np.zeros_like(lam)
    np.put_along_axis(hawkes, orden, lam, -1)
    r = vistos[:, -1].astype(np.float32)
    racha = escaneo((r * np.exp((-kappa_r * beta.astype(np.float32)).astype(np.float32))).astype(np.float32), r)
    return {'vistos': vistos.transpose(0, 2, 1).astype(np.float32), 'hawkes': hawkes.transpose(0, 2, 1),
            'racha': racha, 'claves': claves, 'orden_ng': orden, 'repetido': rep}


def respuesta_racha(lay, racha):
    """asrn/nucleo.py:865-878: piecewise-linear response on log1p(racha) / paso, flat past the last node."""
    d_racha = lay['d_racha'].astype(np.float32)
    u_racha = np.cumsum(d_racha, dtype=np.float32)
    nodes = d_racha.shape[0]
    x = np.minimum((np.log1p(racha.astype(np.float32)) / np.float32(lay.racha_paso)).astype(np.float32),
                   np.float32(nodes - 1))
    i = np.clip(np.floor(np.nan_to_num(x, nan=0.0)), 0, nodes - 2).astype(np.int64)
    return (u_racha[i] + (x - i.astype(np.float32)) * d_racha[1:][i]).astype(np.float32)


def combinar(lay, acc, h, half):
    """asrn/estable.py:376-403: gate logit in fp32 and h' = h + sigmoid(logit) * o(salida / tables with candidates)."""
    pt = acc['peso_total'].astype(np.float32)
    salida = (acc['salida'].astype(np.float32) / np.maximum(pt, 1)).astype(np.float32)
    mejor = np.where(pt > 0, acc['mejor'], 0).astype(np.float32)
    if lay.mejor_max is not None:
        mejor = np.clip(mejor, -lay.mejor_max, lay.mejor_max).astype(np.float32)
    senales = np.concatenate([pt / np.float32(lay.T), mejor, acc['pico'] / np.maximum(pt, 1),
                              acc['peso_ctx'] / np.float32(lay.Tc)], -1).astype(np.float32)
    logit = linear(h, lay['g.weight'], lay['g.bias'])
    logit = (logit + linear(senales, lay['g_conf.weight'], lay['g_conf.bias'], half)).astype(np.float32)
    logit = (logit + (acc['vistos'] * lay['w_vistos']).sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    hk = np.log1p(acc['hawkes'].astype(np.float32)).astype(np.float32)
    logit = (logit + (hk * lay['u_hawkes']).sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    logit = (logit + respuesta_racha(lay, acc['racha'])[..., None]).astype(np.float32)
    if lay.tope_puerta is not None:
        c = np.float32(lay.tope_puerta)
        logit = (c * np.tanh(logit / c)).astype(np.float32)
    aporte = linear(salida, lay['o.weight'], None, half)
    gate = (1.0 / (1.0 + np.exp(-logit.astype(np.float64)))).astype(np.float32)
    if half:
        return (h + bf16(bf16(gate) * aporte)).astype(np.float32)
    return (h + gate * aporte).astype(np.float32)


def layer_forward(lay, E, h, tokens, half=False, return_parts=False, ids_override=None):
    """asrn/estable.py:407-421: h' = layer(E, h, tokens). ids_override (B, L, T): bucket ids to use instead of the
    ones of this restatement's own phi (to compare a pipeline conditioned on its own bucket ids)."""
    sig = firmas_de_piezas(tokens)
    Qc, Kc, beta, log_alfa = contexto(lay, h, half)
    Bt = np.cumsum(beta, axis=1)
    acc = acumular(lay, E, Qc, Kc, Bt, log_alfa, sig, half, ids_override=ids_override)
    rep = repeticion(lay, sig, beta, Bt, log_alfa)
    acc.update(rep)
    out = combinar(lay, acc, h, half)
    if return_parts:
        acc.update(Qc=Qc, Kc=Kc, beta=beta, log_alfa=log_alfa, Bt=Bt, sig=sig, out=out)
        return acc
    return out


# --------------------------------------------------------------------------------------------------------------------
# Vectorised restatement (the reference's window formulation), for timing the CPU path on realistic sizes
# --------------------------------------------------------------------------------------------------------------------

def acumular_fast(lay, E, Qc, Kc, Bt, log_alfa, sig, half, ids_override=None):
    """asrn/estable.py:204-272 as the reference computes it on the CPU: every row sorted by bucket, cut into blocks of
    C with a zero block in front, windows (W, C, 2C) of the previous + current block, batched products, exact-mask
    softmax, copy of the next token's value, back to text order and summed over the tables. ids_override (B, L, T):
    bucket ids to use instead of this restatement's own."""
    B, L, d = E.shape
    T, C, K = lay.T, lay.C, lay.K
    n_pad = (-L) % C
    R = (L + n_pad) // C + 1
    BT = B * T
    phi, V = phi_y_valores(lay, E, half)
    ids = ids_de(phi, T, lay.nb) if ids_override is None else np.asarray(ids_override, np.int32)
    rows = ids.transpose(0, 2, 1).reshape(BT, L)
    orden = np.argsort(rows, axis=-1, kind='stable')
    nulo = B * L
    fuente = np.full((BT, R * C), nulo, np.int64)
    fuente[:, C:C + L] = orden + np.repeat(np.arange(0, nulo, L), T)[:, None]
    real = fuente != nulo
    ids_o = np.full((BT, R * C), -1, np.int64)
    ids_o[:, C:C + L] = np.take_along_axis(rows, orden, -1)

    def ordenar(x):
        k = x.shape[-1]
        return np.concatenate([x.reshape(nulo, k), np.zeros((1, k), x.dtype)])[fuente.reshape(-1)].reshape(BT, -1, k)

    def preguntas(x):
        return x.reshape(BT * R, C, *x.shape[2:])[1:]

    def llaves(x):
        flat = x.reshape(BT * R * C, *x.shape[2:])
        w = np.lib.stride_tricks.sliding_window_view(flat, 2 * C, axis=0)[::C]
        return np.moveaxis(w, -1, 1)

    phi_o, V_o = ordenar(phi), ordenar(V)
    Qc_o, Kc_o, Pf_o = ordenar(Qc), ordenar(Kc), ordenar(anteriores(sig, K))
    s1 = np.matmul(preguntas(phi_o), llaves(phi_o).transpose(0, 2, 1))
    s2 = np.matmul(preguntas(Qc_o), llaves(Kc_o).transpose(0, 2, 1))
    if half:
        sc = bf16(bf16(bf16(s1) / np.float32(lay.temperatura)) + bf16(bf16(s2) * np.float32(lay.cf ** -0.5)))
    else:
        sc = (s1 / np.float32(lay.temperatura) + s2 * np.float32(lay.cf ** -0.5)).astype(np.float32)
    ln = largo_seguido(preguntas(Pf_o)[:, :, None, :], llaves(Pf_o)[:, None, :, :])
    sc = (sc + lay['w_sufijo'].astype(np.float32)[ln]).astype(np.float32)
    tasa = np.tile(lay['gamma'].astype(np.float32) / np.float32(C), B)
    B_o = ordenar(Bt[..., None])[..., 0]
    la_o = ordenar(log_alfa[..., None])[..., 0]
    tasa_w = preguntas(np.broadcast_to(tasa[:, None], (BT, R * C)).copy())[:, 0]
    dt = (llaves(B_o)[:, None, :] - preguntas(B_o)[:, :, None]).astype(np.float32)
    sc = (sc + llaves(la_o)[:, None, :]).astype(np.float32)
    sc = (sc + dt * tasa_w[:, None, None]).astype(np.float32)
    i = np.arange(C)[:, None]
    j = np.arange(2 * C)
    ant = (j >= i) & (j < C + i)
    valido = (preguntas(ids_o)[:, :, None] == llaves(ids_o)[:, None, :]) & llaves(real)[:, None, :] & ant
    hay = valido.any(-1, keepdims=True)
    mx = np.where(valido, sc, -np.inf).max(-1, keepdims=True)
    ref = np.where(hay, mx, 0).astype(np.float32)
    with np.errstate(invalid='ignore', over='ignore'):
        e = np.where(valido, np.exp((sc - ref).astype(np.float32)), 0).astype(np.float32)
    att = (e / np.where(hay, e.sum(-1, keepdims=True, dtype=np.float32), 1)).astype(np.float32)
    Vk = llaves(V_o)
    if half:
        out = bf16(np.matmul(bf16(att), Vk))
    else:
        out = np.matmul(att, Vk).astype(np.float32)
    en_orden = np.empty_like(orden)
    np.put_along_axis(en_orden, orden, np.arange(L)[None, :].repeat(BT, 0), 1)
    fila = (en_orden + np.arange(0, BT * R * C, R * C)[:, None]).reshape(-1)
    salida = out.reshape(-1, d)[fila].reshape(B, T, L, d).sum(1, dtype=np.float32)
    if half:
        salida = bf16(salida)
    mxs = np.where(hay, mx, PROHIBIDO).astype(np.float32)
    pk = att.max(-1, keepdims=True)
    sen = np.concatenate([hay.astype(np.float32), mxs, pk], -1).reshape(-1, 3)[fila].reshape(B, T, L, 3)
    hay_t = sen[..., 0:1]
    mejor = np.maximum(np.where(hay_t > 0, sen[..., 1:2], PROHIBIDO).max(1), PROHIBIDO).astype(np.float32)
    return {'salida': salida, 'peso_total': hay_t.sum(1), 'mejor': mejor, 'pico': (sen[..., 2:3] * hay_t).sum(1),
            'peso_ctx': hay_t[:, T - lay.Tc:].sum(1), 'senal': sen, 'phi': phi, 'ids': ids,
            'orden': orden.astype(np.int32)}


def layer_forward_fast(lay, E, h, tokens, half=False, return_parts=False, ids_override=None):
    """layer_forward with the vectorised scoring (same results up to fp32 summation order)."""
    sig = firmas_de_piezas(tokens)
    Qc, Kc, beta, log_alfa = contexto(lay, h, half)
    Bt = np.cumsum(beta, axis=1)
    acc = acumular_fast(lay, E, Qc, Kc, Bt, log_alfa, sig, half, ids_override=ids_override)
    acc.update(repeticion(lay, sig, beta, Bt, log_alfa))
    out = combinar(lay, acc, h, half)
    if return_parts:
        acc.update(Qc=Qc, Kc=Kc, beta=beta, log_alfa=log_alfa, Bt=Bt, sig=sig, out=out)
        return acc
    return out
