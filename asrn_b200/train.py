"""Training on the device: the bucket attention with its backward and the linear-recurrence scan with its backward,
as autograd functions over the C-ABI kernels (asrn_bucket_attn_forward / _backward, asrn_scan_forward / _backward).

BucketAttention.apply takes what the reference's fused attention takes (asrn/nucleo.py:461-515, called by
asrn/estable.py:282-291): phi, V, Qc, Kc, the clock Bt, log_alfa, w_sufijo, gamma, the previous signatures Pf, the
bucket order and sorted ids of every (sequence, table) row, T, C and the two score scales; it returns the attention
output summed over the tables (B, L, d) and the per-table signals (B T, L, 3). Its backward recomputes the scores
(nothing of (windows, C, 2C) is stored) and fills per-slot buffers without atomics, added here in a fixed order
(asrn/nucleo.py:491-515). escaneo(a, b) is S_i = a_i S_{i-1} + b_i along the last dimension with the backward of
asrn/nucleo.py:518-537. Both run on CUDA only and raise elsewhere."""
import math

import torch

from . import _lib


def _p(t):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError('asrn_b200.train runs on CUDA tensors only')


def _clock_parts(Bt, Bt_bajo):
    """The clock as fp32 high and low parts: high = Bt in fp32, low = the rest of a 64-bit clock (asrn/estable.py:
    282-287), or the given low part, or zero for an fp32 clock."""
    hi = Bt.detach().float().contiguous()
    if Bt_bajo is not None:
        lo = Bt_bajo.detach().float().contiguous()
    elif Bt.dtype == torch.float64:
        lo = (Bt.detach() - hi.double()).float().contiguous()
    else:
        lo = torch.zeros_like(hi)
    return hi, lo


class BucketAttention(torch.autograd.Function):
    """Bucket attention of all tables, forward and backward on the device."""

    @staticmethod
    def forward(ctx, phi, V, Qc, Kc, Bt, log_alfa, w, gamma, Pf, orden, ids_o, T, C, escala_phi, escala_c,
                Bt_bajo=None):
        _need_cuda(phi, V, Qc, Kc, Bt, log_alfa, w, gamma, Pf, orden, ids_o)
        B, L, P = phi.shape
        D, CF, K = V.shape[-1], Qc.shape[-1], Pf.shape[-1]
        half = phi.dtype == torch.bfloat16
        act = torch.bfloat16 if half else torch.float32
        if any(x.dtype != act for x in (phi, V, Qc, Kc)):
            raise TypeError('phi, V, Qc and Kc must all be float32 or all bfloat16')
        ent = [x.contiguous() for x in (phi, Qc, Kc, V)]
        pf = Pf.detach().float().contiguous()
        hi, lo = _clock_parts(Bt, Bt_bajo)
        la = log_alfa.detach().float().contiguous()
        orden32 = orden.to(torch.int32).contiguous()
        ids32 = ids_o.to(torch.int32).contiguous()
        w32, g32 = w.detach().float().contiguous(), gamma.detach().float().contiguous()
        out = torch.empty(B * T, L, D, dtype=act, device=V.device)
        sen = torch.empty(B * T, L, 3, dtype=torch.float32, device=V.device)
        _lib.check(_lib.lib().asrn_bucket_attn_forward(
            B, L, T, C, P, CF, K, D, *[_p(x) for x in ent], _p(pf), _p(hi), _p(lo), _p(la), _p(orden32), _p(ids32),
            _p(w32), _p(g32), float(escala_phi), float(escala_c), int(half), _p(out), _p(sen),
            _lib.stream_ptr(V.device)), 'asrn_bucket_attn_forward')
        ctx.save_for_backward(*ent, pf, hi, lo, la, orden32, ids32, w32, g32)
        ctx.datos = (B, L, P, D, CF, K, T, C, float(escala_phi), float(escala_c), half,
                     [x.dtype for x in (phi, Qc, Kc, V, Bt, log_alfa)])
        ctx.mark_non_differentiable(sen)
        return out.view(B, T, L, D).sum(1), sen

    @staticmethod
    def backward(ctx, dsalida, _dsen):
        phi, Qc, Kc, V, pf, hi, lo, la, orden32, ids32, w32, g32 = ctx.saved_tensors
        B, L, P, D, CF, K, T, C, escala_phi, escala_c, half, tipos = ctx.datos
        BT, dev = B * T, V.device
        NB = (L + C - 1) // C
        act = V.dtype
        f32 = dict(dtype=torch.float32, device=dev)
        G = dict(phi_q=torch.empty(BT, L, P, dtype=act, device=dev), qc=torch.empty(BT, L, CF, dtype=act, device=dev),
                 b_q=torch.empty(BT, L, **f32), phi_k=torch.empty(2, BT, L, P, dtype=act, device=dev),
                 kc=torch.empty(2, BT, L, CF, dtype=act, device=dev), v=torch.empty(2, BT, L, D, dtype=act, device=dev),
                 la=torch.empty(2, BT, L, **f32), b_k=torch.empty(2, BT, L, **f32))
        partes = torch.empty(BT, NB, K + 2, **f32)
        dout = dsalida.to(act).contiguous()
        _lib.check(_lib.lib().asrn_bucket_attn_backward(
            B, L, T, C, P, CF, K, D, _p(phi), _p(Qc), _p(Kc), _p(V), _p(pf), _p(hi), _p(lo), _p(la), _p(orden32),
            _p(ids32), _p(w32), _p(g32), escala_phi, escala_c, int(half), _p(dout), _p(G['phi_q']), _p(G['qc']),
            _p(G['b_q']), _p(G['phi_k']), _p(G['kc']), _p(G['v']), _p(G['la']), _p(G['b_k']), _p(partes),
            _lib.stream_ptr(dev)), 'asrn_bucket_attn_backward')

        def sumar(q, k):               # the tables (and the two places of every key) -> (B, L, ...), in fp32
            total = k.view(2, B, T, *k.shape[2:]).sum((0, 2), dtype=torch.float32)
            return total if q is None else total + q.view(B, T, *q.shape[1:]).sum(1, dtype=torch.float32)
        per_table = partes.view(B, T, NB, K + 2).sum((0, 2))                        # (T, K + 2)
        tp, tq, tk, tv, tb, tl = tipos
        return (sumar(G['phi_q'], G['phi_k']).to(tp), sumar(None, G['v']).to(tv),
                G['qc'].view(B, T, L, CF).sum(1, dtype=torch.float32).to(tq), sumar(None, G['kc']).to(tk),
                sumar(G['b_q'], G['b_k']).to(tb), sumar(None, G['la']).to(tl), per_table[:, 1:].sum(0),
                per_table[:, 0] / C, None, None, None, None, None, None, None, None)


class _Scan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        S = _scan(a, b)
        ctx.save_for_backward(a, S)
        return S

    @staticmethod
    def backward(ctx, g):
        a, S = ctx.saved_tensors
        rows, L = a.numel() // a.shape[-1], a.shape[-1]
        g32 = g.float().contiguous()
        ga = torch.empty_like(a) if ctx.needs_input_grad[0] else None
        gb = torch.empty_like(a) if ctx.needs_input_grad[1] else None
        _lib.check(_lib.lib().asrn_scan_backward(rows, L, _p(a), _p(S), _p(g32), _p(ga), _p(gb),
                                                 _lib.stream_ptr(a.device)), 'asrn_scan_backward')
        return ga, gb


def _scan(a, b):
    rows, L = a.numel() // a.shape[-1], a.shape[-1]
    S = torch.empty_like(a)
    _lib.check(_lib.lib().asrn_scan_forward(rows, L, _p(a), _p(b), _p(S), _lib.stream_ptr(a.device)),
               'asrn_scan_forward')
    return S


def escaneo(a, b):
    """S_i = a_i S_{i-1} + b_i over the last dimension (S_{-1} = 0), fp32, with a gradient when a or b needs one
    (asrn/nucleo.py:188-197, 518-537)."""
    _need_cuda(a, b)
    a, b = torch.broadcast_tensors(a, b)
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise TypeError('escaneo takes float32 tensors')
    a, b = a.contiguous(), b.contiguous()
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad):
        return _Scan.apply(a, b)
    return _scan(a, b)


_FORBIDDEN = -1e9          # score of "not allowed" (asrn/nucleo.py:86)


class _Take(torch.autograd.Function):
    """w[i] for a short w (the streak response's nodes) read at every position: the backward adds each entry's
    positions by a one-hot reduction (deterministic; PyTorch's indexing backward sorts millions of indices into a
    few entries). The reference does the same with a reduction per entry (asrn/nucleo.py:136-158)."""

    @staticmethod
    def forward(ctx, w, i):
        ctx.save_for_backward(i)
        ctx.n = w.shape[0]
        return w[i]

    @staticmethod
    def backward(ctx, g):
        (i,) = ctx.saved_tensors
        one_hot = torch.nn.functional.one_hot(i.reshape(-1), ctx.n).to(torch.float32)
        return (one_hot * g.reshape(-1, 1).float()).sum(0).to(g.dtype), None


def layer_forward_train(layer, E, h, piezas=None):
    """Differentiable forward of an ASRNLayer (the reference's asrn/estable.py:407-421 with its default protections),
    used by ASRNLayer.forward when a gradient is wanted. The index work runs on this library's kernels without a
    gradient (bucket ids and their stable sort, asrn_bucket_sort; the n-gram keys, their order and repeats,
    asrn_repetition), the bucket attention and the two scans on the training kernels above (forward and backward),
    and the dense projections, LayerNorm and gate as PyTorch ops, as in the reference:
      context   LN(h); Qc, Kc = LN(h) W in the autocast type; the clock projection in fp32; beta = min(softplus, beta_max)
                in fp64, log_alfa = max(logsigmoid + ln 2, log_alfa_min); Bt = cumsum(beta)     (asrn/estable.py:153-194)
      hash      phi = [word MLP(E), context MLP([E, E_prev])], V = v(E) of the next position     (asrn/nucleo.py:644-659)
      attention BucketAttention over the per-table bucket order, then the table signals          (asrn/estable.py:282-300)
      memory    Hawkes intensities and the streak from the n-gram order (two scans)              (asrn/estable.py:304-321)
      gate      h + sigmoid(logit) o(salida / tables with candidates)                            (asrn/estable.py:376-403)"""
    import torch.nn.functional as F
    from . import stages
    _need_cuda(E, h)
    p = layer.protecciones
    B, L, d = E.shape
    T, nb, C, cf, K, n = layer.n_tablas, layer.n_bits, layer.chunk, layer.confirmar, layer.sufijo, layer.vistos
    dev = E.device
    auto = torch.is_autocast_enabled('cuda')
    act = torch.get_autocast_dtype('cuda') if auto else torch.float32
    if auto and act != torch.bfloat16:
        raise NotImplementedError('the training path supports fp32 and bf16 autocast')
    with torch.autocast('cuda', enabled=False):
        sig = piezas.to(torch.float32) if piezas is not None else E.float() @ layer.r_firma.float()
    # context
    hh32 = layer.ln_ctx(h)
    hh = hh32.to(act)
    y = F.linear(hh, torch.cat([layer.cq.weight, layer.ck.weight]))
    with torch.autocast('cuda', enabled=False):
        u = F.linear(hh32.float(), layer.w_reloj.float(), layer.b_reloj.float())
    beta = F.softplus(u[..., 0])
    log_alfa = F.logsigmoid(u[..., 1]) + math.log(2)
    if p.beta_max is not None:
        beta = beta.clamp(max=p.beta_max)
    if p.log_alfa_min is not None:
        log_alfa = log_alfa.clamp(min=p.log_alfa_min)
    beta = beta.double()
    Qc, Kc = y[..., :cf], y[..., cf:2 * cf]
    Bt = beta.cumsum(1)
    # hash and values
    E16 = E.to(act)
    pal = layer.afin_palabra
    yv = F.linear(E16, torch.cat([pal[0].weight, layer.v.weight]), F.pad(pal[0].bias, (0, d)))
    hp, vv = yv.split([pal[0].out_features, d], dim=-1)
    llave = torch.cat([E16, F.pad(E16, (0, 0, 1, 0))[:, :L]], dim=-1)
    phi = torch.cat([pal[2](pal[1](hp)), layer.afin_contexto(llave)], dim=-1)
    V = F.pad(vv, (0, 0, 0, 1))[:, 1:]
    phi, V, Qc, Kc = (t.to(act).contiguous() for t in (phi, V, Qc, Kc))
    with torch.no_grad():
        bits = (phi.detach().float().view(B, L, T, nb) > 0).to(torch.int32)
        ids = (bits * layer.pot.to(torch.int32)).sum(-1, dtype=torch.int32)                 # (B, L, T)
        ids_rows = ids.transpose(1, 2).reshape(B * T, L).to(torch.int16)
        orden, ids_o = stages.bucket_sort(ids_rows, nb)
        ids_o = ids_o.to(torch.int32) & 0xFFFF
        pad = torch.full((B, K), float('nan'), device=dev)
        prev = torch.cat([pad, sig.detach()], 1)
        Pf = torch.stack([prev[:, K - 1 - k:K - 1 - k + L] for k in range(K)], -1)         # t-1, ..., t-K
    salida, senal = BucketAttention.apply(phi, V, Qc, Kc, Bt, log_alfa, layer.w_sufijo, layer.gamma, Pf, orden,
                                          ids_o, T, C, 1.0 / layer.temperatura, cf ** -0.5)
    sen = senal.view(B, T, L, 3)
    hay_t, mx_t, pico_t = sen[..., 0:1], sen[..., 1:2], sen[..., 2:3]
    mejor = torch.where(hay_t > 0, mx_t, torch.full_like(mx_t, _FORBIDDEN)).amax(1).clamp(min=_FORBIDDEN)
    pt = hay_t.sum(1)
    pico = (pico_t * hay_t).sum(1)
    peso_ctx = hay_t[:, T - layer.tablas_contexto:].sum(1)
    # n-gram memory: Hawkes intensity per order and the streak
    with torch.no_grad():
        rep = stages.repetition(layer, sig.detach(), beta.detach(), Bt.detach(), log_alfa.detach(), debug=True)
        orden_ng = rep['orden_ng'].long()                                                  # (B, n, L)
        repetido = rep['repetido'].float()
        vistos = rep['vistos'].float()                                                    # (B, L, n)
    kappa, kappa_r = layer.log_kappa.exp(), layer.log_kappa_racha.exp()
    if p.kappa_min is not None:
        kappa, kappa_r = kappa.clamp(min=p.kappa_min), kappa_r.clamp(min=p.kappa_min)
    B_o = torch.gather(Bt.unsqueeze(1).expand(-1, n, -1), -1, orden_ng)
    alfa_o = torch.gather(log_alfa.exp().unsqueeze(1).expand(-1, n, -1), -1, orden_ng)
    dB = F.pad((B_o[..., 1:] - B_o[..., :-1]).clamp(min=0), (1, 0)).float()
    a = repetido * torch.exp(-kappa.float().unsqueeze(-1) * dB)
    lam = escaneo(a, a * F.pad(alfa_o[..., :-1].float(), (1, 0)))
    hawkes = torch.zeros_like(lam).scatter(-1, orden_ng, lam).transpose(1, 2)
    r = vistos[..., -1]
    racha = escaneo((r * torch.exp(-kappa_r.float() * beta.float())).contiguous(), r.contiguous())
    # gate
    pt_d = pt.detach()
    sal = salida / pt.clamp(min=1)
    mejor = torch.where(pt_d > 0, mejor, torch.zeros_like(pt_d))
    if p.mejor_max is not None:
        mejor = mejor.clamp(-p.mejor_max, p.mejor_max)
    senales = torch.cat([pt_d / T, mejor, pico / pt_d.clamp(min=1), peso_ctx.detach() / layer.tablas_contexto], -1)
    with torch.autocast('cuda', enabled=False):
        logit = F.linear(h, layer.g.weight.to(h.dtype), layer.g.bias.to(h.dtype))
    logit = logit + layer.g_conf(senales).to(logit.dtype)
    logit = logit + (vistos.to(logit.dtype) * layer.w_vistos.to(logit.dtype)).sum(-1, keepdim=True)
    logit = logit + (torch.log1p(hawkes).to(logit.dtype) * layer.u_hawkes.to(logit.dtype)).sum(-1, keepdim=True)
    x = (torch.log1p(racha) / layer.racha_paso).clamp(max=layer.d_racha.shape[0] - 1)
    i = torch.nan_to_num(x.detach(), nan=0.0).floor().long().clamp(0, layer.d_racha.shape[0] - 2)
    resp = _Take.apply(layer.u_racha, i) + (x - i) * _Take.apply(layer.d_racha[1:], i)
    logit = logit + resp.unsqueeze(-1).to(logit.dtype)
    if p.tope_puerta is not None:
        logit = p.tope_puerta * torch.tanh(logit / p.tope_puerta)
    aporte = layer.o(sal.to(act))
    return h + torch.sigmoid(logit).to(aporte.dtype) * layer.drop(aporte)
