"""Torch-facing calls of each stage of the layer forward (the C ABI's stage entry points), one per reference seam:

    context       CapaASRNEstable._contexto + firmas_de_piezas          asrn/estable.py:153-194, asrn/nucleo.py:161-164
    clock         Bt = beta.cumsum(1)                                    asrn/estable.py:418
    hash          _phi_y_valores + _ids (values: rows of Ea)             asrn/nucleo.py:644-664
    ids_from_phi  _ids                                                   asrn/nucleo.py:661-664
    bucket_sort   ids.argsort(dim=-1, stable=True)                       asrn/estable.py:220-221
    candidates    the candidate window + suffix lengths (verification)   asrn/estable.py:232-265
    score         _acumular after the projection                        asrn/estable.py:204-300
    repetition    _repeticion (+ keys / n-gram order / repeated flags)   asrn/estable.py:304-321
    gate          _combinar                                              asrn/estable.py:376-403

All tensors are CUDA tensors; every call runs on the current stream.
"""
import torch

from . import _lib
from .layer import ctypes_ref

_ACT = {True: torch.bfloat16, False: torch.float32}


def _L():
    return _lib.lib()


def _s(dev):
    return _lib.stream_ptr(dev)


def _p(t):
    return _lib.ptr(t)


def _cfg(layer, B, L, half):
    return _lib.make_config(layer, B, L, half)


def context(layer, h, piezas=None, E=None, half=False):
    B, L, d = h.shape
    dev = h.device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _cfg(layer, B, L, half)
    cf = layer.confirmar
    out = dict(Qc=torch.empty(B, L, cf, dtype=_ACT[half], device=dev),
               Kc=torch.empty(B, L, cf, dtype=_ACT[half], device=dev),
               beta=torch.empty(B, L, dtype=torch.float64, device=dev),
               log_alfa=torch.empty(B, L, dtype=torch.float32, device=dev),
               glogit=torch.empty(B, L, dtype=torch.float32, device=dev),
               sig=torch.empty(B, L, dtype=torch.float32, device=dev))
    h = h.float().contiguous()
    tok = None if piezas is None else piezas.to(torch.int64).contiguous()
    Ec = None if E is None else E.float().contiguous()
    _lib.check(_L().asrn_context(ctypes_ref(cfg), ctypes_ref(w), _p(prep), _p(h), _p(Ec), _p(tok), _p(out['Qc']),
                                 _p(out['Kc']), _p(out['beta']), _p(out['log_alfa']), _p(out['glogit']),
                                 _p(out['sig']), _s(dev)), 'asrn_context')
    return out


def clock(beta):
    beta = beta.to(torch.float64).contiguous()
    Bt = torch.empty_like(beta)
    B, L = beta.shape
    _lib.check(_L().asrn_clock(B, L, _p(beta), _p(Bt), _s(beta.device)), 'asrn_clock')
    return Bt


def hash(layer, E, half=False):
    B, L, d = E.shape
    dev = E.device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _cfg(layer, B, L, half)
    P = layer.n_tablas * layer.n_bits
    E = E.float().contiguous()
    Ea = torch.empty(B, L, d, dtype=torch.bfloat16, device=dev) if half else E
    phi = torch.empty(B, L, P, dtype=_ACT[half], device=dev)
    ids_rows = torch.empty(B * layer.n_tablas, L, dtype=torch.int16, device=dev)
    _lib.check(_L().asrn_hash(ctypes_ref(cfg), ctypes_ref(w), _p(prep), _p(E), _p(Ea), _p(phi), _p(ids_rows),
                              _s(dev)), 'asrn_hash')
    return dict(Ea=Ea, phi=phi, ids_rows=ids_rows)


def ids_from_phi(phi, T, nb):
    B, L, P = phi.shape
    phi = phi.float().contiguous()
    ids_rows = torch.empty(B * T, L, dtype=torch.int16, device=phi.device)
    _lib.check(_L().asrn_ids_from_phi(B, L, T, nb, _p(phi), _p(ids_rows), _s(phi.device)), 'asrn_ids_from_phi')
    return ids_rows


def ids_rows_to_btl(ids_rows, B, T):
    """(B*T, L) uint16 stored as int16 -> (B, L, T) int32 (the reference's _ids layout)."""
    x = ids_rows.to(torch.int32) & 0xFFFF
    return x.view(B, T, -1).transpose(1, 2).contiguous()


def bucket_sort(ids_rows, nb):
    """ids_rows (rows, L) int16 (uint16 bits) -> (orden int32, ids_o int16), both (rows, L)."""
    rows, L = ids_rows.shape
    dev = ids_rows.device
    ids_rows = ids_rows.contiguous()
    orden = torch.empty(rows, L, dtype=torch.int32, device=dev)
    ids_o = torch.empty(rows, L, dtype=torch.int16, device=dev)
    nbytes = _L().asrn_bucket_sort_workspace_bytes(rows, L, nb)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.check(_L().asrn_bucket_sort(rows, L, nb, _p(ids_rows), _p(orden), _p(ids_o), _p(ws), nbytes, _s(dev)),
               'asrn_bucket_sort')
    return orden, ids_o


def score(layer, orden, ids_o, phi, Qc, Kc, sig, Bt, log_alfa, Ea, half=False):
    B, L, _ = phi.shape
    dev = phi.device
    T, d = layer.n_tablas, layer.d
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _cfg(layer, B, L, half)
    act = _ACT[half]
    phi, Qc, Kc, Ea = (x.to(act).contiguous() for x in (phi, Qc, Kc, Ea))
    orden, ids_o = orden.to(torch.int32).contiguous(), ids_o.contiguous()
    sig, la = sig.float().contiguous(), log_alfa.float().contiguous()
    Bt = Bt.to(torch.float64).contiguous()
    acc = torch.zeros(B, L, d, dtype=act, device=dev)            # the compute type: bf16 accumulator under autocast
    hay = torch.empty(B, L, T, dtype=torch.uint8, device=dev)
    mx = torch.empty(B, L, T, dtype=torch.float32, device=dev)
    pk = torch.empty(B, L, T, dtype=torch.float32, device=dev)
    _lib.check(_L().asrn_score(ctypes_ref(cfg), ctypes_ref(w), _p(prep), _p(orden), _p(ids_o), _p(phi), _p(Qc), _p(Kc),
                               _p(sig), _p(Bt), _p(la), _p(Ea), _p(acc), _p(hay), _p(mx), _p(pk), _s(dev)),
               'asrn_score')
    return dict(acc=acc, hay=hay, mx=mx, pk=pk)


def candidates(orden, ids_o, sig, T, C, K):
    """(cand (rows, L, C) int32, suffix (rows, L, C) uint8): the scoring kernel's candidate windows."""
    rows, L = orden.shape
    B = rows // T
    dev = orden.device
    cand = torch.empty(rows, L, C, dtype=torch.int32, device=dev)
    suf = torch.empty(rows, L, C, dtype=torch.uint8, device=dev)
    _lib.check(_L().asrn_candidates(B, L, T, C, K, _p(orden.to(torch.int32).contiguous()), _p(ids_o.contiguous()),
                                    _p(sig.float().contiguous()), _p(cand), _p(suf), _s(dev)), 'asrn_candidates')
    return cand, suf


def repetition(layer, sig, beta, Bt, log_alfa, debug=False):
    B, L = sig.shape
    dev = sig.device
    n = layer.vistos
    w, _keep, prep = layer.prepared(dev, False)
    cfg = _cfg(layer, B, L, False)
    sig, la = sig.float().contiguous(), log_alfa.float().contiguous()
    beta, Bt = beta.to(torch.float64).contiguous(), Bt.to(torch.float64).contiguous()
    out = dict(vistos=torch.empty(B, L, n, dtype=torch.uint8, device=dev),
               hawkes=torch.empty(B, L, n, dtype=torch.float32, device=dev),
               racha=torch.empty(B, L, dtype=torch.float32, device=dev))
    if debug:
        out.update(keys=torch.empty(B, L, n, dtype=torch.float64, device=dev),
                   orden_ng=torch.empty(B, n, L, dtype=torch.int32, device=dev),
                   repetido=torch.empty(B, n, L, dtype=torch.uint8, device=dev))
    nbytes = _L().asrn_repetition_workspace_bytes(ctypes_ref(cfg))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.check(_L().asrn_repetition(ctypes_ref(cfg), ctypes_ref(w), _p(prep), _p(sig), _p(beta), _p(Bt), _p(la),
                                    _p(out['vistos']), _p(out['hawkes']), _p(out['racha']), _p(out.get('keys')),
                                    _p(out.get('orden_ng')), _p(out.get('repetido')), _p(ws), nbytes, _s(dev)),
               'asrn_repetition')
    return out


def gate(layer, h, glogit, acc, hay, mx, pk, vistos, hawkes, racha, half=False):
    B, L, d = h.shape
    dev = h.device
    w, _keep, prep = layer.prepared(dev, half)
    cfg = _cfg(layer, B, L, half)
    h = h.float().contiguous()
    out = torch.empty_like(h)
    acc = acc.to(_ACT[half])                                    # the compute type (as score leaves it)
    args = [x.contiguous() for x in (glogit, acc, hay, mx, pk, vistos, hawkes, racha)]
    nbytes = _L().asrn_gate_workspace_bytes(ctypes_ref(cfg))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.check(_L().asrn_gate(ctypes_ref(cfg), ctypes_ref(w), _p(prep), _p(h), *[_p(x) for x in args], _p(out),
                              _p(ws), nbytes, _s(dev)), 'asrn_gate')
    return out
