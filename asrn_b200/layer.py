"""ASRNLayer: the drop-in replacement of asrn.ASRNLayer (asrn.estable.CapaASRNEstable), forward on B200 kernels.

Parameters, buffers, their names, shapes and initialisation order are those of the reference
(asrn/nucleo.py:585-630, asrn/estable.py:147-149), so a reference state_dict loads unchanged and the same seed gives
the same weights. forward(E, h, piezas=None) -> h' has the reference's signature and semantics
(asrn/estable.py:407-421); it runs only on CUDA tensors, through libasrn_b200.so. bfloat16 autocast
(torch.autocast('cuda', dtype=torch.bfloat16)) selects the kernels' bf16 mode, which follows the reference's
autocast rounding chain; without autocast everything is fp32 (fp64 clock and n-gram keys).
"""
import dataclasses
import math

import torch
import torch.nn as nn

from . import _lib


@dataclasses.dataclass(frozen=True)
class Protecciones:
    """Numeric protections (asrn/estable.py:57-77). Protecciones() is group A, the reference's default."""
    mascara_exacta: bool = True
    reloj_64: bool = True
    beta_max: float = 1e4
    log_alfa_min: float = -30.0
    mejor_max: float = 1e4
    tope_puerta: float = None
    kappa_min: float = None

    @classmethod
    def ninguna(cls):
        return cls(mascara_exacta=False, reloj_64=False, beta_max=None, log_alfa_min=None, mejor_max=None)

    @classmethod
    def textos_largos(cls, largo_entrenamiento=1024):
        return cls(tope_puerta=10.0, kappa_min=1.0 / (4 * largo_entrenamiento))


Protections = Protecciones


def compute_half(device_type='cuda'):
    """True under bfloat16 autocast on CUDA; fp16 autocast is not implemented by these kernels."""
    if not torch.is_autocast_enabled(device_type):
        return False
    dt = torch.get_autocast_dtype(device_type)
    if dt == torch.bfloat16:
        return True
    raise NotImplementedError(f'asrn_b200 kernels implement fp32 and bfloat16 autocast, not {dt}')


class _LayerForward(torch.autograd.Function):
    """The fused inference forward through the C ABI. It keeps no intermediates, so it has no backward: when a
    gradient is wanted ASRNLayer.forward takes the training path (asrn_b200.train.layer_forward_train) instead."""

    @staticmethod
    def forward(ctx, layer, E, h, piezas, half, ngram):
        return layer._run(E, h, piezas, half, ngram)

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError('the fused forward has no backward; ASRNLayer.forward uses the training path when '
                                  'a gradient is wanted')


class ASRNLayer(nn.Module):
    """Same arguments as the reference layer (asrn/estable.py:147, asrn/nucleo.py:585-586)."""

    def __init__(self, d, protecciones=None, n_tablas=8, n_bits=14, afin_oculto=128, chunk=32, tablas_contexto=4,
                 confirmar=16, sufijo=4, vistos=4, dropout=0.0, nodos_racha=16, racha_max=256):
        super().__init__()
        assert 0 < tablas_contexto < n_tablas and nodos_racha >= 2
        self.d = d
        self.n_tablas, self.n_bits, self.chunk = n_tablas, n_bits, chunk
        self.tablas_contexto, self.confirmar, self.sufijo, self.vistos = tablas_contexto, confirmar, sufijo, vistos
        mitad = max(8, afin_oculto // 2)
        # module creation order fixes the RNG draws: the same as the reference
        self.afin_palabra = nn.Sequential(nn.Linear(d, mitad), nn.GELU(),
                                          nn.Linear(mitad, (n_tablas - tablas_contexto) * n_bits))
        self.afin_contexto = nn.Sequential(nn.Linear(2 * d, mitad), nn.GELU(),
                                           nn.Linear(mitad, tablas_contexto * n_bits))
        self.v = nn.Linear(d, d, bias=False)
        self.o = nn.Linear(d, d, bias=False)
        self.g = nn.Linear(d, 1)
        self.temperatura = (n_tablas * n_bits) ** 0.5
        self.register_buffer('pot', 2 ** torch.arange(n_bits))
        self.g_conf = nn.Linear(4, 1)
        nn.init.zeros_(self.g_conf.weight)
        nn.init.zeros_(self.g_conf.bias)
        self.cq = nn.Linear(d, confirmar, bias=False)
        nn.init.zeros_(self.cq.weight)
        self.ck = nn.Linear(d, confirmar, bias=False)
        self.ln_ctx = nn.LayerNorm(d)
        self.w_vistos = nn.Parameter(torch.zeros(vistos))
        g_v = torch.Generator().manual_seed(12345)
        self.register_buffer('c_vistos', torch.rand(vistos, generator=g_v, dtype=torch.float64) + 0.5)
        self.w_sufijo = nn.Parameter(torch.zeros(sufijo + 1))
        self.register_buffer('r_firma', torch.randn(d))
        self.drop = nn.Dropout(dropout)
        self.w_reloj = nn.Parameter(torch.zeros(2, d))
        self.b_reloj = nn.Parameter(torch.tensor([math.log(math.e - 1), 0.0]))
        self.gamma = nn.Parameter(torch.zeros(n_tablas))
        self.log_kappa = nn.Parameter(-torch.log(chunk * 4.0 ** torch.arange(vistos)))
        self.log_kappa_racha = nn.Parameter(torch.tensor([-math.log(8.0 * chunk)]))
        self.u_hawkes = nn.Parameter(torch.zeros(vistos))
        self.racha_paso = math.log1p(racha_max) / (nodos_racha - 1)
        self.d_racha = nn.Parameter(torch.zeros(nodos_racha))
        self.protecciones = protecciones or Protecciones()
        self._prepared = {}

    @property
    def u_racha(self):
        return self.d_racha.cumsum(0)

    # ---- device-side weights -------------------------------------------------------------------------------------

    def _check_protections(self):
        p = self.protecciones
        if not (p.mascara_exacta and p.reloj_64):
            raise NotImplementedError('asrn_b200 implements the default protections (exact mask, 64-bit clock); '
                                      'Protecciones.ninguna() is not available in this build')

    def _check_supported(self):
        self._check_protections()
        if self.training and self.drop.p > 0:
            raise NotImplementedError('dropout at training time runs on the training path only (a gradient wanted)')

    def _weights(self, device):
        """LayerWeights of the current parameters (contiguous device copies, cast to the reference's dtypes)."""
        named = dict(self.named_parameters())
        named.update(dict(self.named_buffers()))
        sd = {}
        for field, name in _lib.WEIGHT_NAMES.items():
            t = named[name].detach()
            sd[field] = t.to(device=device, dtype=torch.float64 if field == 'c_vistos' else torch.float32).contiguous()
        w = _lib.LayerWeights(**{f: sd[f].data_ptr() for f in _lib.WEIGHT_FIELDS})
        return w, sd

    def _version(self):
        return tuple((t.data_ptr(), t._version) for t in list(self.parameters()) + list(self.buffers()))

    def prepared(self, device, half):
        """(LayerWeights, tensors kept alive, prepared buffer) for this device and precision, cached until a
        parameter changes."""
        key = (str(device), bool(half))
        ver = self._version()
        hit = self._prepared.get(key)
        if hit is not None and hit[0] == ver:
            return hit[1]
        w, keep = self._weights(device)
        cfg = _lib.make_config(self, 1, 1, half)
        nbytes = _lib.lib().asrn_layer_prepared_bytes(ctypes_ref(cfg))
        if nbytes == 0:
            raise NotImplementedError('layer options not supported by libasrn_b200')
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _lib.check(_lib.lib().asrn_layer_prepare(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(buf), nbytes,
                                                 _lib.stream_ptr(device)), 'asrn_layer_prepare')
        val = (w, keep, buf)
        self._prepared[key] = (ver, val)
        return val

    # ---- forward -------------------------------------------------------------------------------------------------

    def forward(self, E, h, piezas=None, ngram=None):
        """E (B, L, d) token vectors, h (B, L, d) state, piezas (B, L) token ids (or None: signatures E . r_firma).
        Returns h' (B, L, d). ngram: the n-gram sort of piezas made by ngram_sort() (by this layer or another one with
        the same vistos and c_vistos); the layer then skips its own sort (the result is the same).
        When a gradient is wanted (grad enabled and E or h requiring one, or the layer training with parameters that
        do), the differentiable training path runs (asrn_b200.train.layer_forward_train: the bucket attention and
        scans on the training kernels, forward and backward); otherwise the fused inference forward."""
        if torch.is_grad_enabled() and (E.requires_grad or h.requires_grad or
                                        (self.training and any(q.requires_grad for q in self.parameters()))):
            from .train import layer_forward_train
            self._check_protections()
            if not (E.is_cuda and h.is_cuda):
                raise RuntimeError('asrn_b200.ASRNLayer runs on CUDA tensors only (there is no CPU implementation)')
            return layer_forward_train(self, E, h, piezas)
        half = compute_half(h.device.type) if h.is_cuda else False
        return _LayerForward.apply(self, E, h, piezas, half, ngram)

    def ngram_sort(self, piezas):
        """The n-gram sort of the token rows piezas (B, L) that every ASRN layer of a model repeats (its keys depend
        only on the tokens and on c_vistos, equal in every layer: asrn/nucleo.py:610, :691-701), made once on the
        device; pass it to forward(..., ngram=...)."""
        if not piezas.is_cuda:
            raise RuntimeError('asrn_b200: the n-gram sort runs on CUDA tensors only')
        B, L = piezas.shape
        dev = piezas.device
        tok = piezas.detach().to(torch.int64).contiguous()
        half = compute_half(dev.type)
        self._check_supported()
        w, _keep, prep = self.prepared(dev, half)
        cfg = _lib.make_config(self, B, L, half)
        L_ = _lib.lib()
        nbytes = L_.asrn_ngram_shared_bytes(ctypes_ref(cfg))
        buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        wsb = L_.asrn_repetition_workspace_bytes(ctypes_ref(cfg))
        ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
        if B * L:
            _lib.check(L_.asrn_ngram_shared_sort(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), _lib.ptr(tok),
                                                 _lib.ptr(buf), nbytes, _lib.ptr(ws), wsb, _lib.stream_ptr(dev)),
                       'asrn_ngram_shared_sort')
        return NgramSort(buf, nbytes, tok, self.vistos)

    def _run(self, E, h, piezas, half, ngram=None):
        self._check_supported()
        if not (E.is_cuda and h.is_cuda):
            raise RuntimeError('asrn_b200.ASRNLayer runs on CUDA tensors only (there is no CPU implementation)')
        if E.shape != h.shape or E.dim() != 3 or E.shape[-1] != self.d:
            raise ValueError(f'E and h must be (B, L, {self.d}); got {tuple(E.shape)} and {tuple(h.shape)}')
        dev = h.device
        B, L, _ = h.shape
        E32 = E.detach().to(torch.float32).contiguous()
        h32 = h.detach().to(torch.float32).contiguous()
        tok = None
        if piezas is not None:
            if piezas.shape != (B, L):
                raise ValueError(f'piezas must be (B, L) = ({B}, {L}); got {tuple(piezas.shape)}')
            tok = piezas.detach().to(device=dev, dtype=torch.int64).contiguous()
        out = torch.empty_like(h32)
        if B * L == 0:
            return out.to(h.dtype)
        w, _keep, prep = self.prepared(dev, half)
        cfg = _lib.make_config(self, B, L, half)
        L_ = _lib.lib()
        nbytes = L_.asrn_layer_workspace_bytes(ctypes_ref(cfg))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        if ngram is None:
            _lib.check(L_.asrn_layer_forward(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), _lib.ptr(E32),
                                             _lib.ptr(h32), _lib.ptr(tok), _lib.ptr(out), _lib.ptr(ws), nbytes,
                                             _lib.stream_ptr(dev)), 'asrn_layer_forward')
        else:
            if tok is None or ngram.vistos != self.vistos or ngram.tokens.shape != (B, L) or \
                    ngram.tokens.data_ptr() != tok.data_ptr() and not torch.equal(ngram.tokens, tok):
                raise ValueError('ngram: made for other tokens or another number of n-gram orders')
            _lib.check(L_.asrn_layer_forward_ngram(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), _lib.ptr(E32),
                                                   _lib.ptr(h32), _lib.ptr(tok), _lib.ptr(ngram.buf), ngram.nbytes,
                                                   _lib.ptr(out), _lib.ptr(ws), nbytes, _lib.stream_ptr(dev)),
                       'asrn_layer_forward_ngram')
        return out if h.dtype == torch.float32 else out.to(h.dtype)


class NgramSort:
    """The sorted n-gram keys and positions of a batch of token rows (ASRNLayer.ngram_sort), shared by the ASRN
    layers of a model forward."""

    def __init__(self, buf, nbytes, tokens, vistos):
        self.buf, self.nbytes, self.tokens, self.vistos = buf, nbytes, tokens, vistos


def ctypes_ref(x):
    import ctypes
    return ctypes.byref(x)


CapaASRNEstable = ASRNLayer
