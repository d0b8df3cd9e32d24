"""The ASRN language model around the layer: embedding -> local blocks with an ASRN layer after every `largo_cada`
blocks -> ln_f -> tied head. Mirror of asrn.nucleo.ModeloASRN / BloqueLocal / crear_modelo
(asrn/nucleo.py:969-1119) with the same module names (state_dict compatible) and initialisation order.

The ASRN layers are asrn_b200.ASRNLayer (CUDA kernels of libasrn_b200.so). Under bf16 autocast on CUDA each local
block runs as the fused asrn_local_block (an LN kernel and three persistent tcgen05 GEMMs with the conv, GELU, bias and
residual folded in); in fp32 the local blocks, and in every mode the embedding and head, are PyTorch ops.
"""
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer import ASRNLayer


def firmas_de_piezas(piezas):
    """Token id -> fp32 signature (asrn/nucleo.py:161-164)."""
    return piezas.to(torch.float32)


class BloqueLocal(nn.Module):
    """Causal local context: dense convolution over the k-1 previous tokens and the current one, then an MLP
    (asrn/nucleo.py:969-1014, the default mezcla='conv')."""

    def __init__(self, d, k=4, ff=128, dropout=0.0, mezcla='conv', memoria_max=1024):
        super().__init__()
        if mezcla != 'conv':
            raise NotImplementedError("asrn_b200 builds the default local block (mezcla='conv')")
        self.k, self.mezcla = k, mezcla
        self.ln1 = nn.LayerNorm(d)
        self.conv = nn.Conv1d(d, d, k)
        self.ln2 = nn.LayerNorm(d)
        self.ff = nn.Sequential(nn.Linear(d, ff), nn.GELU(), nn.Linear(ff, d))
        self.drop = nn.Dropout(dropout)

    def forward(self, h):
        if self._fused_ok(h):
            return self._fused(h)
        z = self.ln1(h)
        c = F.gelu(self.conv(F.pad(z.transpose(1, 2), (self.k - 1, 0))).transpose(1, 2))
        h = h + self.drop(c)
        return h + self.drop(self.ff(self.ln2(h)))

    def _fused_ok(self, h):
        """The fused CUDA block (asrn_local_block) serves bf16 autocast on CUDA, fp32 h, no dropout at work, and the
        widths its tiles take; the fp32 model keeps PyTorch's exact fp32 ops."""
        if not (h.is_cuda and h.dtype == torch.float32 and h.dim() == 3 and torch.is_autocast_enabled('cuda')
                and torch.get_autocast_dtype('cuda') == torch.bfloat16):
            return False
        if self.training and self.drop.p > 0:
            return False
        d, ff = self.conv.in_channels, self.ff[0].out_features
        return d % 128 == 0 and d <= 1024 and ff % 128 == 0 and self.k <= 16 and not torch.is_grad_enabled()

    def _fused_weights(self, dev):
        """bf16 copies autocast would make, the conv as a (d, k d) matrix [o][j d + c] (cached per weight version)."""
        ver = tuple((p.data_ptr(), p._version) for p in self.parameters())
        hit = getattr(self, '_fused_cache', None)
        if hit is not None and hit[0] == ver and hit[1] == str(dev):
            return hit[2]
        d = self.conv.in_channels
        w = {'conv': self.conv.weight.detach().permute(0, 2, 1).reshape(d, self.k * d).to(dev, torch.bfloat16)
                                                            .contiguous(),
             'w1': self.ff[0].weight.detach().to(dev, torch.bfloat16).contiguous(),
             'w2': self.ff[2].weight.detach().to(dev, torch.bfloat16).contiguous()}
        for name, t in (('ln1_w', self.ln1.weight), ('ln1_b', self.ln1.bias), ('bc', self.conv.bias),
                        ('ln2_w', self.ln2.weight), ('ln2_b', self.ln2.bias), ('b1', self.ff[0].bias),
                        ('b2', self.ff[2].bias)):
            w[name] = t.detach().to(dev, torch.float32).contiguous()
        self._fused_cache = (ver, str(dev), w)
        return w

    def _fused(self, h):
        from . import _lib
        h = h.contiguous()
        B, L, d = h.shape
        ff = self.ff[0].out_features
        w = self._fused_weights(h.device)
        L_ = _lib.lib()
        nbytes = L_.asrn_local_block_workspace_bytes(B, L, d, ff)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=h.device)
        out = torch.empty_like(h)
        P = _lib.ptr
        _lib.check(L_.asrn_local_block(B, L, d, self.k, ff, P(h), P(out), P(w['ln1_w']), P(w['ln1_b']), self.ln1.eps,
                                       P(w['conv']), P(w['bc']), P(w['ln2_w']), P(w['ln2_b']), self.ln2.eps,
                                       P(w['w1']), P(w['b1']), P(w['w2']), P(w['b2']), P(ws), nbytes, None,
                                       _lib.stream_ptr(h.device)), 'asrn_local_block')
        return out


LocalBlock = BloqueLocal


def _escalar_profundo(modulo, n_capas):
    """Deep-model start (asrn/nucleo.py:1035-1044): outputs added to the state shrink by 1/sqrt(2 n_capas)."""
    f = 1.0 / (2 * n_capas) ** 0.5
    if isinstance(modulo, BloqueLocal):
        modulo.conv.weight.mul_(f)
        modulo.ff[2].weight.mul_(f)
    else:
        modulo.o.weight.mul_(f)


class ModeloASRN(nn.Module):
    """Same arguments and module names as the reference model (asrn/nucleo.py:1054-1078)."""

    def __init__(self, V, d=64, n_capas=2, largo_cada=2, ff=None, k=4, init_profundo=None, checkpoint=False,
                 dropout=0.0, mezcla='conv', memoria_max=1024, protecciones=None, **opciones_capa):
        super().__init__()
        assert n_capas >= 2 and largo_cada >= 1
        assert V <= 2 ** 24, 'token signatures are exact up to 2**24 tokens'
        self.config = dict(V=V, d=d, n_capas=n_capas, largo_cada=largo_cada, ff=ff or 2 * d, k=k, dropout=dropout,
                           mezcla=mezcla, memoria_max=memoria_max, opciones_capa=dict(opciones_capa))
        self.n_capas, self.checkpoint = n_capas, checkpoint
        self.init_profundo = n_capas >= 8 if init_profundo is None else bool(init_profundo)
        self.pos_largo = [i for i in range(n_capas - 1) if i % largo_cada == 0]
        self.emb = nn.Embedding(V, d)
        nn.init.normal_(self.emb.weight, std=0.02)
        self.ln_f = nn.LayerNorm(d)
        self.head = nn.Linear(d, V, bias=False)
        self.head.weight = self.emb.weight
        self.bloques = nn.ModuleList([BloqueLocal(d, k, ff or 2 * d, dropout, mezcla, memoria_max)
                                      for _ in range(n_capas)])
        self.largos = nn.ModuleList([ASRNLayer(d, protecciones, dropout=dropout, **opciones_capa)
                                     for _ in self.pos_largo])
        if self.init_profundo:
            with torch.no_grad():
                for b in self.bloques:
                    _escalar_profundo(b, n_capas)
                for c in self.largos:
                    _escalar_profundo(c, n_capas)

    def forward(self, x):
        if self.emb.weight.dtype in (torch.float16, torch.bfloat16):
            raise ValueError(f'the model has {self.emb.weight.dtype} weights: ASRN needs float32 weights; use '
                             'torch.autocast for bf16 (asrn/nucleo.py:1025-1032)')
        E = self.emb(x)
        # the n-gram sort depends only on the tokens and on c_vistos: made once for every ASRN layer (the reference
        # repeats it in each one; docs/ARCHITECTURE.md:525, asrn/nucleo.py:1088-1103)
        ng = self.largos[0].ngram_sort(x) if x.is_cuda and len(self.largos) > 1 and self._ngram_shared() else None
        h, j = E, 0
        for i, blq in enumerate(self.bloques):
            h = blq(h)
            if i in self.pos_largo:
                h = self.largos[j](E, h, x, ngram=ng)
                j += 1
        return self.head(self.ln_f(h))

    def _ngram_shared(self):
        """True when every ASRN layer has the same n-gram orders and c_vistos (checked again after a change)."""
        key = tuple((c.vistos, c.c_vistos.data_ptr(), c.c_vistos._version) for c in self.largos)
        if getattr(self, '_ng_key', None) != key:
            c0 = self.largos[0]
            self._ng_ok = all(c.vistos == c0.vistos and torch.equal(c.c_vistos.cpu(), c0.c_vistos.cpu())
                              for c in self.largos)
            self._ng_key = key
        return self._ng_ok

    def num_parametros(self):
        return sum(p.numel() for p in self.parameters())


ASRNModel = ModeloASRN


def crear_modelo(V, d=64, n_capas=2, largo_cada=2, semilla=None, protecciones=None, **kw):
    """asrn.create_model (asrn/__init__.py:60-64 -> asrn/nucleo.py:1114-1119): the model with the stable layer;
    semilla fixes torch's RNG right before construction, so the weights equal the reference's for that seed."""
    if semilla is not None:
        torch.manual_seed(semilla)
    return ModeloASRN(V, d, n_capas, largo_cada, protecciones=protecciones, **kw)


create_model = crear_modelo


# ---- model files (the reference's format: asrn/nucleo.py:2050-2133) --------------------------------------------------
# A file holds {'config': model.config, 'pesos': state_dict} as torch.save wrote it; the parameter names are the
# reference's, so files written by the reference's guardar() / entrenar() load here and the other way round.

_NEW_IN_V87 = ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha')


def guardar(modelo, archivo):
    """Write the model's configuration and weights (asrn/nucleo.py:2068-2074); written to a temporary file, flushed to
    disk and renamed, so an interrupted write leaves the previous file intact."""
    import os
    carpeta = os.path.dirname(os.path.abspath(archivo))
    os.makedirs(carpeta, exist_ok=True)
    tmp = archivo + '.tmp'
    estado = {k: v.detach().cpu() for k, v in modelo.state_dict().items()}
    try:
        with open(tmp, 'wb') as f:
            torch.save({'config': modelo.config, 'pesos': estado}, f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, archivo)
    except BaseException:
        if os.path.exists(tmp):
            os.remove(tmp)
        raise


def _migrate_streak(pesos):
    """Files of the reference's v86 stored the streak response per node ('u_racha'); v87 stores its increments
    ('d_racha'): d = [u_0, u_1 - u_0, ...], an exact conversion (asrn/nucleo.py:2096-2107)."""
    viejos = [n for n in pesos if n.rsplit('.', 1)[-1] == 'u_racha']
    if not viejos:
        return pesos
    pesos = dict(pesos)
    for n in viejos:
        u = pesos.pop(n)
        pesos[n[:-len('u_racha')] + 'd_racha'] = torch.cat([u[:1], u[1:] - u[:-1]])
    return pesos


def cargar(archivo, dispositivo=None, confiar=False, protecciones=None):
    """Load a model written by guardar() here or by the reference's guardar() / entrenar() (its v83 to v89 files;
    asrn/nucleo.py:2110-2133, asrn/__init__.py:73-75). Read with torch.load(weights_only=True) unless confiar=True.
    Weights missing from files older than v87 keep their initial (neutral) values, as the reference does; any other
    missing or unexpected weight is an error. Returns the model on `dispositivo` (default: cuda) in eval mode."""
    import os
    if not os.path.isfile(archivo):
        raise FileNotFoundError(f'no such file: {archivo}')
    try:
        r = torch.load(archivo, map_location='cpu', weights_only=True)
    except Exception as e:
        if not confiar:
            raise ValueError(f'{archivo}: could not be read in safe mode ({type(e).__name__}); pass confiar=True for a '
                             'file of your own') from e
        r = torch.load(archivo, map_location='cpu', weights_only=False)
    if not isinstance(r, dict) or 'config' not in r or 'pesos' not in r:
        raise ValueError(f'{archivo}: not a model written by guardar() / entrenar() of ASRN')
    c = dict(r['config'])
    m = ModeloASRN(c['V'], c['d'], c['n_capas'], c['largo_cada'], c['ff'], c['k'], init_profundo=False,
                   dropout=c.get('dropout', 0.0), mezcla=c.get('mezcla', 'conv'), memoria_max=c.get('memoria_max', 1024),
                   protecciones=protecciones, **c['opciones_capa'])
    faltan, sobran = m.load_state_dict(_migrate_streak(r['pesos']), strict=False)
    raros = [n for n in faltan if n.rsplit('.', 1)[-1] not in _NEW_IN_V87]
    if sobran or raros:
        raise ValueError(f'weights that are not ASRN v83-v89 weights: missing {raros}, unexpected {list(sobran)}')
    return m.to(dispositivo or ('cuda' if torch.cuda.is_available() else 'cpu')).eval()


save = guardar
load = cargar
