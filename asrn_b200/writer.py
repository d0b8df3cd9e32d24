"""Incremental generation with the O(1) per-token writer: generate / escribir (asrn/nucleo.py:1965-2043).

Writer mirrors the reference's _Escritor in O(1) mode (asrn/nucleo.py:1717-1854): a prompt pass that runs the model and
keeps, per ASRN layer, the caches of every position (signature, clock, log_alfa, phi, Kc), the per-bucket rings of the
C most recent bucket mates and the n-gram Hawkes table; then one step per new token that touches only T x C candidates
per layer. The ASRN work of a step runs in the kernels of libasrn_b200.so (asrn_gen_*, plus the layer stages on the
new token); the local blocks, embedding and head are PyTorch ops. The rows of E (the values) are cached once, shared
by every layer.

generate() keeps the reference's sampling semantics (temperature, top_k, top_p, repetition penalty, no-repeat
n-grams, stop token, conserving the probability of continuing a quote), sampling on the host with the same seeded
generator, so greedy decoding (top_k=1) and seeded sampling give the reference's tokens.
"""
import ctypes

import torch
import torch.nn.functional as F

from . import _lib, stages
from .layer import compute_half, ctypes_ref


def _next_pow2(x):
    p = 1
    while p < x:
        p <<= 1
    return p


class _LayerState:
    pass


class Writer:
    """O(1) writer over an ASRNModel (asrn/nucleo.py:1717-1854)."""

    def __init__(self, modelo, memoria_de_lo_ajeno=True):
        self.m = modelo
        self.ajeno = memoria_de_lo_ajeno

    # ---- helpers --------------------------------------------------------------------------------------------------

    def _act(self):
        return torch.bfloat16 if self.half else torch.float32

    def _cfg(self, capa, B, L):
        return _lib.make_config(capa, B, L, self.half)

    @staticmethod
    def _grow(x, cap):
        y = x.new_zeros((x.shape[0], cap) + tuple(x.shape[2:]))
        y[:, :x.shape[1]] = x
        return y

    def _grow_all(self):
        cap = 2 * self.cap
        self.sig = self._grow(self.sig, cap)
        self.ea = self._grow(self.ea, cap)
        for st in self.layers:
            for name in ('phi', 'kc', 'bt', 'la'):
                setattr(st, name, self._grow(getattr(st, name), cap))
            if 2 * cap > st.hcap:
                raise NotImplementedError('the n-gram table was sized for the capacity given to inicio(); '
                                          'pass capacidad >= prompt + new tokens')
        self.cap = cap

    # ---- prompt ---------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def inicio(self, x0, capacidad=0):
        """Prompt pass (asrn/nucleo.py:1750-1794). x0 (B, L0) int64 on the model's device. Returns the logits of the
        last position (B, V)."""
        m = self.m
        self.half = compute_half(x0.device.type) if x0.is_cuda else False
        act = self._act()
        B, L0 = x0.shape
        dev = x0.device
        self.B, self.L0, self.t = B, L0, L0
        self.cap = max(L0 + 1, capacidad)
        E = m.emb(x0)
        d = E.shape[-1]
        self.sig = torch.zeros(B, self.cap, dtype=torch.float32, device=dev)
        self.sig[:, :L0] = x0.to(torch.float32)
        self.ea = torch.zeros(B, self.cap, d, dtype=act, device=dev)
        self.ea[:, :L0] = E.to(act)
        self.e_last = E[:, -1].clone()
        self.buf, self.layers = [], []
        h, j = E, 0
        for i, blq in enumerate(m.bloques):
            u = blq.ln1(h)
            self.buf.append(F.pad(u, (0, 0, blq.k - 1, 0))[:, u.shape[1]:])
            h = blq(h)
            if i in m.pos_largo:
                h = self._prompt_layer(m.largos[j], E, h, x0)
                j += 1
        return m.head(m.ln_f(h[:, -1:]))[:, -1]

    def _prompt_layer(self, capa, E, h, x0):
        B, L0 = x0.shape
        dev = x0.device
        half, act = self.half, self._act()
        T, nb, C, P = capa.n_tablas, capa.n_bits, capa.chunk, capa.n_tablas * capa.n_bits
        ctx = stages.context(capa, h, x0, half=half)
        Bt = stages.clock(ctx['beta'])
        hs = stages.hash(capa, E, half=half)
        orden, ids_o = stages.bucket_sort(hs['ids_rows'], nb)
        sc = stages.score(capa, orden, ids_o, hs['phi'], ctx['Qc'], ctx['Kc'], ctx['sig'], Bt, ctx['log_alfa'],
                          hs['Ea'], half=half)
        rep = stages.repetition(capa, ctx['sig'], ctx['beta'], Bt, ctx['log_alfa'])
        h_new = stages.gate(capa, h, ctx['glogit'], sc['acc'], sc['hay'], sc['mx'], sc['pk'], rep['vistos'],
                            rep['hawkes'], rep['racha'], half=half)
        st = _LayerState()
        st.capa = capa
        st.phi = torch.zeros(B, self.cap, P, dtype=act, device=dev)
        st.phi[:, :L0] = hs['phi']
        st.kc = torch.zeros(B, self.cap, capa.confirmar, dtype=act, device=dev)
        st.kc[:, :L0] = ctx['Kc']
        st.bt = torch.zeros(B, self.cap, dtype=torch.float64, device=dev)
        st.bt[:, :L0] = Bt
        st.la = torch.zeros(B, self.cap, dtype=torch.float32, device=dev)
        st.la[:, :L0] = ctx['log_alfa']
        st.racha = rep['racha'][:, -1].contiguous().clone()
        lib = _lib.lib()
        s = _lib.stream_ptr(dev)
        st.ring = torch.empty(B, T, 1 << nb, C, dtype=torch.int32, device=dev)
        st.count = torch.empty(B, T, 1 << nb, dtype=torch.int32, device=dev)
        n_valid = L0 - 1 if self.ajeno else L0
        _lib.check(lib.asrn_gen_ring_build(B, L0, T, nb, C, n_valid, _lib.ptr(orden), _lib.ptr(ids_o),
                                           _lib.ptr(st.ring), _lib.ptr(st.count), s), 'asrn_gen_ring_build')
        st.hcap = max(64, _next_pow2(2 * self.cap))
        st.table = torch.empty(lib.asrn_gen_hawkes_table_bytes(B, capa.vistos, st.hcap), dtype=torch.uint8,
                               device=dev)
        w, _keep, prep = capa.prepared(dev, half)
        cfg = self._cfg(capa, B, L0)
        _lib.check(lib.asrn_gen_hawkes_build(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), L0, self.cap,
                                             _lib.ptr(self.sig), _lib.ptr(st.bt), _lib.ptr(st.la),
                                             _lib.ptr(rep['hawkes'].contiguous()), _lib.ptr(st.table), st.hcap, s),
                   'asrn_gen_hawkes_build')
        self.layers.append(st)
        return h_new

    # ---- one token --------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def paso(self, pieza):
        """One new token per sequence, pieza (B,) (asrn/nucleo.py:1796-1854). Returns the logits (B, V)."""
        m = self.m
        if self.t >= self.cap:
            self._grow_all()
        t = self.t
        dev = self.sig.device
        act = self._act()
        pieza = pieza.view(-1).to(dev)
        B = pieza.shape[0]
        e_t = m.emb(pieza.view(-1, 1))                                       # (B, 1, d)
        self.sig[:, t] = pieza.to(torch.float32)
        self.ea[:, t] = e_t[:, 0].to(act)
        tok = pieza.view(B, 1)
        h, j = e_t, 0
        for i, blq in enumerate(m.bloques):
            ventana = torch.cat([self.buf[i], blq.ln1(h)], 1)
            z = blq.conv(ventana.transpose(1, 2)).transpose(1, 2)
            self.buf[i] = ventana[:, 1:]
            h = h + F.gelu(z)
            h = h + blq.ff(blq.ln2(h))
            if i in m.pos_largo:
                h = self._step_layer(self.layers[j], e_t, h, tok, t)
                j += 1
        self.e_last = e_t[:, 0]
        self.t += 1
        return m.head(m.ln_f(h))[:, -1]

    def _step_layer(self, st, e_t, h, tok, t):
        capa = st.capa
        half = self.half
        B = tok.shape[0]
        dev = tok.device
        T, nb, C, n = capa.n_tablas, capa.n_bits, capa.chunk, capa.vistos
        lib = _lib.lib()
        s = _lib.stream_ptr(dev)
        ctx = stages.context(capa, h, tok, half=half)
        st.bt[:, t] = st.bt[:, t - 1] + ctx['beta'][:, 0]
        st.la[:, t] = ctx['log_alfa'][:, 0]
        hs = stages.hash(capa, torch.stack([self.e_last, e_t[:, 0]], 1), half=half)
        phi_t = hs['phi'][:, 1].contiguous()
        ids_t = hs['ids_rows'].view(B, T, 2)[:, :, 1].contiguous()
        qc_t = ctx['Qc'][:, 0].contiguous()
        acc = torch.zeros(B, 1, capa.d, dtype=torch.float32, device=dev)
        hay = torch.empty(B, 1, T, dtype=torch.uint8, device=dev)
        mx = torch.empty(B, 1, T, dtype=torch.float32, device=dev)
        pk = torch.empty(B, 1, T, dtype=torch.float32, device=dev)
        w, _keep, prep = capa.prepared(dev, half)
        cfg = self._cfg(capa, B, 1)
        _lib.check(lib.asrn_gen_attend(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), t, self.cap, _lib.ptr(ids_t),
                                       _lib.ptr(phi_t), _lib.ptr(qc_t), _lib.ptr(st.ring), _lib.ptr(self.sig),
                                       _lib.ptr(st.bt), _lib.ptr(st.la), _lib.ptr(st.phi), _lib.ptr(st.kc),
                                       _lib.ptr(self.ea), _lib.ptr(acc), _lib.ptr(hay), _lib.ptr(mx), _lib.ptr(pk), s),
                   'asrn_gen_attend')
        vistos = torch.empty(B, 1, n, dtype=torch.uint8, device=dev)
        hawkes = torch.empty(B, 1, n, dtype=torch.float32, device=dev)
        racha = torch.empty(B, 1, dtype=torch.float32, device=dev)
        beta_t = ctx['beta'][:, 0].contiguous()
        la_t = ctx['log_alfa'][:, 0].contiguous()
        _lib.check(lib.asrn_gen_memory(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), t, self.cap, _lib.ptr(self.sig),
                                       _lib.ptr(st.bt), _lib.ptr(beta_t), _lib.ptr(la_t), _lib.ptr(st.table), st.hcap,
                                       _lib.ptr(st.racha), _lib.ptr(vistos), _lib.ptr(hawkes), _lib.ptr(racha), s),
                   'asrn_gen_memory')
        h = stages.gate(capa, h, ctx['glogit'], acc, hay, mx, pk, vistos, hawkes, racha, half=half)
        st.phi[:, t] = phi_t
        st.kc[:, t] = ctx['Kc'][:, 0]
        if not self.ajeno:
            _lib.check(lib.asrn_gen_ring_insert(B, T, nb, C, t, _lib.ptr(ids_t), _lib.ptr(st.ring),
                                                _lib.ptr(st.count), s), 'asrn_gen_ring_insert')
        return h

    def status(self):
        """Device status words of the layers (0 = ok; synchronises)."""
        out = []
        for st in self.layers:
            w, _keep, prep = st.capa.prepared(self.sig.device, self.half)
            cfg = self._cfg(st.capa, self.B, 1)
            out.append(_lib.lib().asrn_layer_status(ctypes_ref(cfg), _lib.ptr(prep), 0,
                                                    _lib.stream_ptr(self.sig.device)))
        return out


Escritor = Writer


# ---- sampling (host side, the reference's semantics: asrn/nucleo.py:1857-1962) ------------------------------------

class _NgramIndex:
    """Per sequence: for each group of n-1 tokens, the tokens that followed it (asrn/nucleo.py:1857-1889)."""

    def __init__(self, texts, n):
        self.n = n
        self.texts = [list(t) for t in texts]
        self.maps = []
        for t in self.texts:
            mp = {}
            for i in range(n - 1, len(t)):
                mp.setdefault(tuple(t[i - n + 1:i]), set()).add(t[i])
            self.maps.append(mp)

    def add(self, tokens):
        for t, mp, p in zip(self.texts, self.maps, tokens):
            t.append(p)
            if len(t) >= self.n:
                mp.setdefault(tuple(t[len(t) - self.n:-1]), set()).add(p)

    def next_mask(self, V, dev):
        mask = torch.zeros(len(self.texts), V, dtype=torch.bool)
        for b, (t, mp) in enumerate(zip(self.texts, self.maps)):
            if len(t) >= self.n:
                follow = mp.get(tuple(t[len(t) - self.n + 1:]), ())
                if follow:
                    mask[b, list(follow)] = True
        return mask.to(dev)


def _brake(lg, recent, penalty, forbidden):
    """Repetition penalty on `recent` tokens and forbidden n-gram closers (asrn/nucleo.py:1912-1920)."""
    if penalty != 1.0:
        seen = torch.zeros_like(lg, dtype=torch.bool).scatter_(1, recent, True)
        lg = torch.where(seen, torch.where(lg > 0, lg / penalty, lg * penalty), lg)
    if forbidden is not None:
        lg = lg.masked_fill(forbidden, -float('inf'))
    return lg


def _keep_quote_mass(q, p, quote):
    """Rescale q so the mass of continuing a quote is p's (asrn/nucleo.py:1934-1942)."""
    mp = (p * quote).sum(-1, keepdim=True)
    mq = (q * quote).sum(-1, keepdim=True)
    ok = (mq > 0) & (mq < 1)
    scale = torch.where(quote, mp / mq.clamp(min=1e-30), (1 - mp) / (1 - mq).clamp(min=1e-30))
    return torch.where(ok, q * scale, q)


def _sample(lg, temperature, top_k, gen, top_p=1.0, quote=None):
    """Temperature, top-k, top-p and the multinomial draw with the seeded CPU generator (asrn/nucleo.py:1945-1962)."""
    p1 = torch.softmax(lg, -1) if quote is not None else None
    lg = lg / max(temperature, 1e-6)
    if top_k and top_k < lg.shape[-1]:
        cut = lg.topk(top_k, dim=-1).values[:, -1:]
        lg = lg.masked_fill(lg < cut, -float('inf'))
    if top_p < 1.0:
        srt, idx = lg.sort(dim=-1, descending=True)
        probs = torch.softmax(srt, -1)
        drop = probs.cumsum(-1) - probs >= top_p
        drop[..., 0] = False
        lg = lg.scatter(1, idx, srt.masked_fill(drop, -float('inf')))
    prob = torch.softmax(lg, -1)
    if quote is not None:
        prob = _keep_quote_mass(prob, p1, quote)
    return torch.multinomial(prob.cpu(), 1, generator=gen).to(lg.device)


@torch.no_grad()
def escribir(modelo, inicio, n_nuevos=200, temperatura=0.8, top_k=40, semilla=0, memoria_de_lo_ajeno=True,
             pena_repeticion=1.0, ventana_pena=64, no_repetir_ngramas=0, parar_en=None, top_p=1.0,
             devolver_logits=True, conservar_cita=True):
    """Write n_nuevos tokens after `inicio` (B, L) or (L,) (asrn/nucleo.py:1965-2043). Returns (sequences int64 on the
    CPU (B, L + n), per-step logits (B, n, V) on the CPU, or None with devolver_logits=False)."""
    was_training = modelo.training
    try:
        modelo.eval()
        if modelo.emb.weight.dtype in (torch.float16, torch.bfloat16):
            raise ValueError('ASRN needs float32 weights; use torch.autocast for bf16 (asrn/nucleo.py:1025-1032)')
        dev = next(modelo.parameters()).device
        gen = torch.Generator(device='cpu').manual_seed(semilla)
        w = Writer(modelo, memoria_de_lo_ajeno)
        x = inicio.to(dev)
        if x.dim() == 1:
            x = x.unsqueeze(0)
        L0 = x.shape[1]
        assert L0 >= 1, 'at least one prompt token is needed'
        V = modelo.config['V']
        if int(x.min()) < 0 or int(x.max()) >= V:
            raise ValueError(f'inicio: tokens outside [0, {V}) (min {int(x.min())}, max {int(x.max())})')
        lg = w.inicio(x, capacidad=L0 + n_nuevos)
        text = x.new_empty(x.shape[0], L0 + n_nuevos)
        text[:, :L0] = x
        length = L0
        quote_ng = _NgramIndex(x.cpu().tolist(), modelo.largos[0].vistos) if conservar_cita else None
        written = _NgramIndex([[] for _ in range(x.shape[0])], no_repetir_ngramas) if no_repetir_ngramas else None
        steps = []
        done = torch.zeros(x.shape[0], dtype=torch.bool, device=dev)
        for k in range(n_nuevos):
            lg = lg.float().clone()
            if devolver_logits:
                steps.append(lg.cpu().clone())
            braked = _brake(lg, text[:, max(0, length - ventana_pena):length], pena_repeticion,
                            written.next_mask(V, dev) if written else None)
            all_out = torch.isneginf(braked).all(-1, keepdim=True)
            lg = torch.where(all_out, lg, braked)
            quote = quote_ng.next_mask(V, dev) if conservar_cita else None
            nxt = _sample(lg, temperatura, top_k, gen, top_p, quote)
            if parar_en is not None:
                nxt = torch.where(done.unsqueeze(1), torch.full_like(nxt, parar_en), nxt)
                done = done | (nxt[:, 0] == parar_en)
            text[:, length] = nxt[:, 0]
            length += 1
            nxt_cpu = nxt[:, 0].cpu()
            for ng in (quote_ng, written):
                if ng is not None:
                    ng.add(nxt_cpu.tolist())
            if parar_en is not None and bool(done.all()):
                break
            if k < n_nuevos - 1:
                lg = w.paso(nxt_cpu)
        x = text[:, :length]
        if not devolver_logits:
            return x.cpu(), None
        return x.cpu(), (torch.stack(steps, 1) if steps else torch.zeros(x.shape[0], 0, V))
    finally:
        modelo.train(was_training)


generate = escribir
