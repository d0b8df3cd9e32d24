"""Incremental generation with the O(1) per-token writer: generate / escribir (asrn/nucleo.py:1965-2043).

Writer mirrors the reference's _Escritor in O(1) mode (asrn/nucleo.py:1717-1854): a prompt pass that runs the model and
keeps, per ASRN layer, the caches of every position (signature, clock, log_alfa, phi, Kc), the per-bucket rings of the
C most recent bucket mates and the n-gram Hawkes table; then one step per new token that touches only T x C candidates
per layer. The ASRN work of a step runs in the kernels of libasrn_b200.so (asrn_gen_*, plus the layer stages on the
new token); the local blocks, embedding and head are PyTorch ops. The rows of E (the values) are cached once, shared
by every layer.

The step is a fixed sequence of launches: the new token's position lives in device memory (the kernels read it and the
step increments it), every buffer is allocated at the prompt for the capacity asked, and the local blocks and head
run in explicit dtypes with weight copies made once (under bf16 autocast: the bf16 copies autocast would make, the
conv as a (d, k*d) matrix), so after one eager step the writer captures the step in a CUDA graph and replays it.

generate() keeps the reference's sampling semantics (temperature, top_k, top_p, repetition penalty, no-repeat
n-grams, stop token, conserving the probability of continuing a quote). The multinomial draw runs on the device with the
random numbers of the reference's seeded CPU generator (asrn_b200.sampling), so greedy decoding (top_k=1) and seeded
sampling give the reference's tokens; per step only the B drawn tokens and a status word come back to the host.
"""
import ctypes

import torch
import torch.nn.functional as F

from . import _lib, stages
from .layer import compute_half, ctypes_ref
from .sampling import DeviceSampler


def _next_pow2(x):
    p = 1
    while p < x:
        p <<= 1
    return p


class _LayerState:
    pass


class _StepWeights:
    """Local-block and head weights in the step's compute type: under bf16 autocast the bf16 copies autocast casts
    them to (round to nearest even), else the fp32 parameters; the conv weight (d, d, k) as a (d, k*d) matrix over the
    window [u_{t-k+1}, ..., u_t] (asrn/nucleo.py:1816-1822)."""

    def __init__(self, m, act):
        self.blocks = []
        for blq in m.bloques:
            d, k = blq.conv.out_channels, blq.k
            wc = blq.conv.weight.detach().permute(0, 2, 1).reshape(d, k * d).to(act).contiguous()
            self.blocks.append((wc, blq.conv.bias.detach().to(act),
                                blq.ff[0].weight.detach().to(act), blq.ff[0].bias.detach().to(act),
                                blq.ff[2].weight.detach().to(act), blq.ff[2].bias.detach().to(act)))
        self.head = m.head.weight.detach().to(act)


def _ln(mod, x):
    return F.layer_norm(x, mod.normalized_shape, mod.weight, mod.bias, mod.eps)


class Writer:
    """O(1) writer over an ASRNModel (asrn/nucleo.py:1717-1854).

    inicio(x0, capacidad) runs the prompt and returns the last position's logits; paso(tokens) appends one token per
    sequence and returns the next logits. grafo=True (default) replays the step as a CUDA graph after its first eager
    run; the graph's logits buffer is overwritten by the next step (paso copies it unless copiar=False)."""

    def __init__(self, modelo, memoria_de_lo_ajeno=True, grafo=True):
        self.m = modelo
        self.ajeno = memoria_de_lo_ajeno
        self.grafo = grafo
        self.graph = None
        self._front_scratch = None     # (B, nq) dot products of the split front kernels

    def _act(self):
        return torch.bfloat16 if self.half else torch.float32

    def _cfg(self, capa, B, L):
        return _lib.make_config(capa, B, L, self.half)

    # ---- prompt ---------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def inicio(self, x0, capacidad=0, lote=None):
        """Prompt pass (asrn/nucleo.py:1750-1794). x0 (B, L0) int64 on the model's CUDA device; capacidad = positions
        to hold (prompt + new tokens); lote = sequences per chunk of the prompt pass (default: about 2^20 tokens per
        chunk). Returns the logits of the last position (B, V)."""
        if not x0.is_cuda:
            raise RuntimeError('asrn_b200 runs on CUDA devices only')
        m = self.m
        self.half = compute_half('cuda')
        act = self._act()
        B, L0 = x0.shape
        dev = x0.device
        d = m.emb.embedding_dim
        self.B, self.L0, self.t = B, L0, L0
        self.cap = max(L0 + 1, capacidad)
        self.graph = None
        self.sig = torch.zeros(B, self.cap, dtype=torch.float32, device=dev)
        self.ea = torch.zeros(B, self.cap, d, dtype=act, device=dev)
        self.e_last = torch.zeros(B, d, dtype=torch.float32, device=dev)
        # per local block, its conv window: the LN1 outputs of the last k positions (oldest first)
        self.buf = [torch.zeros(B, blq.k, d, dtype=act, device=dev) for blq in m.bloques]
        self.lnf = torch.zeros(B, 1, d, dtype=act, device=dev)
        self.layers = [self._new_state(capa, B, dev) for capa in m.largos]
        lote = lote or max(1, min(B, (1 << 20) // max(L0, 1)))
        logits = [self._prompt(x0[b0:b0 + lote], b0) for b0 in range(0, B, lote)]
        self.t_dev = torch.full((1,), L0, dtype=torch.int64, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.sw = _StepWeights(m, act)
        return torch.cat(logits, 0)

    def _new_state(self, capa, B, dev):
        act, cap = self._act(), self.cap
        T, nb, C = capa.n_tablas, capa.n_bits, capa.chunk
        st = _LayerState()
        st.capa = capa
        st.phi = torch.zeros(B, cap, T * nb, dtype=act, device=dev)
        st.kc = torch.zeros(B, cap, capa.confirmar, dtype=act, device=dev)
        st.bt = torch.zeros(B, cap, dtype=torch.float64, device=dev)
        st.la = torch.zeros(B, cap, dtype=torch.float32, device=dev)
        st.racha = torch.zeros(B, dtype=torch.float32, device=dev)
        st.ring = torch.empty(B, T, 1 << nb, C, dtype=torch.int32, device=dev)
        st.count = torch.empty(B, T, 1 << nb, dtype=torch.int32, device=dev)
        st.hcap = max(64, _next_pow2(2 * cap))
        st.table = torch.empty(B, _lib.lib().asrn_gen_hawkes_table_bytes(1, capa.vistos, st.hcap), dtype=torch.uint8,
                               device=dev)
        return st

    def _prompt(self, xc, b0):
        m, act = self.m, self._act()
        Bc, L0 = xc.shape
        b1 = b0 + Bc
        E = m.emb(xc)
        self.sig[b0:b1, :L0] = xc.to(torch.float32)
        self.ea[b0:b1, :L0] = E.to(act)
        self.e_last[b0:b1] = E[:, -1]
        h, j = E, 0
        for i, blq in enumerate(m.bloques):
            u = blq.ln1(h)
            self.buf[i][b0:b1] = F.pad(u, (0, 0, blq.k, 0))[:, L0:].to(act)
            h = blq(h)
            if i in m.pos_largo:
                h = self._prompt_layer(self.layers[j], E, h, xc, b0)
                j += 1
        return m.head(m.ln_f(h[:, -1:]))[:, -1]

    def _prompt_layer(self, st, E, h, xc, b0):
        capa, half = st.capa, self.half
        Bc, L0 = xc.shape
        b1 = b0 + Bc
        T, nb, C = capa.n_tablas, capa.n_bits, capa.chunk
        ctx = stages.context(capa, h, xc, half=half)
        Bt = stages.clock(ctx['beta'])
        hs = stages.hash(capa, E, half=half)
        orden, ids_o = stages.bucket_sort(hs['ids_rows'], nb)
        sc = stages.score(capa, orden, ids_o, hs['phi'], ctx['Qc'], ctx['Kc'], ctx['sig'], Bt, ctx['log_alfa'],
                          hs['Ea'], half=half)
        rep = stages.repetition(capa, ctx['sig'], ctx['beta'], Bt, ctx['log_alfa'])
        h_new = stages.gate(capa, h, ctx['glogit'], sc['acc'], sc['hay'], sc['mx'], sc['pk'], rep['vistos'],
                            rep['hawkes'], rep['racha'], half=half)
        st.phi[b0:b1, :L0] = hs['phi']
        st.kc[b0:b1, :L0] = ctx['Kc']
        st.bt[b0:b1, :L0] = Bt
        st.la[b0:b1, :L0] = ctx['log_alfa']
        st.racha[b0:b1] = rep['racha'][:, -1]
        lib = _lib.lib()
        s = _lib.stream_ptr(xc.device)
        n_valid = L0 - 1 if self.ajeno else L0
        _lib.check(lib.asrn_gen_ring_build(Bc, L0, T, nb, C, n_valid, _lib.ptr(orden), _lib.ptr(ids_o),
                                           _lib.ptr(st.ring[b0:b1]), _lib.ptr(st.count[b0:b1]), s),
                   'asrn_gen_ring_build')
        w, _keep, prep = capa.prepared(xc.device, half)
        cfg = self._cfg(capa, Bc, L0)
        _lib.check(lib.asrn_gen_hawkes_build(ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), L0, self.cap,
                                             _lib.ptr(self.sig[b0:b1]), _lib.ptr(st.bt[b0:b1]),
                                             _lib.ptr(st.la[b0:b1]), _lib.ptr(rep['hawkes'].contiguous()),
                                             _lib.ptr(st.table[b0:b1]), st.hcap, s), 'asrn_gen_hawkes_build')
        return h_new

    # ---- one token --------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def paso(self, pieza, copiar=True):
        """One new token per sequence, pieza (B,) (asrn/nucleo.py:1796-1854). Returns the logits (B, V): a copy, or
        with copiar=False the step's own buffer, valid until the next step."""
        if self.t >= self.cap:
            raise ValueError(f'the writer holds {self.cap} positions; pass capacidad >= prompt + new tokens to '
                             'inicio()')
        self.tok.copy_(pieza.reshape(-1), non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            lg = self.logits
        else:
            lg = self._step()
            if self.grafo and self.t + 1 < self.cap:
                self._capture()
        self.t += 1
        return lg.clone() if copiar else lg

    def _capture(self):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.logits = self._step()
        self.graph = g

    def _step(self):
        """The step's launches: position t is self.t_dev on the device, incremented at the end. Per local block:
        asrn_local_in (the previous block's residual, LN1, conv window), the conv GEMM, asrn_local_mid (GELU +
        residual, LN2), the MLP GEMMs around asrn_local_gelu; the MLP output is added by the next block's
        asrn_local_in (or before an ASRN layer / the head)."""
        m, sw, act, B = self.m, self.sw, self._act(), self.B
        lib = _lib.lib()
        s = _lib.stream_ptr(self.tok.device)
        half = int(self.half)
        with torch.autocast('cuda', enabled=False):
            tok = self.tok
            e_t = F.embedding(tok, m.emb.weight)
            self.sig.index_copy_(1, self.t_dev, tok.to(torch.float32).view(B, 1))
            self.ea.index_copy_(1, self.t_dev, e_t.to(act).view(B, 1, -1))
            h, y, j = e_t, None, 0
            d = h.shape[-1]
            for i, blq in enumerate(m.bloques):
                wc, bc, w1, b1, w2, b2 = sw.blocks[i]
                hin = torch.empty(B, d, dtype=torch.float32, device=h.device)
                _lib.check(lib.asrn_local_in(B, d, blq.k, _lib.ptr(h), _lib.ptr(y), _lib.ptr(hin),
                                             _lib.ptr(blq.ln1.weight), _lib.ptr(blq.ln1.bias), blq.ln1.eps,
                                             _lib.ptr(self.buf[i]), half, s), 'asrn_local_in')
                z = F.linear(self.buf[i].view(B, -1), wc, bc)
                h1 = torch.empty(B, d, dtype=torch.float32, device=h.device)
                v = torch.empty(B, d, dtype=act, device=h.device)
                _lib.check(lib.asrn_local_mid(B, d, _lib.ptr(hin), _lib.ptr(z), _lib.ptr(h1),
                                              _lib.ptr(blq.ln2.weight), _lib.ptr(blq.ln2.bias), blq.ln2.eps,
                                              _lib.ptr(v), half, s), 'asrn_local_mid')
                f = F.linear(v, w1, b1)
                _lib.check(lib.asrn_local_gelu(f.numel(), _lib.ptr(f), half, s), 'asrn_local_gelu')
                h, y = h1, F.linear(f, w2, b2)
                if i in m.pos_largo:
                    h = self._step_layer(self.layers[j], e_t, h, y, tok)     # the layer's front adds y to h
                    y = None
                    j += 1
            _lib.check(lib.asrn_local_in(B, d, 1, _lib.ptr(h), _lib.ptr(y), None, _lib.ptr(m.ln_f.weight),
                                         _lib.ptr(m.ln_f.bias), m.ln_f.eps, _lib.ptr(self.lnf), half, s),
                       'asrn_local_in')
            lg = F.linear(self.lnf.view(B, d), sw.head)
            self.e_last.copy_(e_t)
            self.t_dev += 1
        return lg

    def _step_layer(self, st, e_t, h_prev, y, tok):
        """One ASRN layer for the new tokens: front (context + hash, on h = h_prev + y, formed in the front kernel),
        n-gram memory, candidate attention, gate."""
        capa, half, B = st.capa, self.half, self.B
        dev = tok.device
        T, nb, C, n, cf, d = capa.n_tablas, capa.n_bits, capa.chunk, capa.vistos, capa.confirmar, capa.d
        act = self._act()
        lib = _lib.lib()
        s = _lib.stream_ptr(dev)
        w, _keep, prep = capa.prepared(dev, half)
        cfg = self._cfg(capa, B, 1)
        cr, wr, pr, tp = ctypes_ref(cfg), ctypes_ref(w), _lib.ptr(prep), _lib.ptr(self.t_dev)
        qc = torch.empty(B, cf, dtype=act, device=dev)
        kc = torch.empty(B, cf, dtype=act, device=dev)
        beta = torch.empty(B, dtype=torch.float64, device=dev)
        la = torch.empty(B, dtype=torch.float32, device=dev)
        glogit = torch.empty(B, dtype=torch.float32, device=dev)
        sig = torch.empty(B, dtype=torch.float32, device=dev)
        phi = torch.empty(B, T * nb, dtype=act, device=dev)
        ids = torch.empty(B, T, dtype=torch.int16, device=dev)
        nq = 2 * cf + 3 + 3 * cfg.hidden
        if self._front_scratch is None or self._front_scratch.numel() < B * nq:
            self._front_scratch = torch.empty(B * nq, dtype=torch.float32, device=dev)
        h = torch.empty(B, d, dtype=torch.float32, device=dev)
        _lib.check(lib.asrn_gen_front_residual(cr, wr, pr, _lib.ptr(h_prev), _lib.ptr(y), _lib.ptr(h), _lib.ptr(e_t),
                                               _lib.ptr(self.e_last), _lib.ptr(tok), _lib.ptr(qc), _lib.ptr(kc),
                                               _lib.ptr(beta), _lib.ptr(la), _lib.ptr(glogit), _lib.ptr(sig),
                                               _lib.ptr(phi), _lib.ptr(ids), _lib.ptr(self._front_scratch), s),
                   'asrn_gen_front_residual')
        vistos = torch.empty(B, n, dtype=torch.uint8, device=dev)
        hawkes = torch.empty(B, n, dtype=torch.float32, device=dev)
        racha = torch.empty(B, dtype=torch.float32, device=dev)
        _lib.check(lib.asrn_gen_memory(cr, wr, pr, tp, self.cap, _lib.ptr(self.sig), _lib.ptr(st.bt), _lib.ptr(st.la),
                                       _lib.ptr(beta), _lib.ptr(la), _lib.ptr(st.table), st.hcap, _lib.ptr(st.racha),
                                       _lib.ptr(vistos), _lib.ptr(hawkes), _lib.ptr(racha), s), 'asrn_gen_memory')
        acc = torch.empty(B, d, dtype=torch.float32, device=dev)
        hay = torch.empty(B, T, dtype=torch.uint8, device=dev)
        mx = torch.empty(B, T, dtype=torch.float32, device=dev)
        pk = torch.empty(B, T, dtype=torch.float32, device=dev)
        # bf16: the attention kernel also produces the gate's operand and gate values
        cbuf = torch.empty(B, d, dtype=torch.bfloat16, device=dev) if half else None
        sigma = torch.empty(B, dtype=torch.float32, device=dev) if half else None
        gate_in = [_lib.ptr(x if half else None) for x in (glogit, vistos, hawkes, racha)]
        _lib.check(lib.asrn_gen_attend(cr, wr, pr, tp, self.cap, _lib.ptr(ids), _lib.ptr(phi), _lib.ptr(qc),
                                       _lib.ptr(kc), _lib.ptr(st.ring), _lib.ptr(self.sig), _lib.ptr(st.bt),
                                       _lib.ptr(st.la), _lib.ptr(st.phi), _lib.ptr(st.kc), _lib.ptr(self.ea),
                                       _lib.ptr(acc), _lib.ptr(hay), _lib.ptr(mx), _lib.ptr(pk), *gate_in,
                                       _lib.ptr(cbuf), _lib.ptr(sigma), s), 'asrn_gen_attend')
        h_out = torch.empty(B, d, dtype=torch.float32, device=dev)
        _lib.check(lib.asrn_gen_gate(cr, wr, pr, _lib.ptr(h), _lib.ptr(glogit), _lib.ptr(acc), _lib.ptr(hay),
                                     _lib.ptr(mx), _lib.ptr(pk), _lib.ptr(vistos), _lib.ptr(hawkes), _lib.ptr(racha),
                                     _lib.ptr(h_out), _lib.ptr(cbuf), _lib.ptr(sigma), s), 'asrn_gen_gate')
        if not self.ajeno:
            _lib.check(lib.asrn_gen_ring_insert(B, T, nb, C, tp, _lib.ptr(ids), _lib.ptr(st.ring),
                                                _lib.ptr(st.count), s), 'asrn_gen_ring_insert')
        return h_out

    def status(self):
        """Device status words of the layers (0 = ok; synchronises)."""
        out = []
        for st in self.layers:
            w, _keep, prep = st.capa.prepared(self.sig.device, self.half)
            cfg = self._cfg(st.capa, self.B, 1)
            out.append(_lib.lib().asrn_layer_status(ctypes_ref(cfg), _lib.ptr(prep), 0,
                                                    _lib.stream_ptr(self.sig.device)))
        return out

    def cerrar(self):
        """Release the step's CUDA graph and the state."""
        self.graph = None
        self.logits = None
        self.layers = []


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
        """(B, V) bool on dev: the tokens that followed each sequence's last n-1 tokens (built from index lists)."""
        rows, cols = [], []
        for b, (t, mp) in enumerate(zip(self.texts, self.maps)):
            if len(t) >= self.n:
                follow = mp.get(tuple(t[len(t) - self.n + 1:]), ())
                rows += [b] * len(follow)
                cols += list(follow)
        mask = torch.zeros(len(self.texts), V, dtype=torch.bool, device=dev)
        if rows:
            mask[torch.tensor(rows, device=dev), torch.tensor(cols, device=dev)] = True
        return mask


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


def argmax_rows(x):
    """argmax over the last dimension of a (rows, V) CUDA tensor (fp32 or bf16) with torch.argmax's rule (NaN wins,
    ties keep the lower index), one block per row on the device (asrn_argmax_rows): the greedy token of a step."""
    if not x.is_cuda or x.dim() != 2 or x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError('argmax_rows takes a 2-D float32 or bfloat16 CUDA tensor')
    x = x.contiguous()
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    _lib.check(_lib.lib().asrn_argmax_rows(x.shape[0], x.shape[1], _lib.ptr(x), int(x.dtype == torch.bfloat16),
                                           _lib.ptr(out), _lib.stream_ptr(x.device)), 'asrn_argmax_rows')
    return out


def _sample(lg, temperature, top_k, sampler, top_p=1.0, quote=None):
    """Temperature, top-k, top-p and the multinomial draw (asrn/nucleo.py:1945-1962); the draw is the device replay of
    the reference's seeded CPU generator (asrn_b200.sampling.DeviceSampler)."""
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
    return sampler.sample(prob)


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
        w = Writer(modelo, memoria_de_lo_ajeno)
        x = inicio.to(dev)
        if x.dim() == 1:
            x = x.unsqueeze(0)
        L0 = x.shape[1]
        assert L0 >= 1, 'at least one prompt token is needed'
        V = modelo.config['V']
        if int(x.min()) < 0 or int(x.max()) >= V:
            raise ValueError(f'inicio: tokens outside [0, {V}) (min {int(x.min())}, max {int(x.max())})')
        B = x.shape[0]
        # the reference's torch.Generator('cpu').manual_seed(semilla), replayed on the device (asrn/nucleo.py:1996)
        sampler = DeviceSampler(semilla, B, V, n_nuevos, dev)
        lg = w.inicio(x, capacidad=L0 + n_nuevos)
        text = x.new_empty(B, L0 + n_nuevos)
        text[:, :L0] = x
        length = L0
        quote_ng = _NgramIndex(x.cpu().tolist(), modelo.largos[0].vistos) if conservar_cita else None
        written = _NgramIndex([[] for _ in range(B)], no_repetir_ngramas) if no_repetir_ngramas else None
        steps = []
        done = torch.zeros(B, dtype=torch.bool, device=dev)
        done_host = [False] * B
        for k in range(n_nuevos):
            lg = lg.float()
            if devolver_logits:
                steps.append(lg.cpu())
            braked = _brake(lg, text[:, max(0, length - ventana_pena):length], pena_repeticion,
                            written.next_mask(V, dev) if written else None)
            all_out = torch.isneginf(braked).all(-1, keepdim=True)
            lg = torch.where(all_out, lg, braked)
            quote = quote_ng.next_mask(V, dev) if conservar_cita else None
            nxt = _sample(lg, temperatura, top_k, sampler, top_p, quote)
            toks = sampler.tokens_and_check()            # the step's only device sync: B tokens and a status word
            if parar_en is not None:
                nxt = torch.where(done.unsqueeze(1), torch.full_like(nxt, parar_en), nxt)
                done = done | (nxt[:, 0] == parar_en)
                toks = [parar_en if dn else t for t, dn in zip(toks, done_host)]
                done_host = [dn or t == parar_en for t, dn in zip(toks, done_host)]
            text[:, length] = nxt[:, 0]
            length += 1
            for ng in (quote_ng, written):
                if ng is not None:
                    ng.add(toks)
            if parar_en is not None and all(done_host):
                break
            if k < n_nuevos - 1:
                lg = w.paso(nxt[:, 0])
        status = w.status()
        w.cerrar()
        if any(status):
            raise RuntimeError(f'generation step status words {status} (asrn_status_string names them)')
        x = text[:, :length]
        if not devolver_logits:
            return x.cpu(), None
        return x.cpu(), (torch.stack(steps, 1) if steps else torch.zeros(x.shape[0], 0, V))
    finally:
        modelo.train(was_training)


generate = escribir
