"""Generate the golden fixtures of tests/golden/*.npz by running the reference implementation on the CPU.

Run from the repository root in a container that has the reference checkout (read-only is fine):
    python tests/golden/make_golden.py /path/to/reference

Each fixture stores seeded inputs, the layer's parameters (state_dict names of asrn.estable.CapaASRNEstable) and the
reference's own intermediates and outputs, captured by calling the reference's methods:
  _contexto -> Qc, Kc, beta, log_alfa (asrn/estable.py:153-194); Bt = beta.cumsum(1) (asrn/estable.py:418)
  _phi_y_valores -> phi, V (asrn/nucleo.py:644-659); _ids (asrn/nucleo.py:661-664)
  stable argsort of the per-table ids (asrn/estable.py:220-221)
  _acumular -> salida and the per-table signals (hay, max, peak) (asrn/estable.py:204-300)
  _claves_vistos / _ordenar_claves / _repeticion (asrn/nucleo.py:688-701, asrn/estable.py:304-321)
  forward -> h' (asrn/estable.py:407-421)
The model fixture adds create_model + forward + generate (asrn/__init__.py:60-64, asrn/nucleo.py:1088-1103, 1965-2043).
The generation-state fixture runs the O(1) writer _Escritor(o1=True) (asrn/nucleo.py:1717-1854) on a model whose rings
overflow (chunk 4, 2 bits) and records, after the prompt and after every step, each layer's rings and counts
(_anillo_desde / _anillo_meter, asrn/nucleo.py:1585-1618), the candidate positions of the step (_candidatos,
asrn/nucleo.py:1621-1631) and the Hawkes state of every n-gram key (_MemoriaHawkes, asrn/nucleo.py:1634-1714).
The gradient fixtures run the reference's own autograd through _acumular and escaneo (asrn/estable.py:204-263,
asrn/nucleo.py:188-197, 518-537), and through the whole layer forward (asrn/estable.py:407-421).
The fixtures are read by the tests on any machine; this script is the only place that imports the reference.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from asrn_b200 import synthetic  # noqa: E402


def _move(capa, seed=1, gamma=(0.5, 3.0)):
    """Push the parameters that start neutral (zero) off zero so every term of the layer is exercised
    (the recipe of the reference's own tests: tests/test_estable.py:44-53)."""
    import asrn.nucleo as v89
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for n, p in capa.named_parameters():
            if n in v89._NUEVOS_V87 or n in ('cq.weight', 'w_sufijo', 'w_vistos', 'g_conf.weight', 'g_conf.bias'):
                p.add_(torch.randn(p.shape, generator=g) * 0.5)
        if gamma is not None:
            capa.gamma.copy_(torch.linspace(gamma[0], gamma[1], capa.n_tablas))


def _np(x):
    x = x.detach()
    if x.dtype == torch.bfloat16:
        x = x.float()
    return x.cpu().numpy()


def layer_case(name, d, B, L, V, bf16, opts, seed=0, tokens=None, keep_values=True):
    import asrn
    torch.manual_seed(seed)
    capa = asrn.ASRNLayer(d, **opts)
    _move(capa, seed=seed + 1)
    capa.eval()
    if tokens is None:
        x = synthetic.zipf_tokens(B, L, V, 1.1, seed)
        x = synthetic.plant_repeats(x, 0.25, 4, max(4, L // 4), seed=seed + 1)
    else:
        x = tokens
    x = torch.from_numpy(x)
    g = torch.Generator().manual_seed(seed + 7)
    table = torch.randn(V, d, generator=g)
    E = table[x]
    h = torch.randn(B, L, d, generator=g)
    out = {}
    captured = {}
    orig = capa._senales

    def grab(salida, senal):
        captured['senal'] = senal.detach().clone()
        return orig(salida, senal)

    capa._senales = grab
    with torch.no_grad(), torch.autocast('cpu', dtype=torch.bfloat16, enabled=bf16):
        sig = asrn.firmas_de_piezas(x)
        Qc, Kc, beta, log_alfa = capa._contexto(h)
        Bt = beta.cumsum(1)
        phi, Vv = capa._phi_y_valores(E)
        ids = capa._ids(phi)
        T = capa.n_tablas
        ids_rows = ids.transpose(1, 2).reshape(B * T, L)
        orden = ids_rows.argsort(dim=-1, stable=True)
        acc = capa._acumular(E, Qc, Kc, Bt, log_alfa, sig)
        claves = capa._claves_vistos(sig)
        orden_ng, repetido = capa._ordenar_claves(claves)
        rep = capa._repeticion(sig, beta, Bt, log_alfa)
        y = capa(E, h, x)
    capa._senales = orig
    out.update(tokens=x.numpy(), E=_np(E), h=_np(h), sig=_np(sig), Qc=_np(Qc), Kc=_np(Kc), beta=_np(beta),
               log_alfa=_np(log_alfa), Bt=_np(Bt), phi=_np(phi), V=_np(Vv), ids=_np(ids),
               orden=orden.numpy().astype(np.int32), salida=_np(acc['salida']),
               peso_total=_np(acc['peso_total']), mejor=_np(acc['mejor']), pico=_np(acc['pico']),
               peso_ctx=_np(acc['peso_ctx']), senal=_np(captured['senal']), claves=_np(claves),
               orden_ng=orden_ng.numpy().astype(np.int32), repetido=repetido.numpy(), vistos=_np(rep['vistos']),
               hawkes=_np(rep['hawkes']), racha=_np(rep['racha']), out=_np(y))
    if not keep_values:
        del out['V']
    for k, v in capa.state_dict().items():
        out['param.' + k] = _np(v)
    meta = dict(d=d, B=B, L=L, V=V, bf16=int(bf16), **{k: v for k, v in opts.items()})
    for k, v in meta.items():
        out['meta.' + k] = np.array(v)
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def model_case(name, V, d, n_capas, B, L, L0, n_new, seed=0):
    import asrn
    m = asrn.create_model(V=V, d=d, n_capas=n_capas, semilla=seed)
    for c in m.largos:
        _move(c, seed=seed + 3)
    m.eval()
    x = torch.from_numpy(synthetic.uniform_bytes_with_repeats(B, L, seed) % V)
    with torch.no_grad():
        logits = m(x)
    out = dict(tokens=x.numpy(), logits=logits.numpy())
    for ajeno in (True, False):
        seqs, steps = asrn.generate(m, x[:, :L0], n_nuevos=n_new, top_k=1, memoria_de_lo_ajeno=ajeno)
        tag = 'ajeno' if ajeno else 'propia'
        out[f'gen_{tag}_seqs'] = seqs.numpy()
        out[f'gen_{tag}_logits'] = steps.numpy()
    for k, v in m.state_dict().items():
        out['param.' + k] = _np(v)
    meta = dict(V=V, d=d, n_capas=n_capas, B=B, L=L, L0=L0, n_new=n_new, seed=seed)
    for k, v in meta.items():
        out['meta.' + k] = np.array(v)
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


SAMPLED_SETTINGS = [
    dict(temperatura=0.8, top_k=40, semilla=3),
    dict(temperatura=0.9, top_k=20, top_p=0.9, semilla=5, pena_repeticion=1.3, no_repetir_ngramas=3),
    dict(temperatura=1.0, top_k=0, semilla=11, conservar_cita=False),
    dict(temperatura=0.7, top_k=8, semilla=2**40 + 17),
]


def gen_sampled_case(name):
    """Seeded sampling by the reference's generate on the model_small fixture's weights and prompts: the tokens of
    each setting of SAMPLED_SETTINGS (its draws come from torch.multinomial on a seeded CPU generator)."""
    import asrn
    z = np.load(os.path.join(HERE, 'model_small.npz'))
    V, d, n_capas = int(z['meta.V']), int(z['meta.d']), int(z['meta.n_capas'])
    L0, n_new = int(z['meta.L0']), int(z['meta.n_new'])
    m = asrn.create_model(V=V, d=d, n_capas=n_capas)
    m.load_state_dict({k[6:]: torch.from_numpy(np.asarray(z[k])) for k in z.files if k.startswith('param.')})
    m.eval()
    x0 = torch.from_numpy(z['tokens'][:, :L0])
    out = {'settings': np.array(json.dumps(SAMPLED_SETTINGS))}
    for i, kw in enumerate(SAMPLED_SETTINGS):
        seqs, _ = asrn.generate(m, x0, n_nuevos=n_new, devolver_logits=False, **kw)
        out[f'seqs_{i}'] = seqs.numpy()
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def _hawkes_dump(mem, B, n):
    """(b, order, key, Bu, A) of every key of a _MemoriaHawkes, sorted by (b, order, key)."""
    rows = []
    for b in range(B):
        for j in range(n):
            for key, r in mem.mapas[b * n + j].items():
                rows.append((b, j, key, float(mem.Bu[r]), float(mem.A[r])))
    rows.sort(key=lambda t: (t[0], t[1], t[2]))
    a = np.array(rows, dtype=np.float64).reshape(-1, 5)
    return a[:, :2].astype(np.int32), a[:, 2], a[:, 3], a[:, 4].astype(np.float32)


def gen_state_case(name, B=2, L0=40, n_new=24, seed=0):
    """The O(1) writer's state on overflowing rings (chunk 4, 2 bits: 4 buckets per table), moved parameters, for
    memoria_de_lo_ajeno on and off; the steps are fed the text's own next tokens (teacher forcing)."""
    import asrn
    from asrn import nucleo
    torch.manual_seed(seed + 1)
    m = asrn.create_model(V=60, d=32, n_capas=3, largo_cada=1, chunk=4, n_bits=2)
    for c in m.largos:
        _move(c, seed=seed + 3)
    m.eval()
    g = torch.Generator().manual_seed(seed + 2)
    N = L0 + n_new
    x = torch.randint(0, 60, (B, N), generator=g)
    x[:, N // 2:N // 2 + N // 4] = x[:, :N // 4]
    out = dict(tokens=x.numpy())
    for ajeno in (True, False):
        tag = 'ajeno' if ajeno else 'propia'
        esc = nucleo._Escritor(m, ajeno, o1=True)
        with torch.no_grad():
            lg = esc.inicio(x[:, :L0], capacidad=N)
            logits = [lg]
            for j, (anillo, cuenta) in enumerate(esc.anillos):
                # copies: the writer updates its rings and caches in place at every step
                out[f'{tag}.prompt.l{j}.ring'] = anillo.numpy().copy()
                out[f'{tag}.prompt.l{j}.count'] = cuenta.numpy().copy()
                out[f'{tag}.prompt.l{j}.ids'] = esc.cache[j]['ids'][:, :L0].numpy().copy()
                bj, key, bu, A = _hawkes_dump(esc.hawkes[j], B, m.largos[j].vistos)
                out[f'{tag}.prompt.l{j}.hawkes_bj'], out[f'{tag}.prompt.l{j}.hawkes_key'] = bj, key
                out[f'{tag}.prompt.l{j}.hawkes_bu'], out[f'{tag}.prompt.l{j}.hawkes_a'] = bu, A
            for k in range(n_new - 1):
                t = L0 + k
                before = [a.clone() for a, _ in esc.anillos]
                lg = esc.paso(x[:, t])
                logits.append(lg)
                for j, (anillo, cuenta) in enumerate(esc.anillos):
                    ids_t = esc.cache[j]['ids'][:, t].long()                           # (B, T)
                    Tn = ids_t.shape[1]
                    cand = before[j][torch.arange(B).unsqueeze(1), torch.arange(Tn).unsqueeze(0), ids_t]
                    out[f'{tag}.step{k}.l{j}.ids_t'] = ids_t.numpy().astype(np.int32)
                    out[f'{tag}.step{k}.l{j}.cand'] = cand.numpy().copy()
                    out[f'{tag}.step{k}.l{j}.ring'] = anillo.numpy().copy()
                    out[f'{tag}.step{k}.l{j}.count'] = cuenta.numpy().copy()
                    bj, key, bu, A = _hawkes_dump(esc.hawkes[j], B, m.largos[j].vistos)
                    out[f'{tag}.step{k}.l{j}.hawkes_bj'], out[f'{tag}.step{k}.l{j}.hawkes_key'] = bj, key
                    out[f'{tag}.step{k}.l{j}.hawkes_bu'], out[f'{tag}.step{k}.l{j}.hawkes_a'] = bu, A
        out[f'{tag}.logits'] = torch.stack(logits, 1).numpy().copy()
    for k, v in m.state_dict().items():
        out['param.' + k] = _np(v)
    meta = dict(V=60, d=32, n_capas=3, largo_cada=1, chunk=4, n_bits=2, B=B, L0=L0, n_new=n_new, seed=seed)
    for k, v in meta.items():
        out['meta.' + k] = np.array(v)
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def checkpoint_case(name, seed=0):
    """A model file written by the reference's own guardar() (asrn/nucleo.py:2068-2074), the same weights as a v86
    file (the streak response stored per node as 'u_racha', asrn/nucleo.py:2096-2107), and the reference's logits of
    a forward on seeded tokens (fp32)."""
    import asrn
    m = asrn.create_model(V=64, d=32, n_capas=3, largo_cada=1, semilla=seed, chunk=8, n_bits=4)
    for c in m.largos:
        _move(c, seed=seed + 5)
    m.eval()
    asrn.guardar(m, os.path.join(HERE, name + '.pt'))
    pesos = {k: v.detach().clone() for k, v in m.state_dict().items()}
    for k in [k for k in pesos if k.endswith('d_racha')]:
        pesos[k[:-len('d_racha')] + 'u_racha'] = torch.cumsum(pesos.pop(k), 0)
    torch.save({'config': m.config, 'pesos': pesos}, os.path.join(HERE, name + '_v86.pt'))
    x = torch.from_numpy(synthetic.uniform_bytes_with_repeats(2, 96, seed) % 64)
    with torch.no_grad():
        lg = m(x)
    np.savez_compressed(os.path.join(HERE, name + '.npz'), tokens=x.numpy(), logits=lg.numpy())
    print(f'{name}: {os.path.getsize(os.path.join(HERE, name + ".pt")) / 1024:.0f} KB')


def init_case(name, V, d, n_capas, seed):
    """Checksums of create_model's freshly initialised weights (same seed -> same weights in the build)."""
    import asrn
    m = asrn.create_model(V=V, d=d, n_capas=n_capas, semilla=seed)
    out = {}
    for k, v in m.state_dict().items():
        t = v.detach().double()
        out['sum.' + k] = np.array(float(t.sum()))
        out['sumsq.' + k] = np.array(float((t * t).sum()))
        out['first.' + k] = t.reshape(-1)[:8].numpy()
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def grad_case(name, d, B, L, V, opts, seed=0):
    """Gradients of the bucket attention and of the linear-recurrence scan, from the reference's own autograd on the
    CPU: _acumular (asrn/estable.py:204-263, backward through torch.bmm, _softmax_valido, _TiempoRelativo,
    _DesordenarSumar) with phi, V, Qc, Kc, Bt, log_alfa as leaves, loss = sum(salida * G); escaneo (asrn/nucleo.py:
    188-197, backward _Escaneo, asrn/nucleo.py:518-537) with loss = sum(S * g)."""
    import asrn
    import asrn.nucleo as v89
    torch.manual_seed(seed)
    capa = asrn.ASRNLayer(d, **opts)
    _move(capa, seed=seed + 1)
    capa.eval()
    x = synthetic.zipf_tokens(B, L, V, 1.1, seed)
    x = torch.from_numpy(synthetic.plant_repeats(x, 0.25, 4, max(4, L // 4), seed=seed + 1))
    g = torch.Generator().manual_seed(seed + 7)
    E = torch.randn(V, d, generator=g)[x]
    h = torch.randn(B, L, d, generator=g)
    with torch.no_grad():
        sig = asrn.firmas_de_piezas(x)
        Qc, Kc, beta, log_alfa = capa._contexto(h)
        Bt = beta.cumsum(1)
        phi, Vv = capa._phi_y_valores(E)
        ids = capa._ids(phi)
    T = capa.n_tablas
    ids_rows = ids.transpose(1, 2).reshape(B * T, L)
    orden = ids_rows.argsort(dim=-1, stable=True)
    leaves = {k: t.detach().clone().requires_grad_() for k, t in
              dict(phi=phi, V=Vv, Qc=Qc, Kc=Kc, Bt=Bt, log_alfa=log_alfa).items()}
    captured = {}
    orig_senales = capa._senales

    def grab(salida, senal):
        captured['senal'] = senal.detach().clone()
        return orig_senales(salida, senal)

    capa._senales = grab
    capa._phi_y_valores = lambda E_: (leaves['phi'], leaves['V'])
    acc = capa._acumular(E, leaves['Qc'], leaves['Kc'], leaves['Bt'], leaves['log_alfa'], sig)
    G = torch.randn(B, L, d, generator=g)
    (acc['salida'] * G).sum().backward()
    out = dict(sig=_np(sig), orden=orden.numpy().astype(np.int32),
               ids_o=torch.gather(ids_rows, 1, orden).numpy().astype(np.int32), G=_np(G),
               salida=_np(acc['salida']), senal=_np(captured['senal']), w_sufijo=_np(capa.w_sufijo),
               gamma=_np(capa.gamma), grad_w_sufijo=_np(capa.w_sufijo.grad), grad_gamma=_np(capa.gamma.grad))
    for k, t in leaves.items():
        out[k] = _np(t)
        out['grad_' + k] = _np(t.grad)
    # the scan: a in [0, 1) with resets (a = 0), b and the upstream gradient g of normal draws, rows x L
    a = torch.rand(3, 1000, generator=g, dtype=torch.float64).float()
    a[:, ::97] = 0
    a.requires_grad_()
    b = torch.randn(3, 1000, generator=g).requires_grad_()
    S = v89.escaneo(a, b)
    gS = torch.randn(3, 1000, generator=g)
    (S * gS).sum().backward()
    out.update(scan_a=_np(a), scan_b=_np(b), scan_S=_np(S), scan_g=_np(gS), scan_grad_a=_np(a.grad),
               scan_grad_b=_np(b.grad))
    meta = dict(B=B, L=L, d=d, T=T, nb=capa.n_bits, C=capa.chunk, cf=capa.confirmar, K=capa.sufijo,
                temperatura=float(capa.temperatura), opts=opts)
    out['meta'] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def layer_grad_case(name, d, B, L, V, opts, seed=0):
    """The whole layer's gradients from the reference's autograd on the CPU (asrn/estable.py:407-421, fp32): E and h
    as leaves, loss = sum(forward(E, h, tokens) * G); the output, the gradients of E and h and of every parameter."""
    import asrn
    torch.manual_seed(seed)
    capa = asrn.ASRNLayer(d, **opts)
    _move(capa, seed=seed + 1)
    with torch.no_grad():                     # the streak response and the Hawkes weights off zero too
        g0 = torch.Generator().manual_seed(seed + 5)
        capa.d_racha.add_(torch.randn(capa.d_racha.shape, generator=g0) * 0.3)
        capa.u_hawkes.add_(torch.randn(capa.u_hawkes.shape, generator=g0) * 0.5)
    capa.train()
    x = synthetic.zipf_tokens(B, L, V, 1.1, seed)
    x = torch.from_numpy(synthetic.plant_repeats(x, 0.25, 4, max(4, L // 4), seed=seed + 1))
    g = torch.Generator().manual_seed(seed + 7)
    E = torch.randn(V, d, generator=g)[x].requires_grad_()
    h = torch.randn(B, L, d, generator=g).requires_grad_()
    y = capa(E, h, x)
    G = torch.randn(B, L, d, generator=g)
    (y * G).sum().backward()
    out = dict(tokens=x.numpy(), E=_np(E), h=_np(h), G=_np(G), y=_np(y), grad_E=_np(E.grad), grad_h=_np(h.grad))
    for k, t in capa.state_dict().items():
        out['param.' + k] = _np(t)
    for k, t in capa.named_parameters():
        out['grad.' + k] = _np(t.grad) if t.grad is not None else np.zeros(tuple(t.shape), np.float32)
    out['meta'] = np.frombuffer(json.dumps(dict(d=d, B=B, L=L, opts=opts)).encode(), dtype=np.uint8)
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **out)
    print(f'{name}: {os.path.getsize(path) / 1024:.0f} KB')


def main(ref):
    sys.path.insert(0, ref)
    torch.set_num_threads(8)
    layer_case('layer_f32', 64, 2, 256, 64, False, {})
    layer_case('layer_bf16', 64, 2, 256, 64, True, {})
    layer_case('layer_f32_opts', 48, 2, 200, 24, False, dict(chunk=8, n_bits=6, confirmar=20, sufijo=6, vistos=3))
    layer_case('layer_f32_d96', 96, 2, 150, 40, False, dict(chunk=16, n_bits=4))
    layer_case('layer_f32_short', 32, 1, 5, 12, False, dict(chunk=16, n_bits=4))
    layer_case('layer_f32_one', 32, 1, 1, 12, False, dict(chunk=16, n_bits=4))
    layer_case('layer_bf16_d256', 256, 1, 512, 256, True, {}, keep_values=False)
    layer_case('layer_f32_d256', 256, 1, 512, 256, False, {}, keep_values=False)
    model_case('model_small', V=256, d=64, n_capas=4, B=2, L=192, L0=96, n_new=24)
    init_case('init_cfg1', V=256, d=64, n_capas=4, seed=0)
    gen_state_case('gen_state')
    checkpoint_case('ckpt_ref')
    gen_sampled_case('gen_sampled')
    grad_case('grad_crowded', 64, 2, 300, 40, dict(chunk=16, n_bits=4))
    grad_case('grad_default', 64, 2, 256, 64, {}, seed=3)
    layer_grad_case('layer_grad_crowded', 64, 2, 200, 40, dict(chunk=16, n_bits=4))
    layer_grad_case('layer_grad_default', 64, 2, 160, 64, {}, seed=2)
    grad_case('grad_ragged', 48, 2, 203, 24, dict(chunk=8, n_bits=6, confirmar=20, sufijo=6, vistos=3), seed=4)
    layer_grad_case('layer_grad_ragged', 48, 2, 203, 24, dict(chunk=8, n_bits=6, confirmar=20, sufijo=6, vistos=3),
                    seed=4)


if __name__ == '__main__':
    if len(sys.argv) < 2:
        sys.exit('usage: python tests/golden/make_golden.py <path of the reference checkout> [case ...]')
    if len(sys.argv) > 2:                       # only the named cases
        sys.path.insert(0, sys.argv[1])
        torch.set_num_threads(8)
        for case in sys.argv[2:]:
            {'gen_state': lambda: gen_state_case('gen_state'),
             'checkpoint': lambda: checkpoint_case('ckpt_ref'),
             'gen_sampled': lambda: gen_sampled_case('gen_sampled'),
             'grad': lambda: (grad_case('grad_crowded', 64, 2, 300, 40, dict(chunk=16, n_bits=4)),
                              grad_case('grad_default', 64, 2, 256, 64, {}, seed=3)),
             'layer_grad': lambda: (layer_grad_case('layer_grad_crowded', 64, 2, 200, 40, dict(chunk=16, n_bits=4)),
                                    layer_grad_case('layer_grad_default', 64, 2, 160, 64, {}, seed=2)),
             'grad_ragged': lambda: (
                 grad_case('grad_ragged', 48, 2, 203, 24, dict(chunk=8, n_bits=6, confirmar=20, sufijo=6, vistos=3),
                           seed=4),
                 layer_grad_case('layer_grad_ragged', 48, 2, 203, 24,
                                 dict(chunk=8, n_bits=6, confirmar=20, sufijo=6, vistos=3), seed=4))}[case]()
    else:
        main(sys.argv[1])
