"""GPU parity of the O(1) generation step (asrn_gen_* entry points through asrn_b200.generate) and of the model
forward, against the reference's own outputs (tests/golden/model_small.npz) and against the whole-text forward.

Bars: greedy sequences identical; logits within 1e-4 max-norm relative (fp32)."""
import numpy as np
import pytest
import torch

from conftest import load_fixture, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _exact_fp32_torch_ops():
    """The local blocks and the head are PyTorch ops: compare them in true fp32 (cuDNN defaults to TF32 for
    convolutions), as the reference's golden outputs were made on the CPU."""
    old = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = old


def _model_from_fixture(dev):
    import asrn_b200
    z, params, meta = load_fixture('model_small')
    m = asrn_b200.create_model(V=meta['V'], d=meta['d'], n_capas=meta['n_capas'])
    m.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})
    return m.to(dev).eval(), z, meta


def test_model_forward_matches_reference(cuda):
    m, z, meta = _model_from_fixture(cuda)
    with torch.no_grad():
        lg = m(torch.from_numpy(z['tokens']).to(cuda)).cpu().numpy()
    assert rel_err(lg, z['logits']) <= 1e-4


@pytest.mark.parametrize('ajeno', [True, False])
def test_generate_greedy_matches_reference(ajeno, cuda):
    import asrn_b200
    m, z, meta = _model_from_fixture(cuda)
    tag = 'ajeno' if ajeno else 'propia'
    x0 = torch.from_numpy(z['tokens'][:, :meta['L0']])
    seqs, steps = asrn_b200.generate(m, x0.to(cuda), n_nuevos=meta['n_new'], top_k=1, memoria_de_lo_ajeno=ajeno)
    assert np.array_equal(seqs.numpy(), z[f'gen_{tag}_seqs'])
    assert rel_err(steps.numpy(), z[f'gen_{tag}_logits']) <= 1e-4


def _small_moved_model(cuda, **kw):
    import asrn_b200
    torch.manual_seed(1)
    m = asrn_b200.create_model(V=60, d=32, n_capas=3, largo_cada=1, chunk=4, n_bits=2, **kw)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for c in m.largos:
            for name, p in c.named_parameters():
                if name in ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha',
                            'cq.weight', 'w_sufijo', 'w_vistos', 'g_conf.weight'):
                    p.add_(torch.randn(p.shape, generator=g) * 0.5)
    return m.to(cuda).eval()


def _text(B, N, cuda, seed=2):
    gx = torch.Generator().manual_seed(seed)
    x = torch.randint(0, 60, (B, N), generator=gx)
    x[:, N // 2:N // 2 + N // 4] = x[:, :N // 4]
    return x.to(cuda)


@pytest.mark.parametrize('B,L0,n', [(2, 40, 50), (1, 2, 30), (3, 1, 20)])
def test_writer_steps_equal_whole_text(B, L0, n, cuda):
    """Step by step == the model on the whole text (tests/test_nucleo.py:118-140), with buckets that overflow their
    rings (chunk 4, 2 bits: 4 buckets per table) and moved parameters; memory of its own writing (ajeno off)."""
    import asrn_b200
    torch.manual_seed(1)
    m = asrn_b200.create_model(V=60, d=32, n_capas=3, largo_cada=1, chunk=4, n_bits=2)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for c in m.largos:
            for name, p in c.named_parameters():
                if name in ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha',
                            'cq.weight', 'w_sufijo', 'w_vistos', 'g_conf.weight'):
                    p.add_(torch.randn(p.shape, generator=g) * 0.5)
    m = m.to(cuda).eval()
    gx = torch.Generator().manual_seed(2)
    x = torch.randint(0, 60, (B, L0 + n), generator=gx)
    x[:, (L0 + n) // 2:(L0 + n) // 2 + (L0 + n) // 4] = x[:, :(L0 + n) // 4]
    x = x.to(cuda)
    w = asrn_b200.Writer(m, memoria_de_lo_ajeno=False)
    lgs = [w.inicio(x[:, :L0], capacidad=L0 + n)]
    lgs += [w.paso(x[:, t]) for t in range(L0, L0 + n - 1)]
    steps = torch.stack(lgs, 1)
    with torch.no_grad():
        whole = m(x[:, :L0 + n - 1])[:, L0 - 1:]
    assert rel_err(steps.cpu().numpy(), whole.cpu().numpy()) <= 1e-4
    assert all(s == 0 for s in w.status())


def test_generate_sampling_is_seeded(cuda):
    """Non-greedy sampling with temperature / top-k / top-p / repetition penalty / no-repeat n-grams is deterministic
    for a seed and respects the stop token."""
    import asrn_b200
    m, z, meta = _model_from_fixture(cuda)
    x0 = torch.from_numpy(z['tokens'][:1, :32]).to(cuda)
    a = asrn_b200.generate(m, x0, n_nuevos=12, temperatura=0.9, top_k=20, top_p=0.9, semilla=5, pena_repeticion=1.3,
                           no_repetir_ngramas=3)[0]
    b = asrn_b200.generate(m, x0, n_nuevos=12, temperatura=0.9, top_k=20, top_p=0.9, semilla=5, pena_repeticion=1.3,
                           no_repetir_ngramas=3)[0]
    assert torch.equal(a, b) and a.shape == (1, 44)
    stop = int(a[0, 33])
    c, lg = asrn_b200.generate(m, x0, n_nuevos=12, temperatura=0.9, top_k=20, top_p=0.9, semilla=5,
                               pena_repeticion=1.3, no_repetir_ngramas=3, parar_en=stop, devolver_logits=False)
    assert lg is None and int(c[0, -1]) == stop


@pytest.mark.parametrize('ajeno', [True, False])
def test_writer_graph_equals_eager(ajeno, cuda):
    """The step replayed as a CUDA graph gives the eager step's logits, and a prompt pass in chunks of one sequence
    the unchunked one's (to the last bits: the prompt's layer forward sums its tables with fp32 atomics)."""
    import asrn_b200
    m = _small_moved_model(cuda)
    x = _text(3, 70, cuda)
    out = []
    for grafo, lote in ((False, None), (True, None), (True, 1)):
        w = asrn_b200.Writer(m, memoria_de_lo_ajeno=ajeno, grafo=grafo)
        lgs = [w.inicio(x[:, :30], capacidad=70, lote=lote)]
        lgs += [w.paso(x[:, t]) for t in range(30, 69)]
        assert (w.graph is not None) == grafo
        assert all(s == 0 for s in w.status())
        out.append(torch.stack(lgs, 1))
        w.cerrar()
    assert rel_err(out[1].cpu().numpy(), out[0].cpu().numpy()) <= 1e-5
    assert rel_err(out[2].cpu().numpy(), out[0].cpu().numpy()) <= 1e-5


def test_gen_step_is_deterministic(cuda):
    """The step sums its candidate tables in a fixed order (no atomics): two runs from the same state are bit-equal."""
    import asrn_b200
    m = _small_moved_model(cuda)
    x = _text(3, 60, cuda)
    w = asrn_b200.Writer(m, grafo=False)
    w.inicio(x[:, :40], capacidad=60)
    mutable = [w.sig, w.ea, w.t_dev, w.e_last] + list(w.buf)
    for st in w.layers:
        mutable += [st.phi, st.kc, st.bt, st.la, st.table, st.racha, st.ring, st.count]
    saved = [t.clone() for t in mutable]
    w.tok.copy_(x[:, 40])
    a = w._step().clone()
    for dst, src in zip(mutable, saved):
        dst.copy_(src)
    b = w._step().clone()
    assert torch.equal(a, b)


def test_writer_bf16_steps_equal_whole_text(cuda):
    """Under bf16 autocast the O(1) steps (bf16 weight copies, graph replay) follow the whole-text forward within the
    bf16 tolerance."""
    import asrn_b200
    m = _small_moved_model(cuda)
    x = _text(2, 80, cuda)
    with torch.autocast('cuda', dtype=torch.bfloat16):
        w = asrn_b200.Writer(m, memoria_de_lo_ajeno=False)
        lgs = [w.inicio(x[:, :40], capacidad=80)]
        lgs += [w.paso(x[:, t]) for t in range(40, 79)]
        with torch.no_grad():
            whole = m(x[:, :79])[:, 39:]
    steps = torch.stack(lgs, 1).float()
    assert rel_err(steps.cpu().numpy(), whole.float().cpu().numpy()) <= 2e-2
    assert all(s == 0 for s in w.status())


def test_gen_position_out_of_range_sets_status(cuda):
    """A device position outside [1, cap) makes the step kernel write nothing and report ASRN_ERR_ARG in the layer's
    status word (the launch itself succeeds: the position is only known on the device)."""
    import ctypes
    import asrn_b200
    from asrn_b200 import _lib
    m = _small_moved_model(cuda)
    x = _text(2, 20, cuda)
    w = asrn_b200.Writer(m, grafo=False)
    w.inicio(x[:, :10], capacidad=12)
    st = w.layers[0]
    capa = st.capa
    bt_before, la_before = st.bt.clone(), st.la.clone()
    wts, _keep, prep = capa.prepared(cuda, False)
    cfg = _lib.make_config(capa, 2, 1, False)
    n = capa.vistos
    beta = torch.ones(2, dtype=torch.float64, device=cuda)
    la = torch.zeros(2, dtype=torch.float32, device=cuda)
    vistos = torch.empty(2, n, dtype=torch.uint8, device=cuda)
    hawkes = torch.empty(2, n, dtype=torch.float32, device=cuda)
    racha = torch.empty(2, dtype=torch.float32, device=cuda)
    for bad_t in (w.cap, 0):
        bad = torch.full((1,), bad_t, dtype=torch.int64, device=cuda)
        rc = _lib.lib().asrn_gen_memory(ctypes.byref(cfg), ctypes.byref(wts), _lib.ptr(prep), _lib.ptr(bad), w.cap,
                                        _lib.ptr(w.sig), _lib.ptr(st.bt), _lib.ptr(st.la), _lib.ptr(beta),
                                        _lib.ptr(la), _lib.ptr(st.table), st.hcap, _lib.ptr(st.racha),
                                        _lib.ptr(vistos), _lib.ptr(hawkes), _lib.ptr(racha), _lib.stream_ptr(cuda))
        assert rc == _lib.ASRN_OK
        assert _lib.lib().asrn_layer_status(ctypes.byref(cfg), _lib.ptr(prep), 1, _lib.stream_ptr(cuda)) == \
            _lib.ASRN_ERR_ARG
    assert torch.equal(st.bt, bt_before) and torch.equal(st.la, la_before)


@pytest.mark.parametrize('half', [False, True])
def test_split_front_equals_single_block_front(half, cuda):
    """asrn_gen_front with a scratch buffer (projections split over (sequence, weight-row slice) blocks, then a
    finishing kernel) gives the same bits as the one-block-per-sequence kernel: every output, fp32 and bf16."""
    import ctypes
    import asrn_b200
    from asrn_b200 import _lib
    torch.manual_seed(5)
    layer = asrn_b200.ASRNLayer(256)
    g = torch.Generator().manual_seed(6)
    with torch.no_grad():
        for n_, p_ in layer.named_parameters():
            if n_ in ('w_reloj', 'b_reloj', 'cq.weight', 'g_conf.weight'):
                p_.add_(torch.randn(p_.shape, generator=g) * 0.5)
    layer = layer.to(cuda)
    B, d = 5, 256
    wts, _keep, prep = layer.prepared(cuda, half)
    cfg = _lib.make_config(layer, B, 1, half)
    act = torch.bfloat16 if half else torch.float32
    h = torch.randn(B, d, generator=g).to(cuda)
    e_t = torch.randn(B, d, generator=g).to(cuda)
    e_p = torch.randn(B, d, generator=g).to(cuda)
    tok = torch.randint(0, 1000, (B,), generator=g).to(cuda)
    T, nb, cf = layer.n_tablas, layer.n_bits, layer.confirmar
    outs = []
    for split in (False, True):
        o = dict(qc=torch.empty(B, cf, dtype=act, device=cuda), kc=torch.empty(B, cf, dtype=act, device=cuda),
                 beta=torch.empty(B, dtype=torch.float64, device=cuda), la=torch.empty(B, device=cuda),
                 gl=torch.empty(B, device=cuda), sig=torch.empty(B, device=cuda),
                 phi=torch.empty(B, T * nb, dtype=act, device=cuda), ids=torch.empty(B, T, dtype=torch.int16,
                                                                                     device=cuda))
        scratch = torch.empty(B * (2 * cf + 3 + 3 * cfg.hidden), device=cuda) if split else None
        rc = _lib.lib().asrn_gen_front(ctypes.byref(cfg), ctypes.byref(wts), _lib.ptr(prep), _lib.ptr(h),
                                       _lib.ptr(e_t), _lib.ptr(e_p), _lib.ptr(tok), _lib.ptr(o['qc']),
                                       _lib.ptr(o['kc']), _lib.ptr(o['beta']), _lib.ptr(o['la']), _lib.ptr(o['gl']),
                                       _lib.ptr(o['sig']), _lib.ptr(o['phi']), _lib.ptr(o['ids']), _lib.ptr(scratch),
                                       _lib.stream_ptr(cuda))
        assert rc == _lib.ASRN_OK
        outs.append(o)
    torch.cuda.synchronize()
    for k in outs[0]:
        assert torch.equal(outs[0][k], outs[1][k]), k
