"""GPU parity of the CUDA path (libasrn_b200.so through the C ABI) against the reference's own outputs
(tests/golden/*.npz) and the CPU oracle (oracle/asrn_oracle.py).

Bars: bucket ids from the reference's phi, sort permutations, candidate indices and suffix-match lengths bit-exact;
fp32 outputs within 1e-4 max-norm relative error; bf16 outputs within 2e-2. End-to-end bucket ids from our own phi may
differ from the reference only where |phi_ref| is within the precision's rounding of 0 (conftest.check_ids_agree).
"""
import numpy as np
import pytest
import torch

from conftest import LAYER_FIXTURES, check_ids_agree, layer_options, load_fixture, rel_err
from oracle import asrn_oracle as O

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-4
TOL_BF16 = 2e-2


def _layer(params, meta, dev):
    import asrn_b200
    layer = asrn_b200.ASRNLayer(meta['d'], **layer_options(meta))
    layer.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})
    return layer.to(dev).eval()


def _t(x, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dtype is None else t.to(dtype)


def _ids_rows(ids_btl, dev):
    B, L, T = ids_btl.shape
    return _t(ids_btl.transpose(0, 2, 1).reshape(B * T, L).astype(np.int16), dev)


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_signpack_of_reference_phi_is_bit_exact(name, cuda):
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    B, L = z['tokens'].shape
    T, nb = z['ids'].shape[-1], layer_options(meta).get('n_bits', 14)
    rows = stages.ids_from_phi(_t(z['phi'], cuda), T, nb)
    got = stages.ids_rows_to_btl(rows, B, T).cpu().numpy()
    assert np.array_equal(got, z['ids'])


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_bucket_sort_of_reference_ids_is_bit_exact(name, cuda):
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    nb = layer_options(meta).get('n_bits', 14)
    orden, ids_o = stages.bucket_sort(_ids_rows(z['ids'], cuda), nb)
    assert np.array_equal(orden.cpu().numpy(), z['orden'])
    B, L, T = z['ids'].shape
    rows = z['ids'].transpose(0, 2, 1).reshape(B * T, L)
    assert np.array_equal(ids_o.cpu().numpy().astype(np.int32) & 0xFFFF, np.take_along_axis(rows, z['orden'], -1))


@pytest.mark.parametrize('L,nb,rows', [(20000, 14, 3), (8193, 4, 2), (30000, 2, 2), (65536, 16, 1), (8192, 14, 2),
                                       (1, 14, 1), (37, 3, 4), (5000, 9, 3), (1000, 16, 2), (2048, 1, 2),
                                       (24, 14, 70000), (9000, 5, 3)])
def test_bucket_sort_long_rows_match_stable_argsort(L, nb, rows, cuda):
    """Rows longer than one tile (the per-tile histogram merge), many ties, tiny rows, one- to three-pass digit splits
    (1, 9, 14, 16 bits) and more rows than one launch's grid holds (70,000)."""
    from asrn_b200 import stages
    g = np.random.default_rng(L + nb)
    ids = g.integers(0, 1 << nb, (rows, L)).astype(np.int64)
    ids[:, L // 3:L // 2] = ids[:, :L // 2 - L // 3]                       # repeated runs
    orden, ids_o = stages.bucket_sort(_t(ids.astype(np.uint16).view(np.int16), cuda), nb)
    ref = np.argsort(ids, axis=-1, kind='stable')
    assert np.array_equal(orden.cpu().numpy(), ref)
    assert np.array_equal(ids_o.cpu().numpy().view(np.uint16).astype(np.int64), np.take_along_axis(ids, ref, -1))


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_candidates_and_suffix_lengths_are_bit_exact(name, cuda):
    """Candidate indices (the <= C most recent bucket mates) and suffix-match lengths vs the window definition."""
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    opts = layer_options(meta)
    C, K = opts.get('chunk', 32), opts.get('sufijo', 4)
    B, L, T = z['ids'].shape
    rows = z['ids'].transpose(0, 2, 1).reshape(B * T, L)
    ids_o = np.take_along_axis(rows, z['orden'], -1)
    cand, suf = stages.candidates(_t(z['orden'], cuda), _t(ids_o.astype(np.int16), cuda), _t(z['sig'], cuda), T, C, K)
    cand, suf = cand.cpu().numpy(), suf.cpu().numpy()
    Pf = O.anteriores(z['sig'], K)
    for r in range(B * T):
        b = r // T
        lo = O.candidatos_filas(ids_o[r], C)
        for s in range(L):
            ks = z['orden'][r, lo[s]:s][::-1]                                  # most recent first
            want = np.full(C, -1)
            want[:ks.size] = ks
            assert np.array_equal(cand[r, s], want), (r, s)
            q = z['orden'][r, s]
            ln = O.largo_seguido(np.broadcast_to(Pf[b, q], (ks.size, K)), Pf[b, ks]) if ks.size else np.zeros(0)
            assert np.array_equal(suf[r, s, :ks.size], ln), (r, s)


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_repetition_memory_matches_reference(name, cuda):
    """n-gram keys, their stable sort and repeated flags bit-exact; Hawkes intensity and streak within 1e-5."""
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    layer = _layer(params, meta, cuda)
    out = stages.repetition(layer, _t(z['sig'], cuda), _t(z['beta'], cuda), _t(z['Bt'], cuda),
                            _t(z['log_alfa'], cuda), debug=True)
    assert np.array_equal(out['keys'].cpu().numpy(), z['claves'], equal_nan=True)
    assert np.array_equal(out['orden_ng'].cpu().numpy(), z['orden_ng'])
    assert np.array_equal(out['repetido'].cpu().numpy().astype(bool), z['repetido'])
    assert np.array_equal(out['vistos'].cpu().numpy().astype(np.float32), z['vistos'])
    assert rel_err(out['hawkes'].cpu().numpy(), z['hawkes']) <= 1e-5
    assert rel_err(out['racha'].cpu().numpy(), z['racha']) <= 1e-5


@pytest.mark.parametrize('L', [1000, 3000, 8192, 12000, 16385, 40000])
def test_repetition_long_rows_match_oracle(L, cuda):
    """Rows sorted in one block (radix sort, row lengths not multiples of 1024) and rows longer than 8192 (tile sort +
    merge passes + tiled scan): keys, sort permutation and repeated flags bit-exact against the oracle; Hawkes
    intensity and streak within 1e-5. Repetitive text (12-token
    vocabulary) so that n-gram groups are long and cross tile boundaries."""
    import asrn_b200
    from asrn_b200 import stages
    from oracle import asrn_oracle as O
    torch.manual_seed(3)
    layer = asrn_b200.ASRNLayer(32)
    g = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for n_, p_ in layer.named_parameters():
            if n_ in ('log_kappa', 'log_kappa_racha'):
                p_.add_(torch.randn(p_.shape, generator=g) * 0.5)
    params = {k: v.detach().numpy().copy() for k, v in layer.state_dict().items()}
    rng = np.random.default_rng(5)
    B = 2
    tok = rng.integers(0, 12, size=(B, L)).astype(np.int64)
    n_rep = min(5000, L // 2 - 100)
    tok[:, L // 2:L // 2 + n_rep] = tok[:, 100:100 + n_rep]
    sig = tok.astype(np.float32)
    beta = rng.uniform(0.01, 2.0, size=(B, L))
    Bt = np.cumsum(beta, axis=1)
    log_alfa = rng.uniform(-3.0, 0.5, size=(B, L)).astype(np.float32)
    lay = O.Layer(params, 32)
    ref = O.repeticion(lay, sig, beta, Bt, log_alfa)
    vis_ref, haw_ref, racha_ref = ref['vistos'], ref['hawkes'], ref['racha']
    claves, orden_ref, rep_ref = ref['claves'], ref['orden_ng'], ref['repetido']
    layer = layer.to(cuda)
    out = stages.repetition(layer, _t(sig, cuda), _t(beta, cuda), _t(Bt, cuda), _t(log_alfa, cuda), debug=True)
    assert np.array_equal(out['keys'].cpu().numpy(), claves, equal_nan=True)
    assert np.array_equal(out['orden_ng'].cpu().numpy(), orden_ref)
    assert np.array_equal(out['repetido'].cpu().numpy().astype(bool), rep_ref)
    assert np.array_equal(out['vistos'].cpu().numpy().astype(bool), vis_ref.astype(bool))
    assert rel_err(out['hawkes'].cpu().numpy(), haw_ref) <= 1e-5
    assert rel_err(out['racha'].cpu().numpy(), racha_ref) <= 1e-5


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_context_matches_reference(name, cuda):
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    layer = _layer(params, meta, cuda)
    out = stages.context(layer, _t(z['h'], cuda), _t(z['tokens'], cuda), half=half)
    tol = TOL_BF16 if half else 1e-5
    assert rel_err(out['Qc'].float().cpu().numpy(), z['Qc']) <= tol
    assert rel_err(out['Kc'].float().cpu().numpy(), z['Kc']) <= tol
    assert rel_err(out['beta'].cpu().numpy(), z['beta']) <= 1e-5
    assert rel_err(out['log_alfa'].cpu().numpy(), z['log_alfa']) <= 1e-5
    assert np.array_equal(out['sig'].cpu().numpy(), z['sig'])
    Bt = stages.clock(out['beta'])
    assert rel_err(Bt.cpu().numpy(), z['Bt']) <= 1e-6


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_hash_projection_matches_reference(name, cuda):
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    layer = _layer(params, meta, cuda)
    out = stages.hash(layer, _t(z['E'], cuda), half=half)
    assert rel_err(out['phi'].float().cpu().numpy(), z['phi']) <= (TOL_BF16 if half else 1e-5)
    B, L, T = z['ids'].shape
    ids = stages.ids_rows_to_btl(out['ids_rows'], B, T).cpu().numpy()
    agree = check_ids_agree(ids, z['ids'], z['phi'], layer.n_bits, half)
    assert agree >= 0.99
    if half:
        assert np.array_equal(out['Ea'].float().cpu().numpy(), O.bf16(z['E']))


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_scoring_of_reference_intermediates_matches_reference(name, cuda):
    """_acumular fed with the reference's own phi / Qc / Kc / clock / sort: signals and the copied output."""
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    layer = _layer(params, meta, cuda)
    B, L, T = z['ids'].shape
    rows = z['ids'].transpose(0, 2, 1).reshape(B * T, L)
    ids_o = np.take_along_axis(rows, z['orden'], -1).astype(np.int16)
    Ea = O.bf16(z['E']) if half else z['E']
    out = stages.score(layer, _t(z['orden'], cuda), _t(ids_o, cuda), _t(z['phi'], cuda), _t(z['Qc'], cuda),
                       _t(z['Kc'], cuda), _t(z['sig'], cuda), _t(z['Bt'], cuda), _t(z['log_alfa'], cuda),
                       _t(Ea, cuda), half=half)
    senal = z['senal'].transpose(0, 2, 1, 3)                                     # (B, L, T, 3)
    assert np.array_equal(out['hay'].cpu().numpy(), senal[..., 0].astype(np.uint8))
    hay = senal[..., 0] > 0
    assert rel_err(out['mx'].cpu().numpy()[hay], senal[..., 1][hay]) <= (1e-3 if half else 1e-5)
    assert np.all(out['mx'].cpu().numpy()[~hay] == -1e9)
    assert rel_err(out['pk'].cpu().numpy(), senal[..., 2]) <= (1e-3 if half else 1e-5)
    Wv = torch.from_numpy(params['v.weight']).to(cuda).double()
    salida = (out['acc'].double() @ Wv.T).cpu().numpy()
    assert rel_err(salida, z['salida']) <= (TOL_BF16 if half else TOL_F32)


@pytest.mark.parametrize('name', LAYER_FIXTURES)
def test_layer_forward_matches_reference(name, cuda):
    """End to end through ASRNLayer.forward (the drop-in API): h' and h' - h against the reference."""
    import asrn_b200
    from asrn_b200 import stages
    z, params, meta = load_fixture(name)
    half = bool(meta['bf16'])
    layer = _layer(params, meta, cuda)
    E, h, x = _t(z['E'], cuda), _t(z['h'], cuda), _t(z['tokens'], cuda)
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
        y = layer(E, h, x)
    assert y.dtype == torch.float32 and y.shape == h.shape
    y = y.cpu().numpy()
    B, L, T = z['ids'].shape
    ids = stages.ids_rows_to_btl(stages.hash(layer, E, half=half)['ids_rows'], B, T).cpu().numpy()
    check_ids_agree(ids, z['ids'], z['phi'], layer.n_bits, half)
    if np.array_equal(ids, z['ids']):
        ref = z['out']
    else:                                                  # compare with the oracle conditioned on our bucket ids
        lay = O.Layer(params, meta['d'], **layer_options(meta))
        ref = O.layer_forward(lay, z['E'], z['h'], z['tokens'], half=half, ids_override=ids)
    tol = TOL_BF16 if half else TOL_F32
    assert rel_err(y, ref) <= tol
    assert rel_err(y - z['h'], ref - z['h']) <= tol


@pytest.mark.parametrize('d,B,L,half,opts', [
    (256, 2, 1024, False, {}),
    (768, 1, 640, True, {}),
    (64, 3, 700, False, dict(chunk=8, n_bits=5, confirmar=20, sufijo=6, vistos=3)),
    (48, 2, 333, True, dict(chunk=16, n_bits=4)),
])
def test_layer_forward_matches_oracle_on_seeded_inputs(d, B, L, half, opts, cuda):
    """Seeded Zipf + planted-repeat inputs (the benchmark distribution), moved parameters, vs the CPU oracle."""
    import asrn_b200
    from asrn_b200 import stages, synthetic
    torch.manual_seed(0)
    layer = asrn_b200.ASRNLayer(d, **opts)
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for n, p in layer.named_parameters():
            if n in ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha', 'cq.weight',
                     'w_sufijo', 'w_vistos', 'g_conf.weight', 'g_conf.bias'):
                p.add_(torch.randn(p.shape, generator=g) * 0.5)
        layer.gamma.copy_(torch.linspace(0.5, 3.0, layer.n_tablas))
    V = 512
    x = synthetic.zipf_tokens(B, L, V, 1.1, seed=3)
    x = synthetic.plant_repeats(x, 0.25, 8, 64, seed=4)
    table = np.random.default_rng(5).standard_normal((V, d)).astype(np.float32)
    E = table[x]
    h = np.random.default_rng(6).standard_normal((B, L, d)).astype(np.float32)
    layer = layer.to(cuda).eval()
    with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
        y = layer(_t(E, cuda), _t(h, cuda), _t(x, cuda)).cpu().numpy()
    ids = stages.ids_rows_to_btl(stages.hash(layer, _t(E, cuda), half=half)['ids_rows'], B, layer.n_tablas)
    ids = ids.cpu().numpy()
    params = {k: v.detach().cpu().numpy() for k, v in layer.state_dict().items()}
    lay = O.Layer(params, d, **opts)
    parts = O.layer_forward(lay, E, h, x, half=half, return_parts=True, ids_override=ids)
    ids_oracle = O.ids_de(O.phi_y_valores(lay, E, half)[0], layer.n_tablas, layer.n_bits)
    check_ids_agree(ids, ids_oracle, O.phi_y_valores(lay, E, half)[0], layer.n_bits, half)
    tol = TOL_BF16 if half else TOL_F32
    assert rel_err(y, parts['out']) <= tol
    assert rel_err(y - h, parts['out'] - h) <= tol


def test_causality_future_does_not_change_past(cuda):
    """Changing tokens after t0 leaves h' before t0 unchanged (tests/test_nucleo.py:1201-1217)."""
    import asrn_b200
    torch.manual_seed(0)
    layer = asrn_b200.ASRNLayer(64).to(cuda).eval()
    with torch.no_grad():
        layer.gamma.copy_(torch.linspace(0.5, 3.0, 8))
        layer.w_sufijo.normal_(std=0.5)
    B, L, t0 = 2, 600, 300
    g = torch.Generator().manual_seed(2)
    x = torch.randint(0, 20, (B, L), generator=g)
    table = torch.randn(20, 64, generator=g)
    h = torch.randn(B, L, 64, generator=g)
    x2 = x.clone()
    x2[:, t0:] = torch.randint(0, 20, (B, L - t0), generator=g)
    h2 = h.clone()
    h2[:, t0:] = torch.randn(B, L - t0, 64, generator=g)
    with torch.no_grad():
        y1 = layer(table[x].to(cuda), h.to(cuda), x.to(cuda))
        y2 = layer(table[x2].to(cuda), h2.to(cuda), x2.to(cuda))
    d = (y1[:, :t0] - y2[:, :t0]).abs().max().item()
    assert d <= 1e-5 * y1[:, :t0].abs().max().item()


def test_signatures_from_vectors_when_no_token_ids(cuda):
    """piezas=None: the signature is E . r_firma (asrn/nucleo.py:634-637)."""
    from asrn_b200 import stages
    z, params, meta = load_fixture('layer_f32')
    layer = _layer(params, meta, cuda)
    E = _t(z['E'], cuda)
    out = stages.context(layer, _t(z['h'], cuda), None, E=E)
    want = z['E'] @ params['r_firma']
    assert rel_err(out['sig'].cpu().numpy(), want) <= 1e-5
    with torch.no_grad():
        y = layer(E, _t(z['h'], cuda), None)
    assert torch.isfinite(y).all()


@pytest.mark.parametrize('d,B,L', [(768, 2, 1000), (64, 3, 300), (256, 1, 4096)])
def test_tensor_core_gemms_match_cuda_core_kernels(d, B, L, cuda):
    """The tcgen05 hash projection and gate GEMM (bf16) against the CUDA-core kernels on the same inputs: bf16 E copy
    bit-exact, phi within bf16 rounding, bucket ids equal except on bits whose phi is within rounding of 0, h' within
    the bf16 tolerance, and the device status word clean (no bounded wait timed out)."""
    import asrn_b200
    from asrn_b200 import _lib, stages
    torch.manual_seed(0)
    layer = asrn_b200.ASRNLayer(d).to(cuda).eval()
    with torch.no_grad():
        layer.gamma.copy_(torch.linspace(0.5, 3.0, 8))
        layer.cq.weight.normal_(std=0.3)
    g = torch.Generator().manual_seed(4)
    x = torch.randint(0, 300, (B, L), generator=g)
    x[:, L // 2:L // 2 + L // 4] = x[:, :L // 4]
    E = (torch.randn(300, d, generator=g)[x]).to(cuda)
    h = torch.randn(B, L, d, generator=g).to(cuda)

    def run():
        hs = stages.hash(layer, E, half=True)
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            y = layer(E, h, x.to(cuda))
        return hs, y

    outs = {'tc': run()}
    with _lib.force_cuda_core():
        outs['simt'] = run()
    assert _lib.gemm_override() is None
    (h_tc, y_tc), (h_si, y_si) = outs['tc'], outs['simt']
    assert torch.equal(h_tc['Ea'], h_si['Ea'])
    phi_tc, phi_si = h_tc['phi'].float().cpu().numpy(), h_si['phi'].float().cpu().numpy()
    assert rel_err(phi_tc, phi_si) <= 2e-2
    ids_tc = stages.ids_rows_to_btl(h_tc['ids_rows'], B, 8).cpu().numpy()
    ids_si = stages.ids_rows_to_btl(h_si['ids_rows'], B, 8).cpu().numpy()
    check_ids_agree(ids_tc, ids_si, phi_si, layer.n_bits, True)
    if np.array_equal(ids_tc, ids_si):
        assert rel_err(y_tc.cpu().numpy(), y_si.cpu().numpy()) <= TOL_BF16
        assert rel_err((y_tc - h).cpu().numpy(), (y_si - h).cpu().numpy()) <= TOL_BF16
    w, _keep, prep = layer.prepared(cuda, True)
    cfg = _lib.make_config(layer, B, L, True)
    import ctypes
    assert _lib.lib().asrn_layer_status(ctypes.byref(cfg), _lib.ptr(prep), 0, _lib.stream_ptr(cuda)) == 0


def test_bounded_wait_gives_up_and_the_context_stays_usable(cuda):
    """A bounded mbarrier wait (the one every tcgen05 kernel uses) on a barrier nothing arrives on, with a 50 ms
    limit: the kernel returns, ASRN_ERR_TIMEOUT is in the status word, its TMEM is freed (a second probe can allocate
    it again) and the next layer forward runs and is correct."""
    import time
    from asrn_b200 import _lib
    lib = _lib.lib()
    for _ in range(2):
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        result = torch.full((1,), 7, dtype=torch.int32, device=cuda)
        t0 = time.perf_counter()
        assert lib.asrn_test_bounded_wait(50_000_000, _lib.ptr(status), _lib.ptr(result), _lib.stream_ptr(cuda)) == 0
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert int(status.item()) == _lib.ASRN_ERR_TIMEOUT
        assert int(result.item()) == 0
        assert 0.04 <= elapsed < 5.0
    z, params, meta = load_fixture('layer_f32')
    layer = _layer(params, meta, cuda)
    with torch.no_grad():
        y = layer(_t(z['E'], cuda), _t(z['h'], cuda), _t(z['tokens'], cuda)).cpu().numpy()
    assert rel_err(y, z['out']) <= TOL_F32


@pytest.mark.parametrize('B,L', [(1, 262144), (3, 40961), (2, 4096), (5, 1), (1, 4097)])
def test_clock_scan_long_and_ragged_rows(B, L, cuda):
    """asrn_clock (B_t = cumsum(beta) in fp64; one block per 4096-slot chunk, which sums the chunks before it itself)
    against numpy's fp64 cumsum: within 1e-12 of the row's largest value (the sums run in another order)."""
    from asrn_b200 import stages
    rng = np.random.default_rng(B * 7 + L)
    beta = rng.gamma(1.5, 0.7, size=(B, L))
    got = stages.clock(torch.from_numpy(beta).to(cuda)).cpu().numpy()
    ref = np.cumsum(beta, axis=1)
    assert np.abs(got - ref).max() <= 1e-12 * np.abs(ref).max()
