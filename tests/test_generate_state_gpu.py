"""The O(1) writer's device state against the reference's own (tests/golden/gen_state.npz, made by running
_Escritor(o1=True), asrn/nucleo.py:1717-1854, on a model whose rings overflow: chunk 4, 2 bits per table).

After the prompt and after every step, for every ASRN layer:
  rings and counts bit-exact (_anillo_desde / _anillo_meter, asrn/nucleo.py:1585-1618);
  the step's candidate positions bit-exact: the ring row of the new token's bucket in every table before the step
  (_candidatos, asrn/nucleo.py:1621-1631), with the new token's bucket ids equal to the reference's;
  the Hawkes table: the same set of n-gram keys per (sequence, order), bit-exact, with the clock of the key's last
  occurrence (Bu) within 1e-6 and A = lambda + alfa within 1e-5 (_MemoriaHawkes, asrn/nucleo.py:1634-1714);
and the step logits within 1e-4 (fp32).
"""
import numpy as np
import pytest
import torch

from conftest import load_fixture, rel_err

pytestmark = pytest.mark.gpu

EMPTY_KEY = 0xFFF8000000000001
ENTRY = np.dtype([('key', '<u8'), ('bu', '<f8'), ('a', '<f4'), ('last', '<i4')])


@pytest.fixture(autouse=True)
def _exact_fp32_torch_ops():
    old = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = old


def _key_bits(k):
    k = np.where(k == 0.0, 0.0, k)                    # -0.0 and +0.0 are one key
    return np.asarray(k, np.float64).view(np.uint64)


def _ids_of_phi(phi, T, nb):
    bits = (phi.reshape(*phi.shape[:-1], T, nb) > 0).astype(np.int64)
    return (bits << np.arange(nb)).sum(-1)


def _check_hawkes(st, z, pre, B, n):
    tab = st.table.cpu().numpy().view(ENTRY).reshape(B, n, st.hcap)
    bj = z[pre + 'hawkes_bj']
    keys, bu, A = _key_bits(z[pre + 'hawkes_key']), z[pre + 'hawkes_bu'], z[pre + 'hawkes_a']
    for b in range(B):
        for j in range(n):
            sel = (bj[:, 0] == b) & (bj[:, 1] == j)
            ours = tab[b, j][tab[b, j]['key'] != EMPTY_KEY]
            assert ours.size == sel.sum(), (pre, b, j, ours.size, sel.sum())
            o = np.argsort(ours['key'])
            r = np.argsort(keys[sel])
            assert np.array_equal(ours['key'][o], keys[sel][r]), (pre, b, j)
            assert rel_err(ours['bu'][o], bu[sel][r]) <= 1e-6, (pre, b, j)
            assert rel_err(ours['a'][o], A[sel][r]) <= 1e-5, (pre, b, j)


@pytest.mark.parametrize('ajeno', [True, False], ids=['ajeno', 'propia'])
def test_writer_state_matches_reference(ajeno, cuda):
    import asrn_b200
    z, params, meta = load_fixture('gen_state')
    tag = 'ajeno' if ajeno else 'propia'
    m = asrn_b200.create_model(V=meta['V'], d=meta['d'], n_capas=meta['n_capas'], largo_cada=meta['largo_cada'],
                               chunk=meta['chunk'], n_bits=meta['n_bits'])
    m.load_state_dict({k: torch.from_numpy(np.asarray(v)) for k, v in params.items()})
    m = m.to(cuda).eval()
    B, L0, n_new = meta['B'], meta['L0'], meta['n_new']
    x = torch.from_numpy(z['tokens']).to(cuda)
    w = asrn_b200.Writer(m, memoria_de_lo_ajeno=ajeno, grafo=False)
    logits = [w.inicio(x[:, :L0], capacidad=L0 + n_new)]
    T, nb = m.largos[0].n_tablas, m.largos[0].n_bits
    for j, st in enumerate(w.layers):
        pre = f'{tag}.prompt.l{j}.'
        ids = _ids_of_phi(st.phi[:, :L0].float().cpu().numpy(), T, nb)
        assert np.array_equal(ids, z[pre + 'ids']), f'layer {j}: prompt bucket ids differ from the reference'
        assert np.array_equal(st.ring.cpu().numpy(), z[pre + 'ring']), pre
        assert np.array_equal(st.count.cpu().numpy().astype(np.int64), z[pre + 'count']), pre
        _check_hawkes(st, z, pre, B, st.capa.vistos)
    for k in range(n_new - 1):
        t = L0 + k
        rings_before = [st.ring.clone() for st in w.layers]
        logits.append(w.paso(x[:, t]))
        for j, st in enumerate(w.layers):
            pre = f'{tag}.step{k}.l{j}.'
            ids_t = _ids_of_phi(st.phi[:, t].float().cpu().numpy(), T, nb)
            assert np.array_equal(ids_t, z[pre + 'ids_t']), pre
            rb = rings_before[j].cpu().numpy()
            cand = rb[np.arange(B)[:, None], np.arange(T)[None, :], ids_t]
            assert np.array_equal(cand, z[pre + 'cand']), pre
            assert np.array_equal(st.ring.cpu().numpy(), z[pre + 'ring']), pre
            assert np.array_equal(st.count.cpu().numpy().astype(np.int64), z[pre + 'count']), pre
            _check_hawkes(st, z, pre, B, st.capa.vistos)
    assert rel_err(torch.stack(logits, 1).cpu().numpy(), z[f'{tag}.logits']) <= 1e-4
    assert all(s == 0 for s in w.status())
