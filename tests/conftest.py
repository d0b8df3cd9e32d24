import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, 'tests', 'golden')
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200); runs the kernels of libasrn_b200.so')


def load_fixture(name):
    """(arrays, params, meta) of tests/golden/<name>.npz (made from the reference by tests/golden/make_golden.py)."""
    z = np.load(os.path.join(GOLDEN, name + '.npz'))
    arrays = {k: z[k] for k in z.files if not k.startswith(('param.', 'meta.'))}
    params = {k[6:]: z[k] for k in z.files if k.startswith('param.')}
    meta = {k[5:]: z[k].item() for k in z.files if k.startswith('meta.')}
    return arrays, params, meta


LAYER_FIXTURES = ['layer_f32', 'layer_bf16', 'layer_f32_opts', 'layer_f32_d96', 'layer_f32_short', 'layer_f32_one',
                  'layer_bf16_d256', 'layer_f32_d256']

LAYER_OPTION_KEYS = ('n_tablas', 'n_bits', 'afin_oculto', 'chunk', 'tablas_contexto', 'confirmar', 'sufijo', 'vistos',
                     'nodos_racha', 'racha_max')


def layer_options(meta):
    return {k: v for k, v in meta.items() if k in LAYER_OPTION_KEYS}


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-12)) if b.size else 0.0


# A bucket bit is the sign of one phi value. An implementation that sums in another order moves phi by about 5e-7 of
# max|phi| in fp32 and 2e-3 in bf16 autocast (the reference's rounding chain with fp32 instead of fp64 accumulation,
# measured on the benchmark's shapes); a bit may differ from the reference only where |phi_ref| is below these bounds.
FLIP_BOUND_F32 = 1e-5
FLIP_BOUND_BF16 = 1e-2


def check_ids_agree(ids_got, ids_ref, phi_ref, nb, half):
    """Our bucket ids differ from the reference's only on bits whose phi is within rounding of zero for the
    precision (fp32: 1e-5 max|phi|, bf16: 1e-2 max|phi|). Returns the fraction of equal (position, table) ids."""
    if np.array_equal(ids_got, ids_ref):
        return 1.0
    B, L, T = ids_ref.shape
    diff = np.asarray(ids_got, np.int64) ^ np.asarray(ids_ref, np.int64)
    bits = (diff[..., None] >> np.arange(nb)) & 1                           # (B, L, T, nb)
    ph = np.abs(np.asarray(phi_ref, np.float32).reshape(B, L, T, nb))
    bound = (FLIP_BOUND_BF16 if half else FLIP_BOUND_F32) * np.abs(phi_ref).max()
    flipped = ph[bits.astype(bool)]
    assert (flipped <= bound).all(), (f'a bucket bit flipped on a phi far from zero: |phi| {flipped.max():.3e} > '
                                      f'{bound:.3e}')
    return float((ids_got == ids_ref).mean())


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('GPU test selected but no CUDA device is visible')
    return torch.device('cuda:0')
