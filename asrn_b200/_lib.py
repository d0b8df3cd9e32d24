"""ctypes binding of libasrn_b200.so (the C ABI declared in include/asrn_b200.h).

The library is loaded from the package directory (built in-tree by asrn_b200.build). There is no fallback: if the
library is missing or was built for another ABI version, every entry point raises.
"""
import ctypes
import math
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libasrn_b200.so')
ABI_VERSION = 4

ASRN_OK, ASRN_ERR_ARG, ASRN_ERR_UNSUPPORTED, ASRN_ERR_WORKSPACE, ASRN_ERR_CUDA, ASRN_ERR_TIMEOUT, ASRN_ERR_DATA = range(7)


class LayerConfig(ctypes.Structure):
    _fields_ = [('B', ctypes.c_int64), ('L', ctypes.c_int64), ('d', ctypes.c_int64),
                ('n_tablas', ctypes.c_int32), ('n_bits', ctypes.c_int32), ('chunk', ctypes.c_int32),
                ('tablas_contexto', ctypes.c_int32), ('confirmar', ctypes.c_int32), ('sufijo', ctypes.c_int32),
                ('vistos', ctypes.c_int32), ('nodos_racha', ctypes.c_int32), ('hidden', ctypes.c_int32),
                ('half', ctypes.c_int32), ('beta_max', ctypes.c_float), ('log_alfa_min', ctypes.c_float),
                ('mejor_max', ctypes.c_float), ('tope_puerta', ctypes.c_float), ('kappa_min', ctypes.c_float),
                ('racha_paso', ctypes.c_double)]


WEIGHT_FIELDS = ['ln_w', 'ln_b', 'cq', 'ck', 'w_reloj', 'b_reloj', 'pal0_w', 'pal0_b', 'pal2_w', 'pal2_b', 'ctx0_w',
                 'ctx0_b', 'ctx2_w', 'ctx2_b', 'v_w', 'o_w', 'g_w', 'g_b', 'g_conf_w', 'g_conf_b', 'w_vistos',
                 'u_hawkes', 'log_kappa', 'log_kappa_racha', 'w_sufijo', 'gamma', 'd_racha', 'c_vistos', 'r_firma']

# state_dict name of each field (asrn/nucleo.py:585-630)
WEIGHT_NAMES = {'ln_w': 'ln_ctx.weight', 'ln_b': 'ln_ctx.bias', 'cq': 'cq.weight', 'ck': 'ck.weight',
                'w_reloj': 'w_reloj', 'b_reloj': 'b_reloj', 'pal0_w': 'afin_palabra.0.weight',
                'pal0_b': 'afin_palabra.0.bias', 'pal2_w': 'afin_palabra.2.weight', 'pal2_b': 'afin_palabra.2.bias',
                'ctx0_w': 'afin_contexto.0.weight', 'ctx0_b': 'afin_contexto.0.bias',
                'ctx2_w': 'afin_contexto.2.weight', 'ctx2_b': 'afin_contexto.2.bias', 'v_w': 'v.weight',
                'o_w': 'o.weight', 'g_w': 'g.weight', 'g_b': 'g.bias', 'g_conf_w': 'g_conf.weight',
                'g_conf_b': 'g_conf.bias', 'w_vistos': 'w_vistos', 'u_hawkes': 'u_hawkes', 'log_kappa': 'log_kappa',
                'log_kappa_racha': 'log_kappa_racha', 'w_sufijo': 'w_sufijo', 'gamma': 'gamma',
                'd_racha': 'd_racha', 'c_vistos': 'c_vistos', 'r_firma': 'r_firma'}


class LayerWeights(ctypes.Structure):
    _fields_ = [(f, ctypes.c_void_p) for f in WEIGHT_FIELDS]


_lib = None

_P = ctypes.c_void_p
_SIGS = {
    'asrn_status_string': (ctypes.c_char_p, [ctypes.c_int]),
    'asrn_abi_version': (ctypes.c_int, []),
    'asrn_layer_prepared_bytes': (ctypes.c_size_t, [_P]),
    'asrn_layer_prepare': (ctypes.c_int, [_P, _P, _P, ctypes.c_size_t, _P]),
    'asrn_layer_status': (ctypes.c_int, [_P, _P, ctypes.c_int, _P]),
    'asrn_layer_workspace_bytes': (ctypes.c_size_t, [_P]),
    'asrn_layer_forward': (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    'asrn_context': (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    'asrn_clock': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _P, _P, _P]),
    'asrn_hash': (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P]),
    'asrn_ids_from_phi': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _P, _P, _P]),
    'asrn_bucket_sort_workspace_bytes': (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]),
    'asrn_bucket_sort': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P,
                                        ctypes.c_size_t, _P]),
    'asrn_score': (ctypes.c_int, [_P] * 17),
    'asrn_bucket_sort_noalloc': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P]),
    'asrn_candidates': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       _P, _P, _P, _P, _P, _P]),
    'asrn_repetition_workspace_bytes': (ctypes.c_size_t, [_P]),
    'asrn_repetition': (ctypes.c_int, [_P] * 14 + [ctypes.c_size_t, _P]),
    'asrn_gen_ring_build': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_int64, _P, _P, _P, _P, _P]),
    'asrn_gen_hawkes_table_bytes': (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int64]),
    'asrn_gen_hawkes_build': (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, ctypes.c_int64, _P, _P, _P, _P, _P,
                                             ctypes.c_int64, _P]),
    'asrn_gen_attend': (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int64] + [_P] * 22),
    'asrn_gen_memory': (ctypes.c_int, [_P] * 4 + [ctypes.c_int64] + [_P] * 6 + [ctypes.c_int64] + [_P] * 5),
    'asrn_gen_ring_insert': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            _P, _P, _P, _P, _P]),
    'asrn_gen_front': (ctypes.c_int, [_P] * 17),
    'asrn_gen_front_residual': (ctypes.c_int, [_P] * 19),
    'asrn_local_in': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, _P,
                                     ctypes.c_float, _P, ctypes.c_int32, _P]),
    'asrn_local_mid': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P, _P, ctypes.c_float, _P,
                                      ctypes.c_int32, _P]),
    'asrn_local_gelu': (ctypes.c_int, [ctypes.c_int64, _P, ctypes.c_int32, _P]),
    'asrn_shard_rows': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
                                       _P, _P, ctypes.c_int64, _P, _P, _P, _P]),
    'asrn_score_shard': (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64] + [_P] * 15),
    'asrn_ngram_chunk_workspace_bytes': (ctypes.c_size_t, [_P]),
    'asrn_ngram_chunk_sort': (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, ctypes.c_int64] + [_P] * 6 +
                              [ctypes.c_size_t, _P]),
    'asrn_ngram_chunk_finish': (ctypes.c_int, [_P, _P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32] +
                                [_P] * 8 + [ctypes.c_size_t, _P]),
    'asrn_racha_workspace_bytes': (ctypes.c_size_t, [_P]),
    'asrn_racha_chunk': (ctypes.c_int, [_P] * 8 + [_P, ctypes.c_size_t, _P]),
    'asrn_shard_workspace_bytes': (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32]),
    'asrn_shard_tails': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                        _P, _P, _P, _P, ctypes.c_size_t, _P]),
    'asrn_shard_merge': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                        ctypes.c_int32, _P, _P, _P, ctypes.c_int64, _P, _P, _P, ctypes.c_int64, _P,
                                        ctypes.c_size_t, _P, _P]),
    'asrn_gen_gate': (ctypes.c_int, [_P] * 16),
    'asrn_gate_workspace_bytes': (ctypes.c_size_t, [_P]),
    'asrn_gate': (ctypes.c_int, [_P] * 14 + [ctypes.c_size_t, _P]),
    'asrn_ngram_shared_bytes': (ctypes.c_size_t, [_P]),
    'asrn_ngram_shared_sort': (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_size_t, _P, ctypes.c_size_t, _P]),
    'asrn_layer_forward_ngram': (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P, _P, ctypes.c_size_t,
                                                _P]),
    'asrn_local_block_workspace_bytes': (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                                           ctypes.c_int32]),
    'asrn_local_block': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        _P, _P, _P, _P, ctypes.c_float, _P, _P, _P, _P, ctypes.c_float, _P, _P, _P, _P,
                                        _P, ctypes.c_size_t, _P, _P]),
    'asrn_bucket_attn_forward': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64] + [ctypes.c_int32] * 6 + [_P] * 12
                                 + [ctypes.c_float, ctypes.c_float, ctypes.c_int32, _P, _P, _P]),
    'asrn_bucket_attn_backward': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64] + [ctypes.c_int32] * 6 + [_P] * 12
                                  + [ctypes.c_float, ctypes.c_float, ctypes.c_int32] + [_P] * 11),
    'asrn_scan_forward': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _P, _P, _P, _P]),
    'asrn_scan_backward': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _P, _P, _P, _P, _P, _P]),
    'asrn_argmax_rows': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_int32, _P, _P]),
    'asrn_sampler_seed_state': (ctypes.c_int, [ctypes.c_uint64, _P]),
    'asrn_sampler_jump_poly': (ctypes.c_int, [ctypes.c_uint64, _P]),
    'asrn_sampler_fill': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _P, _P, _P, _P, _P]),
    'asrn_sample_argmax': (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, _P, _P, _P, _P, _P]),
    'asrn_test_force_cuda_core': (ctypes.c_int, [ctypes.c_int]),
    'asrn_test_bounded_wait': (ctypes.c_int, [ctypes.c_uint64, _P, _P, _P]),
}


def exported_symbols():
    """Names the C ABI exports (the entry points of include/asrn_b200.h)."""
    return sorted(_SIGS)


def lib():
    """The loaded library (loads it on first use; raises if it is missing or of another ABI version)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f'{LIB_PATH} is missing: build it with `python -m asrn_b200.build` '
                               '(the CUDA kernels are the only implementation; there is no fallback)')
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        v = handle.asrn_abi_version()
        if v != ABI_VERSION:
            raise RuntimeError(f'libasrn_b200.so ABI version {v}, expected {ABI_VERSION}: rebuild it')
        _lib = handle
    return _lib


def gemm_override():
    """'cuda_core' while the test hook asrn_test_force_cuda_core holds the bf16 work on the CUDA-core kernels, else
    None (the default: tensor cores)."""
    return 'cuda_core' if lib().asrn_test_force_cuda_core(-1) else None


class force_cuda_core:
    """Test hook as a context manager: the bf16 work inside runs on the CUDA-core kernels."""

    def __enter__(self):
        self.prev = lib().asrn_test_force_cuda_core(1)
        return self

    def __exit__(self, *exc):
        lib().asrn_test_force_cuda_core(self.prev)
        return False


def check(status, what):
    if status != ASRN_OK:
        msg = lib().asrn_status_string(status).decode()
        if status == ASRN_ERR_UNSUPPORTED:
            raise NotImplementedError(f'{what}: {msg}')
        if status in (ASRN_ERR_ARG, ASRN_ERR_WORKSPACE):
            raise ValueError(f'{what}: {msg}')
        raise RuntimeError(f'{what}: {msg}')


def make_config(layer, B, L, half):
    """LayerConfig of an ASRNLayer for a batch (B, L)."""
    p = layer.protecciones
    c = LayerConfig()
    c.B, c.L, c.d = B, L, layer.d
    c.n_tablas, c.n_bits, c.chunk = layer.n_tablas, layer.n_bits, layer.chunk
    c.tablas_contexto, c.confirmar, c.sufijo, c.vistos = layer.tablas_contexto, layer.confirmar, layer.sufijo, \
        layer.vistos
    c.nodos_racha = layer.d_racha.shape[0]
    c.hidden = layer.afin_palabra[0].out_features
    c.half = 1 if half else 0
    c.beta_max = math.inf if p.beta_max is None else p.beta_max
    c.log_alfa_min = -math.inf if p.log_alfa_min is None else p.log_alfa_min
    c.mejor_max = math.inf if p.mejor_max is None else p.mejor_max
    c.tope_puerta = 0.0 if p.tope_puerta is None else p.tope_puerta
    c.kappa_min = 0.0 if p.kappa_min is None else p.kappa_min
    c.racha_paso = layer.racha_paso
    return c


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_ptr(device):
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
