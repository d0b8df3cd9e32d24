"""Model files in the reference's format (asrn/nucleo.py:2050-2133): a file written by the reference's own guardar()
(tests/golden/ckpt_ref.pt, made by tests/golden/make_golden.py), the same weights in the v86 layout (streak response
per node, 'u_racha'), and this package's guardar() -> cargar() round trip. The GPU test runs the loaded model and
compares its logits with the reference's (fp32, 1e-4)."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err


def _ref_state():
    return torch.load(os.path.join(GOLDEN, 'ckpt_ref.pt'), map_location='cpu', weights_only=True)


def test_loads_a_file_written_by_the_reference():
    import asrn_b200
    r = _ref_state()
    m = asrn_b200.cargar(os.path.join(GOLDEN, 'ckpt_ref.pt'), dispositivo='cpu')
    assert m.config == r['config']
    ours = m.state_dict()
    assert sorted(ours) == sorted(r['pesos'])
    for k, v in r['pesos'].items():
        assert torch.equal(ours[k], v), k
    assert not m.training


def test_loads_a_v86_file_with_the_per_node_streak_response():
    import asrn_b200
    r = _ref_state()
    m = asrn_b200.load(os.path.join(GOLDEN, 'ckpt_ref_v86.pt'), dispositivo='cpu')
    for k, v in r['pesos'].items():
        if k.endswith('d_racha'):
            assert torch.allclose(m.state_dict()[k], v, rtol=0, atol=1e-6), k
        else:
            assert torch.equal(m.state_dict()[k], v), k


def test_save_then_load_round_trip_and_rejects_foreign_files(tmp_path):
    import asrn_b200
    m = asrn_b200.create_model(V=40, d=16, n_capas=2, semilla=3, chunk=8, n_bits=3)
    path = str(tmp_path / 'm.pt')
    asrn_b200.save(m, path)
    r = torch.load(path, map_location='cpu', weights_only=True)
    assert set(r) == {'config', 'pesos'} and r['config'] == m.config
    m2 = asrn_b200.cargar(path, dispositivo='cpu')
    for k, v in m.state_dict().items():
        assert torch.equal(m2.state_dict()[k], v), k
    torch.save({'pesos': {}}, str(tmp_path / 'bad.pt'))
    with pytest.raises(ValueError):
        asrn_b200.cargar(str(tmp_path / 'bad.pt'), dispositivo='cpu')
    with pytest.raises(FileNotFoundError):
        asrn_b200.cargar(str(tmp_path / 'missing.pt'))


@pytest.mark.gpu
def test_model_loaded_from_a_reference_file_matches_the_reference_logits(cuda):
    import asrn_b200
    z = np.load(os.path.join(GOLDEN, 'ckpt_ref.npz'))
    old = (torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32)
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        m = asrn_b200.cargar(os.path.join(GOLDEN, 'ckpt_ref.pt'), dispositivo=cuda)
        with torch.no_grad():
            lg = m(torch.from_numpy(z['tokens']).to(cuda)).cpu().numpy()
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = old
    assert rel_err(lg, z['logits']) <= 1e-4
