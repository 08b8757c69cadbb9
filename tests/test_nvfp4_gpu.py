"""GPU parity of the NVFP4 packers against the numpy oracle, bit for bit, through the C ABI."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_ref as R

pytestmark = pytest.mark.gpu


def _mats():
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((384, 1024)) * 0.02).astype(np.float32)
    b = (rng.standard_normal((128, 3584)) * 0.5).astype(np.float32)
    c = np.zeros((256, 64), dtype=np.float32)
    c[3, :16] = 4000.0                 # saturating scale
    c[5, 16:32] = 1e-9                 # below the scale floor
    t = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], dtype=np.float32)
    c[7, :8] = t; c[7, 8:16] = -t      # ties of both quantisers (amax 6 -> scale 1)
    c[9, 32:48] = np.linspace(-3, 3, 16)
    return [a, b, c]


@pytest.mark.parametrize("idx", [0, 1, 2])
def test_tensor_core_layout_bit_exact(idx):
    from qwen35_b200.model import _quantize_matrix_nvfp4_lm
    w = torch.from_numpy(_mats()[idx]).bfloat16()
    ref_p, ref_s = R.quantize_nvfp4_lm(w.float().numpy())
    got = _quantize_matrix_nvfp4_lm(w.cuda())
    assert np.array_equal(got["packed"].cpu().numpy(), ref_p)
    assert np.array_equal(got["scales"].cpu().numpy(), ref_s)


@pytest.mark.parametrize("idx,group", [(0, 32), (1, 32), (2, 32), (0, 16), (1, 64)])
def test_decode_body_layout_bit_exact(idx, group):
    from qwen35_b200.model import _quantize_matrix_nvfp4
    w = torch.from_numpy(_mats()[idx]).bfloat16()
    ref_p, ref_s = R.quantize_nvfp4(w.float().numpy(), group)
    got = _quantize_matrix_nvfp4(w.cuda(), group)
    assert np.array_equal(got["packed"].cpu().numpy(), ref_p)
    assert np.array_equal(got["scales"].cpu().numpy().view(np.uint16), ref_s.view(np.uint16))


def test_padded_rows_and_errors():
    from qwen35_b200.model import _quantize_matrix_nvfp4, _quantize_matrix_nvfp4_lm, _quantize_matrix_nvfp4_tc
    w = (torch.randn(200, 128) * 0.1).bfloat16().cuda()
    q = _quantize_matrix_nvfp4_tc(w)
    assert q["padded_rows"] == 256 and q["packed"].shape == (256, 64)
    ref_p, ref_s = R.quantize_nvfp4_lm(torch.cat([w.cpu().float(), torch.zeros(56, 128)]).numpy())
    assert np.array_equal(q["packed"].cpu().numpy(), ref_p) and np.array_equal(q["scales"].cpu().numpy(), ref_s)
    with pytest.raises(ValueError):
        _quantize_matrix_nvfp4_lm(w)                      # 200 rows
    with pytest.raises(ValueError):
        _quantize_matrix_nvfp4(w, 48)
    with pytest.raises(TypeError):
        _quantize_matrix_nvfp4(w.float(), 32)
