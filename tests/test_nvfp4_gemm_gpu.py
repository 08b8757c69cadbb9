"""GPU parity of the NVFP4 block-scaled tensor-core GEMM (qwen35_b200_gemm_nvfp4, through the C ABI) and of the activation
packer that feeds it.  The expected value is the exact product of the dequantised operands (numpy, f64 sums): every factor
is a product of an E2M1 value and an E4M3 scale, so the only freedom the hardware has is the order and rounding of its f32
sums."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import nvfp4_ref as R

pytestmark = pytest.mark.gpu


def _pack_weights(w):
    from qwen35_b200.model import _quantize_matrix_nvfp4_lm
    return _quantize_matrix_nvfp4_lm(w.cuda().contiguous())


def _pack_act(x):
    from qwen35_b200 import _capi
    lib = _capi.lib()
    T, K = x.shape
    sb = C.c_size_t(0)
    pb = lib.qwen35_b200_nvfp4_act_bytes(T, K, C.byref(sb))
    packed = torch.empty(pb, dtype=torch.uint8, device="cuda")
    scales = torch.empty(sb.value, dtype=torch.uint8, device="cuda")
    _capi.check(lib.qwen35_b200_quantize_act_nvfp4(x.data_ptr(), T, K, packed.data_ptr(), scales.data_ptr(),
                                                   C.c_void_p(torch.cuda.current_stream().cuda_stream)), "quantize_act_nvfp4")
    tpad = (T + 127) // 128 * 128
    return packed.view(tpad, K // 2), scales


@pytest.mark.parametrize("T,K", [(16, 1024), (5, 256), (130, 512)])
def test_activation_packer_equals_the_oracle(T, K):
    torch.manual_seed(T + K)
    x = (torch.randn(T, K) * 0.7).bfloat16()
    packed, scales = _pack_act(x.cuda())
    tpad = (T + 127) // 128 * 128
    xp = torch.zeros(tpad, K)
    xp[:T] = x.float()
    ref_p, ref_s = R.quantize_nvfp4_lm(xp.numpy())
    assert np.array_equal(packed.cpu().numpy(), ref_p)
    assert np.array_equal(scales.cpu().numpy(), ref_s)


@pytest.mark.parametrize("T,N,K,f32", [(16, 256, 1024, True), (1, 128, 256, False), (33, 384, 1024, False), (64, 1024, 3584 - 3584 % 256, False),
                                       (128, 256, 2048, False), (200, 512, 1024, False), (16, 248320, 1024, True)])
def test_gemm_nvfp4_matches_exact_product_of_dequantised_operands(T, N, K, f32):
    from qwen35_b200 import _capi
    lib = _capi.lib()
    torch.manual_seed(T * 3 + N)
    x = (torch.randn(T, K) * 0.5).bfloat16()
    w = (torch.randn(N, K) * 0.05).bfloat16()
    wq = _pack_weights(w)
    ap, asc = _pack_act(x.cuda())
    out = torch.zeros(T, N, dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
    res = None if f32 else torch.randn(T, N, device="cuda").bfloat16()
    st = lib.qwen35_b200_gemm_nvfp4(ap.data_ptr(), asc.data_ptr(), T, wq["packed"].data_ptr(), wq["scales"].data_ptr(), N, K, C.c_float(1.0),
                                    out.data_ptr(), N, 1 if f32 else 0, None if res is None else res.data_ptr(), N,
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    _capi.check(st, "gemm_nvfp4")
    _capi.check(lib.qwen35_b200_status(None), "status")
    # expected: exact products of the dequantised operands (a slab of the vocabulary for the LM-head shape)
    n_chk = min(N, 1024)
    wd = R.dequantize_nvfp4_lm(wq["packed"][:n_chk].cpu().numpy(), wq["scales"].cpu().numpy() if N == n_chk else
                               _atoms_of_rows(wq["scales"].cpu().numpy(), n_chk, K)).astype(np.float64)
    tpad = ap.shape[0]
    ad = R.dequantize_nvfp4_lm(ap.cpu().numpy(), asc.cpu().numpy()).astype(np.float64)[:T]
    ref = torch.from_numpy(ad @ wd.T)
    got = out[:, :n_chk].float().cpu()
    if f32:
        assert float((got - ref.float()).abs().max()) <= 1e-3 * float(ref.abs().max()) + 1e-5
    else:
        exp = (ref.float().bfloat16().float() + res[:, :n_chk].float().cpu()).bfloat16().float()
        assert float((got != exp).float().mean()) <= 0.02                      # an f32 sum near a bf16 rounding boundary
        assert bool(((got - exp).abs() <= (ref.float().abs() + exp.abs()) * 2.0 ** -6 + 2e-3).all())
    if N > n_chk:         # the far end of the vocabulary too
        wd2 = R.dequantize_nvfp4_lm(wq["packed"][-128:].cpu().numpy(), _atoms_of_rows(wq["scales"].cpu().numpy(), 128, K, first_block=N // 128 - 1)).astype(np.float64)
        ref2 = torch.from_numpy(ad @ wd2.T).float()
        assert float((out[:, -128:].float().cpu() - ref2).abs().max()) <= 1e-3 * float(ref2.abs().max()) + 1e-5


def _atoms_of_rows(scales, n_rows, K, first_block=0):
    """The scale atoms of row blocks [first_block, first_block + n_rows / 128) as a compact array."""
    per_block = (K // 64) * 512
    return scales[first_block * per_block:(first_block + n_rows // 128) * per_block]


def test_gemm_nvfp4_rejects_bad_shapes():
    from qwen35_b200 import _capi
    lib = _capi.lib()
    z = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    st = lib.qwen35_b200_gemm_nvfp4(z.data_ptr(), z.data_ptr(), 4, z.data_ptr(), z.data_ptr(), 100, 256, C.c_float(1.0), z.data_ptr(), 100, 0, None, 0, None)
    assert st == 2 and b"multiple of 128" in lib.qwen35_b200_last_error()
