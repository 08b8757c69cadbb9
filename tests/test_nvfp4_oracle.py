"""Known-answer tests of the NVFP4 packer oracle (oracle/nvfp4_ref.py): number formats against NVIDIA's
host conversion functions, tie and saturation cases, the swizzled scale index, pack/unpack round trips."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle import nvfp4_ref as R

HELPER = os.path.join(ROOT, "oracle", "_ref", "nvfp4_hdr_check")


def _helper(values: np.ndarray):
    if not os.path.exists(HELPER):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    bits = values.astype(np.float32).view(np.uint32)
    out = subprocess.run([HELPER], input="\n".join(f"{b:08x}" for b in bits) + "\n", capture_output=True, text=True, check=True).stdout
    rows = [line.split() for line in out.strip().splitlines()]
    e4 = np.array([int(r[1], 16) for r in rows], dtype=np.uint8)
    dec = np.array([int(r[2], 16) for r in rows], dtype=np.uint32).view(np.float32)
    e2 = np.array([int(r[3], 16) for r in rows], dtype=np.uint8)
    return e4, dec, e2


def test_formats_match_nvidia_host_conversions():
    rng = np.random.default_rng(0)
    special = np.array([0.0, 2.0 ** -28, 2.0 ** -11, 2.0 ** -10, 1.5 * 2.0 ** -10, 2.0 ** -9, 2.0 ** -7, 2.0 ** -6,
                        0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0, 447.0, 448.0, 449.0, 480.0, 1e6,
                        0.2499999, 0.2500001, 1.0625, 1.125, 1.1875], dtype=np.float32)
    vals = np.concatenate([special, np.exp(rng.uniform(np.log(1e-4), np.log(600.0), 4000)).astype(np.float32),
                           rng.uniform(0, 7, 4000).astype(np.float32)])
    e4, dec, e2 = _helper(vals)
    assert np.array_equal(R.e4m3_encode(vals), e4)
    assert np.array_equal(R.e4m3_decode(e4), dec)
    assert np.array_equal(R.e2m1_rne(vals), e2)
    neg = -vals[vals > 0]
    _, _, e2n = _helper(neg)
    assert np.array_equal(R.e2m1_rne(neg), e2n)


def test_e2m1_ties():
    t = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    assert R.e2m1_rne(t).tolist() == [0, 2, 2, 4, 4, 6, 6]            # round-to-nearest-even (tensor-core layout)
    assert R.e2m1_threshold(t).tolist() == [1, 2, 3, 4, 5, 6, 7]      # ties up (decode-body layout)
    assert R.e2m1_threshold(-t).tolist() == [9, 10, 11, 12, 13, 14, 15]
    assert R.e2m1_rne(np.array([100.0, -100.0], dtype=np.float32)).tolist() == [7, 15]


def test_all_sixteen_codes_round_trip():
    for scale in (0.001953125, 0.0625, 1.0, 8.0):
        vals = np.concatenate([R.E2M1_VALUES, -R.E2M1_VALUES[1:], [0.0] * 17]).astype(np.float32)[None, :] * np.float32(scale)
        vals = np.tile(vals[:, :32], (128, 2))                         # [128, 64]
        p, s = R.quantize_nvfp4_lm(vals)
        assert np.array_equal(R.dequantize_nvfp4_lm(p, s), vals)
        p2, s2 = R.quantize_nvfp4(vals, 32)
        assert np.allclose(R.dequantize_nvfp4(p2, s2, 32), vals, rtol=2e-3)


def test_zero_block_and_saturation():
    w = np.zeros((128, 64), dtype=np.float32)
    w[0, :16] = 4000.0                      # amax/6 = 666 -> saturates to 448
    p, s = R.quantize_nvfp4_lm(w)
    assert s[R.lm_scale_index(0, 0, 64)] == 0x7E
    assert s[R.lm_scale_index(0, 1, 64)] == 0           # floor 2^-28 rounds to zero in E4M3
    assert (p[0, :8] == 0x77).all() and (p[1:] == 0).all()
    p2, s2 = R.quantize_nvfp4(w, 32)
    assert float(s2[1, 0]) == 1.0 and (p2[1] == 0).all()


def test_swizzled_scale_index():
    cols = 1024
    expect = {}
    for row in (0, 31, 32, 127, 128):
        for sc in (0, 3, 4, 63):
            tile = (row // 128) * (cols // 64) + sc // 4
            expect[(row, sc)] = tile * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + sc % 4
    assert expect[(0, 0)] == 0 and expect[(31, 3)] == 31 * 16 + 3 and expect[(32, 0)] == 4
    assert expect[(127, 63)] == 15 * 512 + 31 * 16 + 12 + 3 and expect[(128, 4)] == 17 * 512
    for (row, sc), v in expect.items():
        assert R.lm_scale_index(row, sc, cols) == v
    # the map is a bijection onto [0, rows/128 * cols/64 * 512)
    r, c = np.meshgrid(np.arange(256), np.arange(cols // 16), indexing="ij")
    idx = R.lm_scale_index(r, c, cols).ravel()
    assert np.array_equal(np.sort(idx), np.arange(2 * (cols // 64) * 512))


def test_random_matrix_error_bound():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((256, 1024)) * 0.02).astype(np.float32)
    for deq in (R.dequantize_nvfp4_lm(*R.quantize_nvfp4_lm(w)), R.dequantize_nvfp4(*R.quantize_nvfp4(w, 32), 32)):
        err = np.abs(deq - w)
        assert err.max() < 0.02 and err.mean() < 0.003


def test_activation_fake_quant_equals_pack_then_unpack():
    """The oracle's NVFP4 view of an activation matrix (used for the FP4 prompt GEMMs) is the tensor-core packer followed
    by its dequantiser, and a projection registered in NVFP4_LINEAR is the exact product of the two dequantised operands."""
    import torch
    import oracle.qwen35_oracle as om
    from oracle.nvfp4_ref import dequantize_nvfp4_lm, quantize_nvfp4_lm
    torch.manual_seed(5)
    x = (torch.randn(128, 256) * 3).bfloat16()
    x[7] = 0
    fq = om.fake_quant_nvfp4_rows(x)
    ref = dequantize_nvfp4_lm(*quantize_nvfp4_lm(x.float().numpy()))
    assert np.array_equal(fq.numpy(), ref)
    w = (torch.randn(128, 256) * 0.1).bfloat16()
    wq = torch.from_numpy(dequantize_nvfp4_lm(*quantize_nvfp4_lm(w.float().numpy())))
    om.NVFP4_LINEAR = {id(w): wq}
    try:
        y = om.linear(x, w)
        y_plain = om.linear(x, w.clone())
    finally:
        om.NVFP4_LINEAR = None
    want = (fq.double() @ wq.double().t())
    assert y.dtype == torch.bfloat16 and float((y.double() - want).abs().max()) <= float(want.abs().max()) * 2.0 ** -8
    assert not torch.equal(y, y_plain)
