"""GPU parity of the NVFP4 packers, through the C ABI: byte for byte against the reference's own kernels (compiled from
its source with its flags, oracle/_ref), and against the numpy oracle, which restates the arithmetic in IEEE operations.
The reference builds with fast-math, whose approximate reciprocal sits one f32 last place from the IEEE quotient for
some scales; an element that falls exactly on a threshold of the E2M1 grid then takes the neighbouring code.  Against
the IEEE oracle the comparison therefore allows a handful of neighbouring codes (and fp16 scales one last place apart);
against the reference's kernels it allows nothing."""
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


def _assert_codes_close(got, ref, what, max_frac=2e-4):
    """Packed E2M1 bytes: identical except for at most max_frac of the nibbles, each of which is the neighbouring code."""
    got, ref = np.asarray(got), np.asarray(ref)
    assert got.shape == ref.shape, what
    g = np.stack([got & 0xF, got >> 4], -1).astype(np.int32)
    r = np.stack([ref & 0xF, ref >> 4], -1).astype(np.int32)
    bad = g != r
    frac = float(bad.mean())
    assert frac <= max_frac, (what, frac)
    if bad.any():
        gm, rm = g[bad] & 7, r[bad] & 7
        assert bool((np.abs(gm - rm) <= 1).all()), what               # neighbouring magnitudes
        assert bool((((g[bad] ^ r[bad]) & 8) == 0).all() | ((gm == 0) | (rm == 0)).all()), what
    return frac


def _assert_half_scales_close(got_u16, ref_u16, what, max_frac=2e-3):
    d = np.abs(got_u16.astype(np.int32) - ref_u16.astype(np.int32))
    assert int(d.max()) <= 1 and float((d > 0).mean()) <= max_frac, (what, int(d.max()), float((d > 0).mean()))


@pytest.mark.parametrize("idx", [0, 1, 2])
def test_tensor_core_layout_bit_exact(idx):
    from qwen35_b200.model import _quantize_matrix_nvfp4_lm
    w = torch.from_numpy(_mats()[idx]).bfloat16()
    ref_p, ref_s = R.quantize_nvfp4_lm(w.float().numpy())
    got = _quantize_matrix_nvfp4_lm(w.cuda())
    _assert_codes_close(got["packed"].cpu().numpy(), ref_p, ("tc packed", idx))
    assert np.array_equal(got["scales"].cpu().numpy(), ref_s)          # amax * (1/6) and the E4M3 conversion are exact either way


@pytest.mark.parametrize("idx,group", [(0, 32), (1, 32), (2, 32), (0, 16), (1, 64)])
def test_decode_body_layout_bit_exact(idx, group):
    from qwen35_b200.model import _quantize_matrix_nvfp4
    w = torch.from_numpy(_mats()[idx]).bfloat16()
    ref_p, ref_s = R.quantize_nvfp4(w.float().numpy(), group)
    got = _quantize_matrix_nvfp4(w.cuda(), group)
    _assert_codes_close(got["packed"].cpu().numpy(), ref_p, ("decode packed", idx, group), max_frac=2e-3)
    _assert_half_scales_close(got["scales"].cpu().numpy().view(np.uint16), ref_s.view(np.uint16), ("decode scales", idx, group))


def test_padded_rows_and_errors():
    from qwen35_b200.model import _quantize_matrix_nvfp4, _quantize_matrix_nvfp4_lm, _quantize_matrix_nvfp4_tc
    w = (torch.randn(200, 128) * 0.1).bfloat16().cuda()
    q = _quantize_matrix_nvfp4_tc(w)
    assert q["padded_rows"] == 256 and q["packed"].shape == (256, 64)
    ref_p, ref_s = R.quantize_nvfp4_lm(torch.cat([w.cpu().float(), torch.zeros(56, 128)]).numpy())
    _assert_codes_close(q["packed"].cpu().numpy(), ref_p, "padded tc packed")
    assert np.array_equal(q["scales"].cpu().numpy(), ref_s)
    with pytest.raises(ValueError):
        _quantize_matrix_nvfp4_lm(w)                      # 200 rows
    with pytest.raises(ValueError):
        _quantize_matrix_nvfp4(w, 48)
    with pytest.raises(TypeError):
        _quantize_matrix_nvfp4(w.float(), 32)


# ---- against the reference's own packer kernels -------------------------------------------------------------
# oracle/_ref/libref_nvfp4.so is the reference's NVFP4 translation unit compiled unchanged with its own flags (including
# --use_fast_math) by oracle/Makefile; its two launchers run the reference's quantize_nvfp4_kernel and
# quantize_nvfp4_lm_kernel (kernel_gb10_nvfp4.cu:1757-1810, 1366-1430).  Test side only: the product never loads it.
def _reference_lib():
    import ctypes as C
    import os
    from conftest import ROOT
    path = os.path.join(ROOT, "oracle", "_ref", "libref_nvfp4.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/libref_nvfp4.so not built (make -C oracle, where the reference checkout is present)")
    lib = C.CDLL(path)
    vp, i = C.c_void_p, C.c_int
    lib.launch_quantize_nvfp4_out.restype = None
    lib.launch_quantize_nvfp4_out.argtypes = [vp, i, i, i, vp, vp, vp]
    lib.launch_quantize_nvfp4_lm_out.restype = None
    lib.launch_quantize_nvfp4_lm_out.argtypes = [vp, i, i, vp, vp, vp]
    return lib


def _model_matrices(full_weights_cpu):
    """One matrix of every shape the 0.8B model quantises (DeltaNet qkv / z / out, attention q / k / o, gate, down) and a
    slab of the LM head, plus the known-answer rows (ties, all-zero blocks, saturation, sub-floor values)."""
    dn = next(l for l in full_weights_cpu["layer_data"] if l["type"] == 0)["ptrs"]
    fa = next(l for l in full_weights_cpu["layer_data"] if l["type"] == 1)["ptrs"]
    mats = [dn[1], dn[2], dn[9], dn[11], dn[13], fa[1], fa[2], fa[6], full_weights_cpu["lm_head_weight"][:4096]]
    mats += [torch.from_numpy(m).bfloat16() for m in _mats()]
    return mats


def test_packers_equal_the_reference_kernels_byte_for_byte(full_weights_cpu):
    import ctypes as C
    from qwen35_b200.model import _quantize_matrix_nvfp4, _quantize_matrix_nvfp4_lm
    ref = _reference_lib()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    n_dec = n_tc = 0
    for w in _model_matrices(full_weights_cpu):
        w = w.cuda().contiguous()
        rows, cols = w.shape
        for group in (32, 16):
            mine = _quantize_matrix_nvfp4(w, group)
            p = torch.zeros_like(mine["packed"]); s = torch.zeros_like(mine["scales"])
            ref.launch_quantize_nvfp4_out(w.data_ptr(), rows, cols, group, p.data_ptr(), s.data_ptr(), st)
            torch.cuda.synchronize()
            assert torch.equal(p, mine["packed"]), (tuple(w.shape), group, "packed", int((p != mine["packed"]).sum()), p.numel())
            assert torch.equal(s.view(torch.int16), mine["scales"].view(torch.int16)), (tuple(w.shape), group, "scales", int((s.view(torch.int16) != mine["scales"].view(torch.int16)).sum()))
            n_dec += 1
        if rows % 128 == 0 and cols % 64 == 0:
            mine = _quantize_matrix_nvfp4_lm(w)
            p = torch.zeros_like(mine["packed"]); s = torch.zeros_like(mine["scales"])
            ref.launch_quantize_nvfp4_lm_out(w.data_ptr(), rows, cols, p.data_ptr(), s.data_ptr(), st)
            torch.cuda.synchronize()
            assert torch.equal(p, mine["packed"]), (tuple(w.shape), "tc packed")
            assert torch.equal(s, mine["scales"]), (tuple(w.shape), "tc scales")
            n_tc += 1
    print(f"{n_dec} decode-layout and {n_tc} tensor-core-layout packings identical to the reference kernels'")
    assert n_dec >= 20 and n_tc >= 8
