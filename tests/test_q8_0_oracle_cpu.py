"""The oracle's Q8_0 and Q4_0 packings (K / V cache formats of the 27B target) pinned to gguf-py's published routines through the
committed fixture tests/golden/q8_0_golden.npz (made by tests/golden/make_q8_0_golden.py with gguf-py 0.19.0), and, when
gguf-py is importable, to the library itself on fresh data."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle.tree_verify_oracle import kv_cache_value, q4_0_dequant, q4_0_quant, q8_0_dequant, q8_0_quant  # noqa: E402


def test_q8_0_matches_golden_fixture_bit_for_bit():
    g = np.load(os.path.join(ROOT, "tests", "golden", "q8_0_golden.npz"))
    q = q8_0_quant(g["x"])
    assert q.dtype == np.uint8 and q.shape == g["q"].shape and np.array_equal(q, g["q"])
    assert np.array_equal(q8_0_dequant(g["q"]).view(np.int32), g["v"].view(np.int32))


def test_q8_0_properties():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 256)).astype(np.float32) * 3
    q = q8_0_quant(x)
    v = q8_0_dequant(q)
    amax = np.abs(x.reshape(-1, 32)).max(1, keepdims=True)
    # half a step of the rounding plus 127 steps x the 2^-11 relative error of storing d as f16
    assert np.all(np.abs(v.reshape(-1, 32) - x.reshape(-1, 32)) <= amax / 127 * (0.5 + 127 * 2.0 ** -11) + 1e-7)
    assert np.array_equal(q8_0_quant(v), q)                                                               # idempotent
    assert np.array_equal(q8_0_quant(np.zeros((1, 32), np.float32)), np.zeros((1, 34), np.uint8))


def test_q8_0_matches_gguf_py_on_fresh_data():
    gguf = pytest.importorskip("gguf")
    from gguf.quants import quantize
    x = np.random.default_rng(5).standard_normal((64, 512)).astype(np.float32) * 10
    assert np.array_equal(q8_0_quant(x), quantize(x, gguf.GGMLQuantizationType.Q8_0))


def test_q4_0_matches_golden_fixture_bit_for_bit():
    """tests/golden/q4_0_golden.npz (made by tests/golden/make_q4_0_golden.py with gguf-py 0.19.0)."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "q4_0_golden.npz"))
    q = q4_0_quant(g["x"])
    assert q.dtype == np.uint8 and q.shape == g["q"].shape and np.array_equal(q, g["q"])
    assert np.array_equal(q4_0_dequant(g["q"]).view(np.int32), g["v"].view(np.int32))


def test_q4_0_properties():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((7, 256)).astype(np.float32) * 3
    q = q4_0_quant(x)
    v = q4_0_dequant(q)
    amax = np.abs(x.reshape(-1, 32)).max(1, keepdims=True)
    # one step is amax / 8; truncation of x / d + 8.5 is rounding to the nearest step, except the clip of +8 steps to +7
    assert np.all(np.abs(v.reshape(-1, 32) - x.reshape(-1, 32)) <= amax / 8 * (1.0 + 16 * 2.0 ** -11) + 1e-7)
    assert q.shape == (7, 144)
    # an all-zero block: d = 0 / -8 = -0.0 (f16 bytes 00 80), every code 8
    assert np.array_equal(q4_0_quant(np.zeros((1, 32), np.float32)), np.array([[0, 0x80] + [0x88] * 16], np.uint8))
    import torch
    t = torch.from_numpy(x)
    assert torch.equal(kv_cache_value(t, "q4_0"), torch.from_numpy(v))
    assert torch.equal(kv_cache_value(t, "f16"), t.half().float())


def test_q4_0_matches_gguf_py_on_fresh_data():
    gguf = pytest.importorskip("gguf")
    from gguf.quants import quantize
    x = np.random.default_rng(6).standard_normal((64, 512)).astype(np.float32) * 10
    assert np.array_equal(q4_0_quant(x), quantize(x, gguf.GGMLQuantizationType.Q4_0))
