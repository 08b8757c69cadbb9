"""The oracle's Q8_0 packing (K / V cache format of the 27B target) pinned to gguf-py's published routines through the
committed fixture tests/golden/q8_0_golden.npz (made by tests/golden/make_q8_0_golden.py with gguf-py 0.19.0), and, when
gguf-py is importable, to the library itself on fresh data."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle.tree_verify_oracle import q8_0_dequant, q8_0_quant  # noqa: E402


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
