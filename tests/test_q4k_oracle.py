"""CPU: the oracle's Q4_K unpacking pinned to gguf-py's published dequantisation, plus the tree helpers."""
import numpy as np
import pytest
import torch

from oracle.tree_verify_oracle import TreeOracle, q4k_dequant, q4k_gemm_operand


def _blocks(n, seed):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    d = (rng.random(n) * 1e-3).astype(np.float16); dm = (rng.random(n) * 5e-3).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2); b[:, 2:4] = dm.view(np.uint8).reshape(n, 2)
    return b


def test_q4k_dequant_matches_gguf_py():
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    b = _blocks(257, 3)
    # extremes: all-ones scale bytes (every 6-bit field 63), zero scales, max nibbles, negative / subnormal / zero d
    b[0, 4:16] = 0xFF; b[1, 4:16] = 0; b[2, 16:] = 0xFF; b[3, 16:] = 0
    b[4, 0:2] = np.array([-0.5], np.float16).view(np.uint8); b[5, 0:2] = np.array([6e-8], np.float16).view(np.uint8); b[6, 0:4] = 0
    ref = dequantize(b.reshape(-1), gguf.GGMLQuantizationType.Q4_K).reshape(-1, 256)
    got = q4k_dequant(b)
    assert got.dtype == np.float32 and np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_q4k_golden_fixture():
    """A committed vector (made by tests/golden/make_q4k_golden.py from gguf-py) keeps the pin without gguf installed."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "q4k_golden.npz"))
    assert np.array_equal(q4k_dequant(z["blocks"]).view(np.uint32), z["values"].view(np.uint32))


def test_random_tree_is_preorder():
    from qwen35_b200.tree_verify import random_tree
    for seed in range(20):
        p = random_tree(33, 8, seed)
        assert p[0] == -1 and all(0 <= p[t] < t for t in range(1, 33))
        depth = [0] * 33
        for t in range(1, 33):
            depth[t] = depth[p[t]] + 1
            # pre-order: the parent of t is on the root-to-(t-1) path
            a, anc = t - 1, set()
            while a >= 0:
                anc.add(a); a = p[a]
            assert p[t] in anc
        assert max(depth) <= 8


def test_accept_walk():
    tokens = [5, 7, 9, 7, 3]
    parents = [-1, 0, 1, 0, 3]
    # root predicts 7: two children carry 7 (nodes 1 and 3), the first in DFS order wins; node 1 predicts 9 -> node 2
    path, nxt = TreeOracle.accept(tokens, parents, [7, 9, 4, 3, 1])
    assert path == [0, 1, 2] and nxt == 4
    path, nxt = TreeOracle.accept(tokens, parents, [8, 9, 4, 3, 1])
    assert path == [0] and nxt == 8


def test_q4k_gemm_operand_is_close_to_the_published_value():
    """The bf16 operand of the GEMM differs from the published f32 dequantisation by bf16 roundings only."""
    b = _blocks(64, 9)
    ref, got = q4k_dequant(b), q4k_gemm_operand(b)
    scale = np.abs(ref).max(axis=1, keepdims=True) + 1e-12
    assert float((np.abs(got - ref) / scale).max()) < 2.0 ** -6
    assert np.array_equal(got, torch.from_numpy(got).bfloat16().float().numpy())      # every value is a bf16 number
