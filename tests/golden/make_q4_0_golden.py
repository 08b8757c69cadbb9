"""Writes tests/golden/q4_0_golden.npz: f32 rows (random, an all-zero block, a block with one huge element, a block whose two
largest magnitudes are equal with opposite signs, values on the truncation boundaries) and their Q4_0 bytes and dequantised
values from gguf-py (gguf.quants.quantize / dequantize), the published Q4_0 packing: 32 elements -> f16 d = (element of
largest magnitude) / -8, 4-bit q = min(15, trunc(x / d + 8.5)), low nibbles elements 0..15, high nibbles 16..31."""
import os

import gguf
import numpy as np
from gguf.quants import dequantize, quantize

rng = np.random.default_rng(404)
x = rng.standard_normal((48, 256)).astype(np.float32)
x[0, :32] = 0.0
x[1, 5] = 1000.0
x[2, :32] = (np.arange(32, dtype=np.float32) - 16.0) * 0.5      # max magnitude -8: d = 1, values on the .5 boundaries
x[3, 7] = 4.0; x[3, 9] = -4.0; x[3, :32] = np.clip(x[3, :32], -4.0, 4.0)      # equal magnitudes, the first one decides the sign
x[4] *= 1e-6
x[5] *= 300.0
q = quantize(x, gguf.GGMLQuantizationType.Q4_0)
v = dequantize(q, gguf.GGMLQuantizationType.Q4_0).astype(np.float32)
np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "q4_0_golden.npz"), x=x, q=q, v=v)
print("wrote", x.shape, "->", q.shape)
