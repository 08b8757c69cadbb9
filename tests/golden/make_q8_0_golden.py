"""Writes tests/golden/q8_0_golden.npz: f32 rows (random, an all-zero block, a block with one huge element, exact halves
that test the rounding mode) and their Q8_0 bytes and dequantised values from gguf-py (gguf.quants.quantize /
dequantize), the published Q8_0 packing: 32 elements -> f16 d = amax / 127, int8 q = round(x / d)."""
import os

import gguf
import numpy as np
from gguf.quants import dequantize, quantize

rng = np.random.default_rng(808)
x = rng.standard_normal((48, 256)).astype(np.float32)
x[0, :32] = 0.0
x[1, 5] = 1000.0
x[2, :32] = np.arange(32, dtype=np.float32) * 0.5            # amax 15.5: halves in q units
x[3] *= 1e-6
x[4] *= 300.0
q = quantize(x, gguf.GGMLQuantizationType.Q8_0)
v = dequantize(q, gguf.GGMLQuantizationType.Q8_0).astype(np.float32)
np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "q8_0_golden.npz"), x=x, q=q, v=v)
print("wrote", x.shape, "->", q.shape)
