"""Writes tests/golden/q4k_golden.npz: random Q4_K super-blocks (with the extreme scale / nibble / d cases) and their
dequantised values from gguf-py (gguf.quants.dequantize), the published Q4_K unpacking."""
import os

import gguf
import numpy as np
from gguf.quants import dequantize

rng = np.random.default_rng(2024)
n = 64
b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
d = (rng.random(n) * 1e-3).astype(np.float16); dm = (rng.random(n) * 5e-3).astype(np.float16)
b[:, 0:2] = d.view(np.uint8).reshape(n, 2); b[:, 2:4] = dm.view(np.uint8).reshape(n, 2)
b[0, 4:16] = 0xFF; b[1, 4:16] = 0; b[2, 16:] = 0xFF; b[3, 16:] = 0
b[4, 0:2] = np.array([-0.5], np.float16).view(np.uint8); b[5, 0:2] = np.array([6e-8], np.float16).view(np.uint8); b[6, 0:4] = 0
vals = dequantize(b.reshape(-1), gguf.GGMLQuantizationType.Q4_K).reshape(-1, 256).astype(np.float32)
np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "q4k_golden.npz"), blocks=b, values=vals, gguf_version=gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")
print("wrote", n, "blocks")
