"""CPU restatement (numpy) of the reference's two NVFP4 weight packers.  TEST INFRASTRUCTURE ONLY.

* `quantize_nvfp4`     decode-body layout, models/qwen35_0p8b/kernel_gb10_nvfp4.cu:1742-1810
                       (quantize_fp4_code + quantize_nvfp4_kernel): groups of `group_size` along K,
                       fp16 scale = amax/6 (1.0 for an all-zero group), threshold quantiser, low nibble =
                       even element.
* `quantize_nvfp4_lm`  tensor-core layout, kernel_gb10_nvfp4.cu:1366-1430 (quantize_nvfp4_lm_kernel):
                       16-element blocks, UE4M3 scale = sat_rn(max(amax/6, 2^-28)), elements divided by the
                       *decoded* scale and rounded to E2M1 with round-to-nearest-even, scales stored in
                       128-row x 4-column swizzled tiles of 512 bytes.

Both follow IEEE f32 arithmetic.  (The reference compiles with --use_fast_math, so its own binary may differ
in the last place of an intermediate quotient; that binary cannot run here.)  The number formats are pinned
against NVIDIA's host conversion functions (oracle/nvfp4_hdr_check.cpp) in tests/test_nvfp4_oracle.py.
"""
from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 >= 0 -> E4M3 byte, round-to-nearest-even, saturating at 448 (0x7e)."""
    x = np.asarray(x, dtype=np.float32)
    out = np.zeros(x.shape, dtype=np.uint8)
    big = x >= np.float32(2.0 ** -6)
    # normal numbers
    m, e = np.frexp(x.astype(np.float64))          # x = m * 2^e, m in [0.5, 1)
    e = e - 1
    frac = m * 2.0 - 1.0                            # in [0, 1)
    q = np.rint(frac * 8.0)
    carry = q == 8
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 0, q)
    code = ((e + 7).astype(np.int64) << 3) | q.astype(np.int64)
    code = np.where(code > 0x7E, 0x7E, code)
    # subnormals: multiples of 2^-9
    qs = np.rint(x.astype(np.float64) * 2.0 ** 9).astype(np.int64)       # 8 becomes the first normal, code 0x08
    out = np.where(big, code, qs).astype(np.uint8)
    return out


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    code = np.asarray(code, dtype=np.int64)
    e = (code >> 3) & 0xF
    m = code & 7
    normal = (1.0 + m / 8.0) * np.exp2(e - 7.0)
    sub = m / 8.0 * 2.0 ** -6
    return np.where(e == 0, sub, normal).astype(np.float32)


def e2m1_rne(x: np.ndarray) -> np.ndarray:
    """float32 -> 4-bit E2M1 code, round-to-nearest-even, saturating at 6; sign in bit 3."""
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x)
    mag = np.select(
        [ax <= 0.25, ax < 0.75, ax <= 1.25, ax < 1.75, ax <= 2.5, ax < 3.5, ax <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return np.where(np.signbit(x), mag | 8, mag).astype(np.uint8)


def e2m1_threshold(x: np.ndarray) -> np.ndarray:
    """The decode-body quantiser: fixed thresholds, ties go up (kernel_gb10_nvfp4.cu:1742-1755)."""
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x)
    mag = np.select(
        [ax < 0.25, ax < 0.75, ax < 1.25, ax < 1.75, ax < 2.5, ax < 3.5, ax < 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return np.where(x < 0, mag | 8, mag).astype(np.uint8)


def _pack_nibbles(codes: np.ndarray) -> np.ndarray:
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def quantize_nvfp4(w: np.ndarray, group_size: int = 32):
    """w float32 [rows, cols] (bf16-valued).  Returns packed uint8 [rows, cols/2], scales float16 [rows, cols/group]."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    g = w.reshape(rows, cols // group_size, group_size)
    amax = np.abs(g).max(axis=-1)
    scale = np.where(amax > 0, amax / np.float32(6.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    codes = e2m1_threshold((g * inv[..., None]).astype(np.float32))
    codes = np.where((amax == 0)[..., None], 0, codes).astype(np.uint8)
    return _pack_nibbles(codes.reshape(rows, cols)), scale.astype(np.float16)


def dequantize_nvfp4(packed: np.ndarray, scales: np.ndarray, group_size: int = 32) -> np.ndarray:
    rows = packed.shape[0]
    codes = np.empty((rows, packed.shape[1] * 2), dtype=np.uint8)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    vals = E2M1_VALUES[codes & 7] * np.where(codes & 8, -1.0, 1.0).astype(np.float32)
    s = np.repeat(scales.astype(np.float32), group_size, axis=1)
    return (vals * s).astype(np.float32)


def lm_scale_index(row: int | np.ndarray, scale_col: int | np.ndarray, cols: int):
    """Byte offset of the scale of (row, 16-element block `scale_col`) in the swizzled layout."""
    tile = (row // 128) * (cols // 64) + (scale_col // 4)
    return tile * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4 + (scale_col % 4)


def quantize_nvfp4_lm(w: np.ndarray):
    """w float32 [rows, cols], rows % 128 == 0, cols % 64 == 0.  Returns packed uint8 [rows, cols/2] and
    the swizzled E4M3 scale bytes uint8 [rows/128 * cols/64 * 512]."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert rows % 128 == 0 and cols % 64 == 0
    g = w.reshape(rows, cols // 16, 16)
    amax = np.abs(g).max(axis=-1)
    scale_f = np.maximum(amax * np.float32(1.0 / 6.0), np.float32(2.0 ** -28)).astype(np.float32)
    code = e4m3_encode(scale_f)
    dec = e4m3_decode(code)
    with np.errstate(divide="ignore"):
        inv = np.where(dec > 0, np.float32(1.0) / dec, np.float32(0.0)).astype(np.float32)
    codes = e2m1_rne((g * inv[..., None]).astype(np.float32))
    packed = _pack_nibbles(codes.reshape(rows, cols))
    scales = np.zeros((rows // 128) * (cols // 64) * 512, dtype=np.uint8)
    r, c = np.meshgrid(np.arange(rows), np.arange(cols // 16), indexing="ij")
    scales[lm_scale_index(r, c, cols)] = code
    return packed, scales


def dequantize_nvfp4_lm(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    rows, half = packed.shape
    cols = half * 2
    codes = np.empty((rows, cols), dtype=np.uint8)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    vals = E2M1_VALUES[codes & 7] * np.where(codes & 8, -1.0, 1.0).astype(np.float32)
    r, c = np.meshgrid(np.arange(rows), np.arange(cols // 16), indexing="ij")
    s = e4m3_decode(scales[lm_scale_index(r, c, cols)])
    return (vals * np.repeat(s, 16, axis=1)).astype(np.float32)
