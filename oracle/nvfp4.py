"""NVFP4 oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/runtime/nvfp4.py:49-68 (quantize) and the math of
:22-39 (``_scaled_mm_v2`` with BlockWise1x16 scales, SWIZZLE_32_4_4, bias,
bf16 out) as "unswizzle + dequantize in fp32, then matmul + bias".
"""
from __future__ import annotations

import numpy as np

from .numerics import E2M1_VALUES, bf16_round, e4m3_decode, e4m3_encode

_THRESHOLDS = ((0.25, False), (0.75, True), (1.25, False), (1.75, True),
               (2.5, False), (3.5, True), (5.0, False))


def e2m1_codes(z: np.ndarray) -> np.ndarray:
    """nvfp4.py:55-61: count of thresholds passed, ties to even; sign 8 iff z < 0."""
    a = np.abs(z)
    code = np.zeros(z.shape, dtype=np.uint8)
    for t, inclusive in _THRESHOLDS:
        code += (a >= t) if inclusive else (a > t)
    return code | ((z < 0).astype(np.uint8) * 8)


def padded_scale_shape(m: int, k: int) -> tuple[int, int]:
    """nvfp4.py:64: rows padded to 128, 16-blocks padded to a multiple of 4."""
    return (m + 127) // 128 * 128, ((k // 16 + 3) // 4) * 4


def swizzle_scales(scales: np.ndarray, m: int, k: int) -> np.ndarray:
    """nvfp4.py:64-67: zero pad, view (pm/128, 4, 32, pk/4, 4), permute (0,3,2,1,4)."""
    pm, pk = padded_scale_shape(m, k)
    padded = np.zeros((pm, pk), dtype=np.uint8)
    padded[:m, : k // 16] = scales
    return padded.reshape(pm // 128, 4, 32, pk // 4, 4).transpose(0, 3, 2, 1, 4).reshape(-1).copy()


def unswizzle_scales(flat: np.ndarray, m: int, k: int) -> np.ndarray:
    pm, pk = padded_scale_shape(m, k)
    blocked = np.asarray(flat, dtype=np.uint8).reshape(pm // 128, pk // 4, 32, 4, 4)
    return blocked.transpose(0, 3, 2, 1, 4).reshape(pm, pk)[:m, : k // 16].copy()


def quantize(matrix: np.ndarray, global_scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    """nvfp4.py:49-68 on a float32 (bf16-valued) [M, K] matrix.

    Returns (packed codes uint8 [M, K/2], swizzled scales uint8 flat). With
    ``global_scale`` g != 1 the block scale is e4m3(max(amax/6*g, 2^-9)) and
    z = (x*g)/s (the per-tensor global-scale mode); g = 1 is the reference.
    """
    x = np.asarray(matrix, dtype=np.float32)
    m, k = x.shape
    g = np.float32(global_scale)
    blocks = x.reshape(m, k // 16, 16)
    amax = np.abs(blocks).max(-1)
    s = (amax / np.float32(6.0)).astype(np.float32) * g
    s = np.where(s < np.float32(2.0 ** -9), np.float32(2.0 ** -9), s).astype(np.float32)
    s = np.where(np.isnan(amax), np.float32(np.nan), s)
    sb = e4m3_encode(s)
    sd = e4m3_decode(sb)
    with np.errstate(invalid="ignore", divide="ignore"):
        z = ((blocks * g).astype(np.float32) / sd[..., None]).astype(np.float32)
    code = e2m1_codes(z).reshape(m, k)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, swizzle_scales(sb, m, k)


def dequantize(packed: np.ndarray, flat_scales: np.ndarray, m: int, k: int) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint8).reshape(m, k // 2)
    codes = np.empty((m, k), dtype=np.uint8)
    codes[:, 0::2] = p & 0xF
    codes[:, 1::2] = p >> 4
    vals = E2M1_VALUES[codes]
    sd = e4m3_decode(unswizzle_scales(flat_scales, m, k))
    return (vals.reshape(m, k // 16, 16) * sd[..., None]).reshape(m, k).astype(np.float32)


def nvfp4_mm(a_packed, a_scales, b_packed, b_scales, bias, m: int, n: int, k: int,
             alpha: float = 1.0, dtype=np.float64, b_dequantized=None) -> np.ndarray:
    """bf16(alpha * dequant(A) @ dequant(B)^T + bias) as float32 values.
    dtype float64 (default) for parity checks; float32 for the timed CPU baseline."""
    a = dequantize(a_packed, a_scales, m, k).astype(dtype)
    b = (dequantize(b_packed, b_scales, n, k) if b_dequantized is None else b_dequantized).astype(dtype)
    acc = (a @ b.T) * dtype(alpha)
    if bias is not None:
        acc = acc + np.asarray(bias, dtype=dtype)[None, :]
    return bf16_round(acc.astype(np.float32))
