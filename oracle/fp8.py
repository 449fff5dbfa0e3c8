"""FP8 per-tensor oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/runtime/fp8.py:31-47.
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round, e4m3_decode, e4m3_encode

FP8_MAX = 448.0


def scale_of(amax) -> np.float32:
    """fp8.py:41: max(amax, 1e-12) / 448 in fp32."""
    return np.float32(max(np.float32(amax), np.float32(1e-12)) / np.float32(FP8_MAX))


def encode(matrix: np.ndarray, scale) -> np.ndarray:
    """fp8.py:42: e4m3(clamp(x / scale, -448, 448))."""
    x = np.asarray(matrix, dtype=np.float32)
    with np.errstate(invalid="ignore"):
        z = np.clip((x / np.float32(scale)).astype(np.float32), -FP8_MAX, FP8_MAX)
    return e4m3_encode(z)


def quantize(matrix: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """fp8.py:41-42: scale = max(amax, 1e-12)/448; q = e4m3(clamp(x/scale))."""
    x = np.asarray(matrix, dtype=np.float32)
    scale = scale_of(np.abs(x).max() if x.size else 0.0)
    return encode(x, scale), scale


def fp8_mm(a_q, scale_a, w_q, scale_w, bias) -> np.ndarray:
    """fp8.py:44-47: bf16((A*sa) @ (W*sw)^T + bias), fp32 accumulation."""
    a = e4m3_decode(a_q).astype(np.float64) * float(scale_a)
    w = e4m3_decode(w_q).astype(np.float64) * float(scale_w)
    acc = a @ w.T
    if bias is not None:
        acc = acc + np.asarray(bias, dtype=np.float64)[None, :]
    return bf16_round(acc.astype(np.float32))
