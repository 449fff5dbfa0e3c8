"""Bit-level numeric helpers (test infrastructure; see oracle/__init__.py).

bf16 rounding and the FP8 E4M3FN / E2M1 encodings restated from the format
definitions so the oracle does not depend on torch's casts.
"""
from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def bf16_bits(x) -> np.ndarray:
    """uint16 bf16 bit patterns of float32 values (RNE)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_encode(x) -> np.ndarray:
    """float32 -> float8_e4m3fn byte, round-to-nearest-even, subnormals kept,
    |x| >= 480 and NaN -> 0x7f (sign kept); equals torch's CPU cast.

    On the float32 bit pattern: a normal result rounds the 23-bit mantissa to
    3 bits (ties to even) with the carry running into the exponent field, then
    rebiases the exponent (127 -> 7); |x| < 2^-6 gives rint(|x| * 512)."""
    a32 = np.ascontiguousarray(x, dtype=np.float32)
    bits = a32.view(np.uint32)
    sign = ((bits >> np.uint32(24)) & np.uint32(0x80)).astype(np.uint8)
    mag = bits & np.uint32(0x7FFFFFFF)
    normal = (mag + np.uint32(0x7FFFF) + ((mag >> np.uint32(20)) & np.uint32(1))) >> np.uint32(20)
    code = normal.astype(np.int64) - (120 << 3)
    a = mag.view(np.float32)
    sub = mag < np.uint32(0x3C800000)                   # |x| < 2^-6
    with np.errstate(over="ignore", invalid="ignore"):  # lanes where sub is False are discarded
        code = np.where(sub, np.rint(a * np.float32(512.0)).astype(np.int64), code)
    code = np.where(mag >= np.uint32(0x43F00000), 0x7F, code)    # |x| >= 480 or NaN
    return code.astype(np.uint8) | sign


def e4m3_decode(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = (b >> 7) & 1
    e = (b >> 3) & 0xF
    m = b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    v = np.where((e == 15) & (m == 7), np.nan, v)
    return np.where(s == 1, -v, v).astype(np.float32)


def fp16_round(x) -> np.ndarray:
    """Round float32 values to float16 (RNE), returned as float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    return fp16_round(x) if dtype == "fp16" else bf16_round(x)
