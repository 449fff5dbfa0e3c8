"""The FP8 quantizer's division by the per-tensor scale, checked on the CPU.

The device computes z = |x| / s for every element of a call with one
correctly rounded reciprocal y = RN(1/s), q = RN(|x| y) and one Markstein
correction step (remainder r = |x| - s q by one fma, q <- RN(q + r y) by
another) instead of a full division per element. This test replays that
sequence in numpy with exact fma emulation for every non-negative finite bf16
x up to just above amax and every scale s = RN(max(amax, 1e-12) / 448) that a
bf16 amax can produce, and requires the quotient to equal numpy's correctly
rounded float32 division (bit for bit wherever the E4M3 code can depend on
it, >= 2^-11) and the E4M3 codes to match everywhere: that is the
reference's x / scale. With RECAVSR_FP8_DIV_ALL=1 it covers all 21,492
scales (4.7e8 pairs, no mismatch; about 90 s); by default every 7th scale
plus the extreme ones.
"""
import os

import numpy as np

from oracle.numerics import bf16_from_bits, e4m3_encode

F32, F64 = np.float32, np.float64


def fma32(a, b, c):
    """RN_float32(a * b + c) exactly, for float32 arrays (no overflow)."""
    p = a.astype(F64) * b.astype(F64)              # exact: 24 + 24 bits
    c64 = c.astype(F64)
    hi = p + c64
    bb = hi - p                                    # TwoSum: hi + lo == p + c exactly
    lo = (p - (hi - bb)) + (c64 - bb)
    r = hi.astype(F32)
    # hi may sit exactly on a float32 midpoint, where lo decides the rounding.
    down = np.where(r.astype(F64) > hi, np.nextafter(r, F32(-np.inf)), r)
    up = np.where(r.astype(F64) < hi, np.nextafter(r, F32(np.inf)), r)
    mid = (down.astype(F64) + up.astype(F64)) * 0.5
    tie = (down != up) & (mid == hi) & (lo != 0)
    return np.where(tie, np.where(lo > 0, up, down), r)


def device_quotient(ax, s):
    """|x| / s as the FP8 quantize kernel computes it (x finite, s finite normal)."""
    y = F32(1.0) / s
    q = ax * y
    r = fma32(-q, np.full_like(q, s), ax)
    return fma32(r, np.full_like(q, y), q)


def _scales():
    amax = bf16_from_bits(np.arange(1, 0x7F80, dtype=np.uint32).astype(np.uint16)).astype(F32)
    amax = np.maximum(amax, F32(1e-12))
    scales = np.unique((amax / F32(448.0)).astype(F32))
    if os.environ.get("RECAVSR_FP8_DIV_ALL") != "1":
        scales = np.unique(np.concatenate([scales[::7], scales[:4], scales[-4:]]))
    return scales


def test_markstein_division_matches_correct_rounding():
    allx = bf16_from_bits(np.arange(0, 0x7F80, dtype=np.uint32).astype(np.uint16)).astype(F32)
    bad = 0
    for s in _scales():
        ax = allx[allx.astype(F64) <= F64(s) * 448.0 * 1.01]     # |x| <= amax and a little above
        want = (ax / s).astype(F32)
        got = device_quotient(ax, F32(s))
        # Bit-exact quotient wherever the E4M3 code can depend on it.
        relevant = want >= F32(2.0 ** -11)
        bad += int(np.count_nonzero(got[relevant] != want[relevant]))
        bad += int(np.count_nonzero(e4m3_encode(np.minimum(got, F32(448.0)))
                                    != e4m3_encode(np.minimum(want, F32(448.0)))))
    assert bad == 0
