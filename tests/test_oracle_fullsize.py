"""Bit-exactness at cfg3's full activation sizes (7040 x 14336 and 7040 x 3072),
where the outputs are too large for fixtures: SHA-256 of the oracle's NVFP4
codes / swizzled scales and FP8 codes (plus the FP8 scale) against those of the
reference's own quantizers (recavsr_infer/runtime/nvfp4.py:49-68,
runtime/fp8.py:41-42), recorded in tests/golden/fullsize_hashes.json by
`tests/golden/make_golden.py <reference> --fullsize`."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from tests.golden import recipes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPES = [(7040, 14336), (7040, 3072)]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


ROWS = 128   # one scale atom of rows: chunks keep every temporary small


def chunked(x):
    """The oracle's NVFP4 codes / swizzled scales and FP8 codes of x, hashed
    128 rows at a time (NVFP4 scales are per row and their swizzled atoms hold
    128 rows; the FP8 scale comes from one amax pass over all rows)."""
    h_codes, h_scales, h_fp8 = hashlib.sha256(), hashlib.sha256(), hashlib.sha256()
    amax = np.float32(0.0)
    for r in range(0, x.shape[0], ROWS):
        amax = max(amax, np.float32(np.abs(x[r:r + ROWS]).max()))
    scale = ofp8.scale_of(amax)
    for r in range(0, x.shape[0], ROWS):
        codes, scales = onv.quantize(x[r:r + ROWS])
        h_codes.update(np.ascontiguousarray(codes).tobytes())
        h_scales.update(np.ascontiguousarray(scales).tobytes())
        h_fp8.update(ofp8.encode(x[r:r + ROWS], scale).tobytes())
    return h_codes.hexdigest(), h_scales.hexdigest(), h_fp8.hexdigest(), scale


def fullsize_hashes() -> dict:
    with open(os.path.join(ROOT, "tests", "golden", "fullsize_hashes.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("m,k", SHAPES)
def test_oracle_quantizers_bit_exact_at_full_size(m, k):
    ref = fullsize_hashes()
    x = recipes.cfg3_activation_large(m, k)
    codes, scales, fp8_codes, scale = chunked(x)
    assert codes == ref[f"nvfp4_{m}x{k}"]["codes"]
    assert scales == ref[f"nvfp4_{m}x{k}"]["scales"]
    assert np.float32(scale) == np.float32(ref[f"fp8_{m}x{k}"]["scale"])
    assert fp8_codes == ref[f"fp8_{m}x{k}"]["codes"]
