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


def fullsize_hashes() -> dict:
    with open(os.path.join(ROOT, "tests", "golden", "fullsize_hashes.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("m,k", SHAPES)
def test_oracle_quantizers_bit_exact_at_full_size(m, k):
    ref = fullsize_hashes()
    x = recipes.cfg3_activation_large(m, k)
    codes, scales = onv.quantize(x)
    assert sha(codes) == ref[f"nvfp4_{m}x{k}"]["codes"]
    assert sha(scales) == ref[f"nvfp4_{m}x{k}"]["scales"]
    q, scale = ofp8.quantize(x)
    assert np.float32(scale) == np.float32(ref[f"fp8_{m}x{k}"]["scale"])
    assert sha(q) == ref[f"fp8_{m}x{k}"]["codes"]
