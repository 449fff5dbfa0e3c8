"""Colour-correction oracle (oracle/colorfix.py) against the reference's own
adain_color_fix / wavelet_color_fix (recavsr_infer/color_fix.py:58-117) run on
the CPU (tests/golden/colorfix_outputs.npz, `make_golden.py <reference>
--colorfix`)."""
import os

import numpy as np
import pytest

from oracle import colorfix as ocf
from tests.golden import recipes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def cg():
    return np.load(os.path.join(ROOT, "tests", "golden", "colorfix_outputs.npz"))


@pytest.mark.parametrize("tag", sorted(recipes.COLORFIX_CASES))
def test_adain_matches_reference(cg, tag):
    dec, ref, _ = recipes.colorfix_inputs(tag)
    np.testing.assert_allclose(ocf.adain_color_fix(dec, ref), cg[f"cf_{tag}_adain"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("tag", sorted(recipes.COLORFIX_CASES))
def test_wavelet_matches_reference(cg, tag):
    """uint8 output: equal except where fp32 summation order moves a value
    across a rounding boundary (measured: 1 of 23040 values, by 1)."""
    dec, _, lq = recipes.colorfix_inputs(tag)
    got, ref = ocf.wavelet_color_fix(dec, lq), cg[f"cf_{tag}_wavelet"]
    assert got.shape == ref.shape and got.dtype == np.uint8
    d = np.abs(got.astype(np.int16) - ref.astype(np.int16))
    assert d.max() <= 1 and (d > 0).mean() <= 1e-3


def test_bicubic_matches_torch_cpu():
    import torch
    import torch.nn.functional as F
    x = np.random.RandomState(3).uniform(0, 1, (2, 3, 7, 11)).astype(np.float32)
    ref = F.interpolate(torch.from_numpy(x), size=(28, 44), mode="bicubic", align_corners=False).numpy()
    np.testing.assert_allclose(ocf.bicubic(x, 28, 44), ref, rtol=0, atol=2e-6)
