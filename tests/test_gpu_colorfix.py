"""Colour correction on the device (recavsr_b200.runtime.colorfix) against the
reference's fixtures and the oracle: AdaIN within 2e-6 (fp32, the plane
statistics in fp64 on both sides), the wavelet correction's uint8 frames within
1 on at most 0.1% of the values (fp32 summation order of the bicubic taps and
the blur), including a 704x1280 frame pair; validation messages."""
import os

import numpy as np
import pytest
import torch

from oracle import colorfix as ocf
from tests.golden import recipes
from tests.util import assert_no_device_error

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "colorfix_outputs.npz")


def _close_u8(got, ref):
    d = np.abs(got.astype(np.int16) - ref.astype(np.int16))
    assert got.shape == ref.shape and d.max() <= 1 and (d > 0).mean() <= 1e-3, (int(d.max()), float((d > 0).mean()))


@pytest.mark.parametrize("tag", sorted(recipes.COLORFIX_CASES))
def test_matches_reference_fixtures(tag):
    from recavsr_b200.runtime.colorfix import adain_color_fix, wavelet_color_fix
    cg = np.load(GOLDEN)
    dec, ref, lq = recipes.colorfix_inputs(tag)
    got = adain_color_fix(torch.from_numpy(dec).cuda(), torch.from_numpy(ref).cuda())
    assert got.dtype == torch.float32 and tuple(got.shape) == dec.shape
    np.testing.assert_allclose(got.cpu().numpy(), cg[f"cf_{tag}_adain"], rtol=0, atol=2e-6)
    _close_u8(wavelet_color_fix(torch.from_numpy(dec).cuda(), lq), cg[f"cf_{tag}_wavelet"])
    assert_no_device_error()


def test_full_frame_and_bf16_input():
    """Two 704x1280 frames decoded in bf16 (as DecoderSession emits them), LQ
    176x320, against the oracle on the same bf16 values."""
    from recavsr_b200.runtime.colorfix import adain_color_fix, wavelet_color_fix
    rs = np.random.RandomState(5)
    coarse = rs.uniform(-1, 1, (1, 3, 2, 45, 81)).astype(np.float32)
    dec = np.repeat(np.repeat(coarse, 16, axis=3), 16, axis=4)[:, :, :, :704, :1280]
    dec = np.clip(dec + rs.uniform(-0.1, 0.1, dec.shape), -1, 1).astype(np.float32)
    dec_bf = torch.from_numpy(dec).bfloat16()
    dec32 = dec_bf.float().numpy()
    lq = rs.randint(0, 256, (2, 176, 320, 3)).astype(np.uint8)
    _close_u8(wavelet_color_fix(dec_bf.cuda(), lq), ocf.wavelet_color_fix(dec32, lq))
    ref = np.clip(rs.uniform(-1, 1, dec.shape) * 0.3, -1, 1).astype(np.float32)
    got = adain_color_fix(dec_bf.cuda(), torch.from_numpy(ref).cuda()).cpu().numpy()
    np.testing.assert_allclose(got, ocf.adain_color_fix(dec32, ref), rtol=0, atol=2e-6)
    assert_no_device_error()


def test_validation_messages():
    from recavsr_b200.runtime.colorfix import adain_color_fix, wavelet_color_fix
    x = torch.zeros(1, 3, 2, 8, 8, device="cuda")
    with pytest.raises(ValueError, match="matching"):
        adain_color_fix(x, x[:, :, :1])
    with pytest.raises(ValueError, match="decoded"):
        wavelet_color_fix(x[0], np.zeros((2, 2, 2, 3), np.uint8))
    with pytest.raises(ValueError, match="uint8 LQ"):
        wavelet_color_fix(x, np.zeros((3, 2, 2, 3), np.uint8))
