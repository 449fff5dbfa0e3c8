"""FlashDecoder's local GQA attention oracle (oracle/flashdecoder.py) against
the reference itself (tests/golden/flashdecoder_outputs.npz, made by
`TRITON_INTERPRET=1 tests/golden/make_golden.py <reference> --flashdecoder`):
its CPU path (recavsr_infer/models/flashdecoder/flashdecoder_wan22.py:38-119,
fp32 SDPA under the visibility mask) on three geometries -- grouped-query
heads 4:1 and 8:2, temporal groups of 1, 2 and 4 frames, windows smaller and
larger than the grid -- and its Triton forward (_local_attention_triton.py:21-131)
in fp16 under the Triton interpreter."""
import os

import numpy as np
import pytest

from oracle import flashdecoder as ofd
from tests.golden import recipes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def fgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "flashdecoder_outputs.npz"))


def _run(tag, dtype=np.float32):
    b, hq, hk, d, h, w, win, grp, tw, qf, nf = recipes.LOCAL_GQA_CASES[tag]
    q, k, v = (x.astype(dtype).astype(np.float32) for x in recipes.local_gqa_inputs(tag))
    return ofd.local_gqa_attention(q, k, v, h, w, win, grp, tw)


@pytest.mark.parametrize("tag", sorted(recipes.LOCAL_GQA_CASES))
def test_local_gqa_attention_matches_reference_cpu_path(fgold, tag):
    got, ref = _run(tag), fgold[f"fd_{tag}_out"]
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-5 * np.abs(ref).max())


def test_local_gqa_attention_matches_reference_triton_kernel(fgold):
    ref = fgold["fd_a_triton_fp16"].astype(np.float32)
    got = _run("a", np.float16)
    # fp16 output rounding: measured 3.3e-4 at max |out| 1.01
    assert np.abs(got - ref).max() <= 1e-3 * max(np.abs(ref).max(), 1.0)


def test_visibility_is_local_and_grouped():
    # 3 x 4 grid, groups of 2 frames, 4 key frames, the last 2 as queries
    m = ofd.visibility(3, 4, 2, 4, (2, 2), 2, 1)
    n = 12
    # a query sees only its own group's two frames (temporal_window 1)...
    assert not m[:, :2 * n].any() and m[:, 2 * n:].any()
    # ...and, in each, the 2 x 2 box [y-1, y] x [x-1, x] truncated at the border
    q = 1 * 4 + 2                                   # (y, x) = (1, 2) of the first query frame
    seen = sorted(int(k) % n for k in np.flatnonzero(m[q]) if k < 3 * n)
    assert seen == [1, 2, 5, 6]
    assert sorted(int(k) % n for k in np.flatnonzero(m[0]) if k < 3 * n) == [0]


@pytest.mark.parametrize("tag", sorted(recipes.DECODER_CASES))
def test_decode_step_matches_reference_session(tag):
    """oracle.flashdecoder.DecoderOracle against the reference's own
    FlashDecoderSession.step (fp32, CPU; tests/golden/decoder_step_outputs.npz,
    `make_golden.py <reference> --decoder-step`): every step's RGB chunk and the
    hidden states leaving the backbone and the temporal refinement, over enough
    steps to trim both caches."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "decoder_step_outputs.npz"))
    c = recipes.DECODER_CASES[tag]
    lat, mean, std, lr = recipes.decoder_inputs(tag)
    o = ofd.DecoderOracle(recipes.decoder_params(tag), dim=c["dim"], num_heads=c["num_heads"],
                          num_kv_groups=c["num_kv_groups"], depth=c["depth"],
                          refinement_depth=c["refinement_depth"], window=c["window"], mean=mean, std=std)
    off = 0
    for i in range(c["steps"]):
        take = 1 if i == 0 else 4
        rgb, backbone, refine = o.step(lat[0, :, i], lr[0, :, off:off + take])
        off += take
        # fp32 on both sides, different summation orders: measured <= 5e-6
        np.testing.assert_allclose(rgb, g[f"dec_{tag}_rgb{i}"][0], rtol=0, atol=2e-5)
        for name, got in (("backbone", backbone), ("refine", refine)):
            ref = g[f"dec_{tag}_{name}{i}"][0]
            assert np.abs(got - ref).max() <= 2e-6 * np.abs(ref).max(), (name, i)
