"""Host-pipeline oracle pinned to the reference and to cv2 (CPU).

* oracle.pipeline.resize_linear_u8 equals cv2.resize(INTER_LINEAR) on uint8
  RGB frames for random up- and down-scales (cv2 is the reference's own
  resize, recavsr_infer/video.py:158);
* enlarge_block + block_tensor equal the reference's outputs recorded in
  tests/golden/pipeline_outputs.npz (uint8 frames and the fp32 model input,
  bit for bit), and so does the strip blend;
* the product's host bookkeeping (recavsr_b200.runtime.pipeline) equals the
  oracle's (scaled sizes, block schedule, strip columns, feather weights).
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import pipeline as op
from tests.golden import make_golden, recipes

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pipeline_outputs.npz")
GOLDEN_CUDA = os.path.join(os.path.dirname(__file__), "golden", "pipeline_cuda_outputs.npz")


@pytest.fixture(scope="module")
def pg():
    return np.load(GOLDEN)


def test_resize_matches_cv2_random_geometries():
    cv2 = pytest.importorskip("cv2")
    rs = np.random.RandomState(3)
    for trial in range(120):
        h, w = rs.randint(1, 50), rs.randint(1, 50)
        H, W = rs.randint(1, 160), rs.randint(1, 160)
        img = rs.randint(0, 256, (h, w, 3)).astype(np.uint8)
        if trial % 3 == 0:
            img = np.full_like(img, 255)
        want = cv2.resize(img, (W, H), interpolation=cv2.INTER_LINEAR)
        np.testing.assert_array_equal(op.resize_linear_u8(img, H, W), want.reshape(H, W, 3),
                                      err_msg=f"{(h, w)} -> {(H, W)}")


def test_resize_matches_cv2_bench_geometries():
    cv2 = pytest.importorskip("cv2")
    for (h, w, H, W) in ((176, 320, 704, 1280), (270, 480, 1080, 1920)):
        img = recipes.lq_frames_u8(1, h, w, seed=7)[0]
        want = cv2.resize(img, (W, H), interpolation=cv2.INTER_LINEAR)
        np.testing.assert_array_equal(op.resize_linear_u8(img, H, W), want)


def test_enlarge_and_block_tensor_match_reference(pg):
    for i, (n, h, w, block, size) in enumerate(make_golden.PIPELINE_ENLARGE):
        frames = recipes.lq_frames_u8(n, h, w, seed=60 + i)
        size = size or op.scaled_size(h, w, 4.0)
        enlarged = op.enlarge_block(frames, size, block)
        np.testing.assert_array_equal(np.transpose(enlarged, (3, 0, 1, 2))[None], pg[f"enlarge{i}_u8"])
        x = op.block_tensor(enlarged)
        assert tuple(x.shape) == tuple(pg[f"enlarge{i}_shape"])
        assert hashlib.sha256(np.ascontiguousarray(x).tobytes()).digest() == pg[f"enlarge{i}_sha256"].tobytes()
        if f"enlarge{i}_f32" in pg:
            np.testing.assert_array_equal(x, pg[f"enlarge{i}_f32"])


def test_block_tensor_cuda_arithmetic_matches_reference():
    """The reference's block_tensor on CUDA (fixture made on a B200 by
    make_golden.py --pipeline-cuda): the oracle's reciprocal form."""
    if not os.path.exists(GOLDEN_CUDA):
        pytest.skip("pipeline_cuda_outputs.npz not generated")
    pc = np.load(GOLDEN_CUDA)
    for i, (n, h, w, block, size) in enumerate(make_golden.PIPELINE_ENLARGE):
        frames = recipes.lq_frames_u8(n, h, w, seed=60 + i)
        size = size or op.scaled_size(h, w, 4.0)
        x = op.block_tensor(op.enlarge_block(frames, size, block), reciprocal=True)
        assert hashlib.sha256(np.ascontiguousarray(x).tobytes()).digest() == pc[f"enlarge{i}_sha256"].tobytes(), i
        if f"enlarge{i}_f32" in pc:
            np.testing.assert_array_equal(x, pc[f"enlarge{i}_f32"])


def test_strip_blend_matches_reference(pg):
    for i, (lq_w, n_strips, overlap, scale, height, n_frames) in enumerate(make_golden.PIPELINE_BLEND):
        cols = op.strip_columns(lq_w, n_strips, overlap, scale)
        np.testing.assert_array_equal(np.array(cols), pg[f"blend{i}_columns"])
        width = op.scaled_size(1, lq_w, scale)[1]
        weights = op.column_weights(cols, scale, width)
        total = op.feather_total(weights, width)
        for t in range(n_frames):
            frames = [pg[f"blend{i}_strip{s}"][t] for s in range(n_strips)]
            np.testing.assert_array_equal(op.blend_frame(frames, weights, total, height, width),
                                          pg[f"blend{i}_out"][t])


def test_runtime_host_bookkeeping_matches_oracle():
    from recavsr_b200.runtime import pipeline as rp
    for h, w, s in ((176, 320, 4.0), (270, 480, 4.0), (13, 21, 3.7), (1, 1, 0.5)):
        assert rp.scaled_size(h, w, s) == op.scaled_size(h, w, s)
    for total in (1, 20, 21, 22, 29, 300):
        assert list(rp.block_schedule(total)) == list(op.block_schedule(total))
    for lq_w, n, ov, sc in ((480, 4, 48, 4.0), (40, 3, 6, 4.0), (33, 2, 5, 2.0), (1000, 8, 32, 2.5)):
        cols = rp.strip_columns(lq_w, n, ov, sc)
        assert cols == op.strip_columns(lq_w, n, ov, sc)
        width = op.scaled_size(1, lq_w, sc)[1]
        for (a0, a), (b0, b) in zip(rp.column_weights(cols, sc, width), op.column_weights(cols, sc, width)):
            assert a0 == b0
            np.testing.assert_array_equal(a, b)
    with pytest.raises(ValueError):
        rp.scaled_size(0, 4)
