"""Frame preparation and strip blending on the device, bit for bit against the
oracle (itself pinned to cv2 and to the reference's fixtures on the CPU):
rc_enlarge_block at the fixture geometries, at the 1280x704 bench block and at
1920x1088 (reflect pad of 8 rows), fp32 and bf16 outputs, prepare_block from
pinned host frames with a short final block; rc_strip_blend on the reference's
strip fixtures and on a 4-strip 1080p frame."""
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import pipeline as op
from oracle.numerics import bf16_round
from tests.golden import make_golden, recipes
from tests.util import assert_no_device_error

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pipeline_outputs.npz")
GOLDEN_CUDA = os.path.join(os.path.dirname(__file__), "golden", "pipeline_cuda_outputs.npz")


@pytest.fixture(scope="module")
def pg():
    return np.load(GOLDEN)


def test_enlarge_block_matches_reference_fixtures(pg):
    """normalize="cpu" against the reference's block_tensor on the CPU, the
    default ("cuda") against the oracle's reciprocal form and, where it was
    generated, against the reference's block_tensor run on CUDA."""
    from recavsr_b200.runtime.pipeline import enlarge_block
    pc = np.load(GOLDEN_CUDA) if os.path.exists(GOLDEN_CUDA) else None
    for i, (n, h, w, block, size) in enumerate(make_golden.PIPELINE_ENLARGE):
        host_frames = recipes.lq_frames_u8(n, h, w, seed=60 + i)
        frames = torch.from_numpy(host_frames).cuda()
        size = size or op.scaled_size(h, w, 4.0)
        x = enlarge_block(frames, size, block=block, normalize="cpu").cpu().numpy()
        assert tuple(x.shape) == tuple(pg[f"enlarge{i}_shape"])
        assert hashlib.sha256(x.tobytes()).digest() == pg[f"enlarge{i}_sha256"].tobytes(), i
        xc = enlarge_block(frames, size, block=block).cpu().numpy()
        np.testing.assert_array_equal(xc, op.block_tensor(op.enlarge_block(host_frames, size, block), True))
        if pc is not None:
            assert hashlib.sha256(xc.tobytes()).digest() == pc[f"enlarge{i}_sha256"].tobytes(), i
        xb = enlarge_block(frames, size, block=block, dtype=torch.bfloat16).float().cpu().numpy()
        np.testing.assert_array_equal(xb, bf16_round(xc))
    assert_no_device_error()


@pytest.mark.parametrize("h,w,n,block", [(176, 320, 8, 8), (270, 480, 3, 8)])
def test_enlarge_block_bench_geometries(h, w, n, block):
    """x4 to 704x1280 (no pad) and to 1080x1920 (8 rows of reflect pad), a
    short block padded with its last frame."""
    from recavsr_b200.runtime.pipeline import enlarge_block
    frames = recipes.lq_frames_u8(n, h, w, seed=h + w)
    size = op.scaled_size(h, w, 4.0)
    got = enlarge_block(torch.from_numpy(frames).cuda(), size, block=block, dtype=torch.bfloat16)
    want = op.block_tensor(op.enlarge_block(frames, size, block), reciprocal=True)
    assert_no_device_error()
    np.testing.assert_array_equal(got.float().cpu().numpy(), bf16_round(want))


def test_prepare_block_from_pinned_host_frames():
    """video.py:138-150 semantics: frames [start, start + valid) of the video,
    padded to the block length with the last one."""
    from recavsr_b200.runtime.pipeline import block_schedule, prepare_block
    video = torch.from_numpy(recipes.lq_frames_u8(31, 44, 80, seed=9)).pin_memory()
    got = [(s, v, b, prepare_block(video, s, v, b, device="cuda")) for s, v, b in block_schedule(31)]
    assert [(s, v, b) for s, v, b, _ in got] == [(0, 21, 21), (21, 8, 8), (29, 2, 8)]
    for s, v, b, x in got:
        want = op.block_tensor(op.enlarge_block(video.numpy()[s:s + v], (176, 320), b), reciprocal=True)
        np.testing.assert_array_equal(x.cpu().numpy(), want)
    with pytest.raises(ValueError):
        prepare_block(video, 30, 2, 8, device="cuda")
    assert_no_device_error()


def test_strip_blend_matches_reference_fixtures(pg):
    from recavsr_b200.runtime.pipeline import StripBlender
    for i, (lq_w, n_strips, overlap, scale, height, n_frames) in enumerate(make_golden.PIPELINE_BLEND):
        cols = op.strip_columns(lq_w, n_strips, overlap, scale)
        width = op.scaled_size(1, lq_w, scale)[1]
        blender = StripBlender(cols, scale, height, width, device="cuda")
        for t in range(n_frames):
            frames = [torch.from_numpy(pg[f"blend{i}_strip{s}"][t]).cuda() for s in range(n_strips)]
            np.testing.assert_array_equal(blender.blend(frames).cpu().numpy(), pg[f"blend{i}_out"][t])
    assert_no_device_error()


def test_strip_blend_1080p_four_strips():
    from recavsr_b200.runtime.pipeline import StripBlender
    cols = op.strip_columns(480, 4, 48, 4.0)
    width = op.scaled_size(1, 480, 4.0)[1]
    weights = op.column_weights(cols, 4.0, width)
    total = op.feather_total(weights, width)
    rs = np.random.RandomState(4)
    frames = [rs.randint(0, 256, (1080, len(w), 3)).astype(np.uint8) for _, w in weights]
    blender = StripBlender(cols, 4.0, 1080, width, device="cuda")
    got = blender.blend([torch.from_numpy(f).cuda() for f in frames]).cpu().numpy()
    np.testing.assert_array_equal(got, op.blend_frame(frames, weights, total, 1080, width))
    assert_no_device_error()
