"""The session-glue oracle (oracle/session.py) against the reference's own
TransformerSession.step (tests/golden/session_outputs.npz, made by
`tests/golden/make_golden.py <reference> --session`): the LQ projector's
streaming output per block, the hidden state entering the first DiT block
(patch embedding + LQ projection + sr_proj of the recycled latents) and the
step result (output head, unpatchify, noise - prediction), each from the
reference's own inputs to that stage."""
import os

import numpy as np
import pytest

from oracle import session as osess
from oracle.numerics import bf16_from_bits, bf16_round
from tests.golden import recipes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def sgold():
    return np.load(os.path.join(ROOT, "tests", "golden", "session_outputs.npz"))


def session_setup(meta):
    dim, heads, ffn, channels, height, width, h1, h2, enc_len = (int(v) for v in meta)
    p = recipes.session_params(dim, channels, h1, h2)
    sst = p["scale_shift_table"].astype(np.float32) + p["temb"].astype(np.float32).reshape(1, 1, dim)
    p["head_shift"], p["head_scale"] = sst[0, 0], sst[0, 1]
    return p, recipes.session_inputs(channels, height, width)


def _rel(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def recycled(sgold, i, p, steps):
    """The recycled latents entering step i: zeros for the prefix, else the
    bf16 copy of the last two frames of the reference's previous result."""
    if i == 0:
        return np.zeros(steps[0][1].shape[1:], np.float32)
    return bf16_round(sgold[f"session_step{i - 1}_result"][0][:, -2:])


def test_lq_projector_streaming_matches_reference(sgold):
    p, steps = session_setup(sgold["session_meta"])
    state = osess.new_lq_state()
    for i, (video, _) in enumerate(steps):
        got = osess.lq_project_stream(video[0], state, p)
        ref = bf16_from_bits(sgold[f"session_step{i}_lqproj"])[0]
        assert got.shape == ref.shape
        # about one bf16 ulp: the reference's bf16 convolutions accumulate in
        # another order (measured 0.4 % max, 0.28 % relative L2)
        rel_l2 = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert _rel(got, ref) < 1e-2 and rel_l2 < 5e-3, (i, _rel(got, ref), rel_l2)


def test_streaming_window_arithmetic():
    # prefix of 21 RGB frames, then 8-frame body blocks (runtime/constants.py)
    assert osess.streaming_window(0, 21, 2) == (0, 20, -3, 11)
    assert osess.streaming_window(21, 8, 2) == (22, 28, 19, 4)
    assert osess.streaming_window(11, 4, 2) == (12, 14, 9, 2)
    with pytest.raises(ValueError):
        osess.streaming_window(21, 1, 2)


def test_embedding_matches_reference(sgold):
    p, steps = session_setup(sgold["session_meta"])
    state = osess.new_lq_state()
    for i, (video, noise) in enumerate(steps):
        got = osess.embed(noise[0], video[0], recycled(sgold, i, p, steps), state, p)
        ref = bf16_from_bits(sgold[f"session_step{i}_hidden_in"])[0]
        assert _rel(got, ref) < 2e-2, (i, _rel(got, ref))


def test_head_matches_reference(sgold):
    p, steps = session_setup(sgold["session_meta"])
    for i, (_, noise) in enumerate(steps):
        hidden = bf16_from_bits(sgold[f"session_step{i}_hidden_out"])[0]
        result, rec = osess.head(hidden, noise[0], p)
        ref = sgold[f"session_step{i}_result"][0]
        # compare the predictions (result = noise - prediction; the noise dominates)
        got_pred, ref_pred = noise[0] - result, noise[0] - ref
        assert _rel(got_pred, ref_pred) < 2e-2, (i, _rel(got_pred, ref_pred))
        np.testing.assert_array_equal(rec, bf16_round(result[:, -2:]))


def test_layer_loop_matches_reference(sgold):
    """The oracle's layer loop (static router, cache commits, NVFP4 DiT blocks of
    oracle/block.py) from the reference's hidden state entering the first block
    to the one leaving the last block, for the prefix and both body blocks,
    with the oracle keeping its own caches across blocks. Bound: the block-level
    one (the reference's bf16 SDPA against the oracle's exact softmax, and NVFP4
    codes flipping on 1-ulp bf16 differences); measured 2.2 % relative L2 and
    at most 5.9 % max-abs on the three blocks."""
    from oracle import block as oblock
    from oracle import rope as orope
    from oracle.block import rms_norm
    from oracle.cache import RouterState
    from tests.test_gpu_block import _oracle_stack_step
    dim, heads, ffn, channels, height, width, h1, h2, enc_len = (int(v) for v in sgold["session_meta"])
    H, W = height // 32, width // 32
    span, d = H * W, dim // heads
    actions = ["recent_2", "none"]
    bp = [recipes.block_params(dim, heads, ffn, enc_len=enc_len, seed=70 + i) for i in range(2)]
    enc, tproj = bp[0]["encoder"][0], bp[0]["timestep_proj"]
    tc, ts, sc, ss = orope.rolling_tables(d, H, W)
    params = []
    for p in bp:
        lin = {n: oblock.QuantLinear(p[n + "_w"], p[n + "_b"]) for n in ("q", "k", "v", "o", "cq", "co", "up", "down")}
        cross_k = rms_norm(osess.linear(enc, p["ck_w"], p["ck_b"]), p["cnorm_k"]).reshape(-1, heads, d)
        cross_v = osess.linear(enc, p["cv_w"], p["cv_b"]).reshape(-1, heads, d)
        modulation = (p["scale_shift_table"].reshape(6, dim).astype(np.float32)
                      + tproj.reshape(6, dim).astype(np.float32))
        params.append({"_linears": lin, "modulation": modulation, "norm_q": p["norm_q"], "norm_k": p["norm_k"],
                       "cnorm_q": p["cnorm_q"], "norm2_w": p["norm2_w"], "norm2_b": p["norm2_b"],
                       "cross_k": cross_k, "cross_v": cross_v, "temporal_cos": tc, "temporal_sin": ts,
                       "spatial_cos": sc, "spatial_sin": ss})
    routers = [RouterState(a) for a in actions]
    caches = [(np.zeros((max(r.capacity, 1) * span, heads, d), np.float32),
               np.zeros((max(r.capacity, 1) * span, heads, d), np.float32)) for r in routers]
    start = 0
    for i, frames in enumerate((6, 2, 2)):
        hidden = bf16_from_bits(sgold[f"session_step{i}_hidden_in"])[0]
        got, _ = _oracle_stack_step(params, routers, caches, hidden, start, frames, H, W, heads)
        ref = bf16_from_bits(sgold[f"session_step{i}_hidden_out"])[0]
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert rel < 0.06 and _rel(got, ref) < 0.15, (i, rel, _rel(got, ref))
        start += frames


def test_lq_projector_streaming_equals_full_sequence():
    """LQ4xProj.forward_streaming projects "a consecutive RGB chunk exactly as
    full-sequence forward" (lq_proj.py:231-236): the prefix / body chunks
    21, 8, 8 streamed equal the 37 frames in one chunk (outputs 6 + 2 + 2)."""
    p = recipes.session_params()
    steps = recipes.session_inputs()
    video = np.concatenate([s[0][0] for s in steps], axis=1)
    state = osess.new_lq_state()
    streamed = np.concatenate([osess.lq_project_stream(s[0][0], state, p) for s in steps])
    full = osess.lq_project_stream(video, osess.new_lq_state(), p)
    assert streamed.shape == full.shape == (10 * 4 * 6, 256)
    # identical windows; float64 sums may differ in the last bit, flipping a rare bf16 rounding
    assert np.mean(streamed == full) > 0.99 and _rel(streamed, full) < 1e-2
