"""Seeded input recipes shared by the golden generator and the tests.

Inputs are drawn with numpy's legacy ``RandomState`` (its streams are stable
across numpy versions) and rounded to bf16, so fixtures only need to store the
reference's outputs; the tests regenerate the inputs bit for bit.
"""
from __future__ import annotations

import numpy as np

from oracle.numerics import bf16_round


def bf16_normal(rs: np.random.RandomState, shape, std=1.0) -> np.ndarray:
    return bf16_round(rs.standard_normal(shape).astype(np.float32) * np.float32(std))


def cfg3_activation(m: int, k: int, seed: int = 2) -> np.ndarray:
    """N(0,1) with 0.1% of entries (chosen with the seed) multiplied by 20."""
    rs = np.random.RandomState(seed)
    x = rs.standard_normal((m, k)).astype(np.float32)
    idx = rs.choice(m * k, size=max(1, (m * k) // 1000), replace=False)
    x.reshape(-1)[idx] *= 20.0
    return bf16_round(x)


def cfg3_weight(n: int, k: int, seed: int = 3) -> np.ndarray:
    rs = np.random.RandomState(seed)
    return bf16_normal(rs, (n, k), 0.02)


def quant_special_rows(k: int = 64) -> np.ndarray:
    """Rows that exercise every branch of the NVFP4 quantizer: zeros, signed
    zeros, exact E2M1 thresholds and midpoints, tiny negatives (code 8),
    subnormal and clamped scales, scales that round to 448 and to the NaN code."""
    rows = []
    z = np.zeros(k, np.float32)
    rows.append(z.copy())
    nz = z.copy(); nz[::2] = -0.0; rows.append(nz)
    # amax = 6 -> scale 1 -> z = x exactly: every threshold and its neighbours
    base = np.array([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                     -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, -6.0], np.float32)
    nxt = np.nextafter(base, np.float32(np.inf)).astype(np.float32)
    prv = np.nextafter(base, np.float32(-np.inf)).astype(np.float32)
    for arr in (base, nxt, prv):
        r = np.tile(arr, k // 16).astype(np.float32)
        r[::16] = 6.0
        rows.append(r)
    tiny = np.full(k, -1e-5, np.float32); tiny[::16] = 1.0; rows.append(tiny)
    rows.append(np.full(k, 1e-6, np.float32))                  # scale clamps to 2^-9
    rows.append(np.linspace(-0.01, 0.01, k).astype(np.float32))  # subnormal scales
    big = np.full(k, 100.0, np.float32); big[::16] = 2688.0; rows.append(big)   # scale 448
    nan_sc = np.full(k, 1.0, np.float32); nan_sc[::16] = 2900.0; rows.append(nan_sc)  # >= 480 -> NaN code
    mid = np.full(k, 1.0, np.float32); mid[::16] = 2784.0; rows.append(mid)    # amax/6 = 464 tie
    rs = np.random.RandomState(7)
    for _ in range(5):
        rows.append(rs.standard_normal(k).astype(np.float32) * np.float32(10.0 ** rs.uniform(-3, 2)))
    return bf16_round(np.stack(rows))


def block_params(dim=256, heads=2, ffn=512, enc_len=16, seed=11):
    """Weights of a stand-in DiT block with the reference's module layout
    (models/transformer_wan.py:786-822): N(0, 0.02) linear weights, small
    random biases, RMSNorm/LayerNorm affine around 1/0, scale_shift_table
    randn/sqrt(dim), timestep projection N(0,1), encoder states N(0,1)."""
    rs = np.random.RandomState(seed)
    p = {}
    for name, (n, k) in {"q": (dim, dim), "k": (dim, dim), "v": (dim, dim), "o": (dim, dim),
                         "cq": (dim, dim), "ck": (dim, dim), "cv": (dim, dim), "co": (dim, dim),
                         "up": (ffn, dim), "down": (dim, ffn)}.items():
        p[name + "_w"] = bf16_normal(rs, (n, k), 0.02)
        p[name + "_b"] = bf16_normal(rs, (n,), 0.02)
    for name in ("norm_q", "norm_k", "cnorm_q", "cnorm_k", "norm2_w"):
        p[name] = bf16_round(1.0 + 0.1 * rs.standard_normal(dim).astype(np.float32))
    p["norm2_b"] = bf16_normal(rs, (dim,), 0.1)
    p["scale_shift_table"] = bf16_round(rs.standard_normal((1, 6, dim)).astype(np.float32) / np.float32(dim ** 0.5))
    p["timestep_proj"] = bf16_normal(rs, (1, 1, 6, dim))
    p["encoder"] = bf16_normal(rs, (1, enc_len, dim))
    return p


def block_inputs(n_tokens, cap_tokens, dim=256, seed=12):
    rs = np.random.RandomState(seed)
    hidden = bf16_normal(rs, (1, n_tokens, dim))
    pk = bf16_normal(rs, (1, cap_tokens, dim))
    pv = bf16_normal(rs, (1, cap_tokens, dim))
    return hidden, pk, pv


def session_params(dim=256, channels=16, h1=64, h2=128, seed=31):
    """Weights of the session glue of a stand-in model (runtime/transformer.py:317-349,
    models/lq_proj.py): patch embedding, sr_proj, proj_out, the LQ projector
    (conv1 over 16x16-unshuffled RGB = 768 channels, conv2, channel norms,
    out_proj), the output scale_shift_table (kept fp32) and temb."""
    rs = np.random.RandomState(seed)
    bn = lambda shape, std: bf16_normal(rs, shape, std)
    norm = lambda n: bf16_round(1.0 + 0.1 * rs.standard_normal(n).astype(np.float32))
    return {
        "patch_w": bn((dim, channels, 1, 2, 2), 0.1), "patch_b": bn((dim,), 0.02),
        "sr_w": bn((dim, dim), 0.02), "sr_b": bn((dim,), 0.02),
        "proj_out_w": bn((channels * 4, dim), 0.02), "proj_out_b": bn((channels * 4,), 0.02),
        "conv1_w": bn((h1, 768, 4, 3, 3), 0.02), "conv1_b": bn((h1,), 0.02), "norm1_w": norm(h1),
        "conv2_w": bn((h2, h1, 4, 3, 3), 0.02), "conv2_b": bn((h2,), 0.02), "norm2_w": norm(h2),
        "out_w": bn((dim, h2), 0.02), "out_b": bn((dim,), 0.02),
        "scale_shift_table": bn((1, 2, dim), dim ** -0.5), "temb": bn((1, 1, dim), 1.0),
    }


def session_inputs(channels=16, height=128, width=192, seed=32, rgb_frames=(21, 8, 8)):
    """Per step: (LQ RGB video [1, 3, T, H, W] uniform(-1, 1) in bf16 values,
    noise [1, C, frames, H/16, W/16] N(0, 1) fp32); prefix then body blocks."""
    rs = np.random.RandomState(seed)
    steps = []
    for i, rgb in enumerate(rgb_frames):
        frames = 6 if i == 0 else 2
        video = bf16_round(rs.uniform(-1, 1, (1, 3, rgb, height, width)).astype(np.float32))
        noise = rs.standard_normal((1, channels, frames, height // 16, width // 16)).astype(np.float32)
        steps.append((video, noise))
    return steps


# FlashDecoder local GQA attention cases:
# tag: (B, HQ, HK, D, height, width, window, group_size, temporal_window, QF, NF)
LOCAL_GQA_CASES = {
    "a": (1, 8, 2, 64, 6, 20, (4, 8), 4, 2, 4, 8),
    "b": (1, 4, 1, 64, 9, 7, (6, 4), 1, 2, 1, 3),
    "c": (2, 4, 4, 32, 5, 6, (10, 12), 2, 1, 2, 6),
}


def local_gqa_inputs(tag, seed=41):
    """q [B, HQ, QF*n, D], k / v [B, HK, NF*n, D], N(0, 1) fp32, for one case."""
    b, hq, hk, d, h, w, _, _, _, qf, nf = LOCAL_GQA_CASES[tag]
    rs = np.random.RandomState(seed + ord(tag))
    n = h * w
    q = rs.standard_normal((b, hq, qf * n, d)).astype(np.float32)
    k = rs.standard_normal((b, hk, nf * n, d)).astype(np.float32)
    v = rs.standard_normal((b, hk, nf * n, d)).astype(np.float32)
    return q, k, v


def cfg3_activation_large(m: int, k: int, seed: int = 2) -> np.ndarray:
    """cfg3 activation for the largest shapes (same distribution as
    cfg3_activation: N(0,1), 0.1 % of the entries x20, bf16 values) drawn with
    numpy's Generator, whose sampling without replacement stays fast at 1e8
    entries."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    idx = rng.choice(m * k, size=max(1, (m * k) // 1000), replace=False)
    x.reshape(-1)[idx] *= 20.0
    # bf16_round's ties-to-even in place on the 32-bit patterns: every value
    # is finite and far below overflow, so the 32-bit sum cannot wrap
    u = x.view(np.uint32)
    u += np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    u &= np.uint32(0xFFFF0000)
    return x


def lq_frames_u8(n: int, h: int, w: int, seed: int = 60) -> np.ndarray:
    """LQ RGB frames as a decoder delivers them, uint8 [n, h, w, 3]: uniform
    noise smoothed by a 3x3 box filter along both axes (integer mean), so
    neighbouring pixels are correlated like video."""
    rs = np.random.RandomState(seed)
    x = rs.randint(0, 256, (n, h + 2, w + 2, 3)).astype(np.int32)
    acc = sum(x[:, dy:dy + h, dx:dx + w] for dy in range(3) for dx in range(3))
    return (acc // 9).astype(np.uint8)


# FlashDecoder decode-step cases: model size (dim, query heads, KV heads,
# backbone depth, refinement depth, mlp ratio), spatial window, latent grid
# (h, w) and the number of decode steps. "s" is a small stand-in; "S" has the
# released variant's widths (dim 512, 8 / 2 heads, SwiGLU 2048) at a reduced
# depth and window.
DECODER_CASES = {
    "s": dict(dim=128, num_heads=2, num_kv_groups=1, depth=2, refinement_depth=1, mlp_ratio=2.0,
              window=(4, 4), h=4, w=6, steps=4),
    "S": dict(dim=512, num_heads=8, num_kv_groups=2, depth=2, refinement_depth=1, mlp_ratio=4.0,
              window=(6, 6), h=6, w=8, steps=3),
}


def decoder_params(tag, seed=51):
    """fp32 state dict of a FlashDecoder (the reference's parameter names,
    flashdecoder_wan22.py:655-688) for one DECODER_CASES entry: linear weights
    N(0, 1/fan_in), biases N(0, 0.02), norm weights 1 + N(0, 0.1)."""
    c = DECODER_CASES[tag]
    rs = np.random.RandomState(seed + ord(tag))
    dim, hd = c["dim"], 64
    kv = c["num_kv_groups"] * hd
    hidden = int(dim * c["mlp_ratio"])
    p = {}

    def lin(name, n, k, bias=True):
        p[name + ".weight"] = (rs.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
        if bias:
            p[name + ".bias"] = (rs.standard_normal(n) * 0.02).astype(np.float32)

    def norm(name, n):
        p[name + ".weight"] = (1.0 + rs.standard_normal(n) * 0.1).astype(np.float32)

    def block(prefix):
        norm(prefix + "attention_norm", dim)
        lin(prefix + "attention.query", dim, dim)
        lin(prefix + "attention.key", kv, dim)
        lin(prefix + "attention.value", kv, dim)
        norm(prefix + "attention.key_norm", hd)
        norm(prefix + "attention.value_norm", hd)
        lin(prefix + "attention.output", dim, dim)
        norm(prefix + "feed_forward_norm", dim)
        lin(prefix + "feed_forward.gate", hidden, dim)
        lin(prefix + "feed_forward.up", hidden, dim)
        lin(prefix + "feed_forward.down", dim, hidden)

    lin("latent_projection", dim, 48)
    for i in range(c["depth"]):
        block(f"backbone.blocks.{i}.")
    lin("temporal_projection", 4 * dim, dim)
    for i in range(c["refinement_depth"]):
        block(f"temporal_refinement.blocks.{i}.")
    lin("spatial_projection.0", hidden, dim)
    lin("spatial_projection.2", 3 * 16 * 16, hidden)
    lin("lr_stem", 48, 3 * 16 * 16)
    lin("lr_early_projection", dim, 4 * 48, bias=False)
    lin("lr_late_projection", dim, 48, bias=False)
    return p


def decoder_inputs(tag, seed=52):
    """The decoder's streaming inputs for one case: normalized DiT latents
    [1, 48, steps, h, w] N(0, 1); the latent normalization (mean N(0, 0.5),
    std U(0.5, 2), 48 each); the target-resolution LQ frames lr_up
    [1, 3, 1 + 4 (steps - 1), 16 h, 16 w] in [-1, 1] (uniform noise smoothed
    over 4 x 4 pixels)."""
    c = DECODER_CASES[tag]
    rs = np.random.RandomState(seed + ord(tag))
    steps, h, w = c["steps"], c["h"], c["w"]
    latents = rs.standard_normal((1, 48, steps, h, w)).astype(np.float32)
    mean = (rs.standard_normal(48) * 0.5).astype(np.float32)
    std = rs.uniform(0.5, 2.0, 48).astype(np.float32)
    frames = 1 + 4 * (steps - 1)
    coarse = rs.uniform(-1, 1, (1, 3, frames, 4 * h, 4 * w)).astype(np.float32)
    lr_up = np.repeat(np.repeat(coarse, 4, axis=3), 4, axis=4)
    return latents, mean, std, np.ascontiguousarray(lr_up)


# Colour correction cases: (frames, decoded height, width, LQ height, width).
COLORFIX_CASES = {"a": (2, 48, 80, 12, 20), "b": (3, 36, 52, 9, 13)}


def colorfix_inputs(tag, seed=71):
    """decoded [1, 3, T, H, W] fp32 in [-1, 1] (smooth noise plus a colour
    cast), the AdaIN reference of the same shape, and LQ uint8 [T, h, w, 3]."""
    t, hh, ww, h, w = COLORFIX_CASES[tag]
    rs = np.random.RandomState(seed + ord(tag))
    coarse = rs.uniform(-1, 1, (1, 3, t, hh // 4 + 1, ww // 4 + 1)).astype(np.float32)
    dec = np.repeat(np.repeat(coarse, 4, axis=3), 4, axis=4)[:, :, :, :hh, :ww]
    dec = np.clip(dec * 0.8 + rs.uniform(-0.2, 0.2, dec.shape) + 0.1, -1, 1).astype(np.float32)
    ref = np.clip(rs.uniform(-1, 1, dec.shape) * 0.5 - 0.2, -1, 1).astype(np.float32)
    lq = rs.randint(0, 256, (t, h, w, 3)).astype(np.uint8)
    return dec, ref, lq
