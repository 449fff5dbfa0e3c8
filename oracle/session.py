"""Session glue oracle (test infrastructure; see oracle/__init__.py).

Restates the non-layer parts of recavsr_infer/runtime/transformer.py:279-349
(TransformerSession.step) and the LQ projector of models/lq_proj.py in numpy:

* CausalConv3d.forward_streaming (lq_proj.py:80-139): strided causal conv with
  kernel (4, 3, 3), spatial padding 1, temporal history of kernel-1 frames and
  the first frame replicated where the window starts before frame 0;
* ChannelRMSNorm3d (lq_proj.py:26-40) and SiLU, pixel unshuffle by 16
  (lq_proj.py:279-285), out_proj over "(t h w) c" tokens (:297-302);
* patch embedding (Conv3d with kernel = stride = (1, 2, 2)), sr_proj, the
  output head (LayerNorm without affine in fp32, * (1 + scale) + shift, bf16,
  proj_out, unpatchify) and `noise - prediction` (transformer.py:317-349).

With bf16=True every value is rounded to bf16 where the reference's bf16 model
rounds (the output of each conv / linear / norm / activation, each residual
add); accumulations run in float64.
"""
from __future__ import annotations

import numpy as np

from .block import layer_norm
from .numerics import bf16_round

KT = 4


def _r(x, bf16):
    return bf16_round(np.asarray(x, np.float32)) if bf16 else np.asarray(x, np.float32)


def streaming_window(seen, chunk, stride, kernel=KT):
    """lq_proj.py:84-100,125: (next endpoint, last endpoint, first needed frame, outputs)."""
    if chunk <= 0:
        raise ValueError("A streaming convolution chunk cannot be empty.")
    next_end = (seen + stride - 1) // stride * stride
    last_in = seen + chunk - 1
    if next_end > last_in:
        raise ValueError("Streaming LQ chunk is too short")
    last_end = last_in // stride * stride
    return next_end, last_end, next_end - (kernel - 1), 1 + (last_end - next_end) // stride


def conv3d(x, w, b, stride_t, stride_s):
    """x [Cin, T, H, W], w [Cout, Cin, kt, 3, 3], spatial padding 1 -> [Cout, To, Ho, Wo] (float64)."""
    cin, t, h, wd = x.shape
    kt = w.shape[2]
    xp = np.zeros((cin, t, h + 2, wd + 2), np.float64)
    xp[:, :, 1:-1, 1:-1] = x
    to = (t - kt) // stride_t + 1
    ho, wo = (h - 1) // stride_s + 1, (wd - 1) // stride_s + 1
    out = np.zeros((w.shape[0], to, ho, wo), np.float64)
    w64 = np.asarray(w, np.float64)
    for dt in range(kt):
        for dy in range(3):
            for dx in range(3):
                sl = xp[:, dt:dt + stride_t * (to - 1) + 1:stride_t,
                        dy:dy + stride_s * (ho - 1) + 1:stride_s,
                        dx:dx + stride_s * (wo - 1) + 1:stride_s]
                out += np.einsum("oc,cthw->othw", w64[:, :, dt, dy, dx], sl)
    if b is not None:
        out += np.asarray(b, np.float64)[:, None, None, None]
    return out


def causal_conv_stream(x, state, w, b, stride_t, stride_s, bf16=True):
    """CausalConv3d.forward_streaming (lq_proj.py:80-139) on x [C, T, H, W];
    state = {"history": array | None, "seen": int}, updated."""
    chunk = x.shape[1]
    next_end, last_end, needed, n_out = streaming_window(state["seen"], chunk, stride_t)
    hist = state["history"]
    if hist is None:
        combined, cstart = x, state["seen"]
    else:
        combined = np.concatenate([hist, x], 1)
        cstart = state["seen"] - hist.shape[1]
    inp = combined[:, max(needed, 0) - cstart:last_end - cstart + 1]
    if needed < 0:
        inp = np.concatenate([np.repeat(combined[:, :1], -needed, 1), inp], 1)
    out = conv3d(inp, w, b, stride_t, stride_s)
    assert out.shape[1] == n_out
    state["history"] = combined[:, -(KT - 1):].copy()
    state["seen"] += chunk
    return _r(out, bf16)


def channel_rms_norm(x, w, eps=1e-6, bf16=True):
    """ChannelRMSNorm3d (lq_proj.py:26-40) over dim 0 of x [C, ...]."""
    x64 = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt((x64 ** 2).mean(0, keepdims=True) + eps)
    shape = (-1,) + (1,) * (x.ndim - 1)
    return _r(x64 * r * np.asarray(w, np.float64).reshape(shape), bf16)


def silu(x, bf16=True):
    x64 = np.asarray(x, np.float64)
    return _r(x64 / (1.0 + np.exp(-x64)), bf16)


def pixel_unshuffle(video, r=16):
    """[C, T, H, W] -> [C*r*r, T, H/r, W/r], channel (c*r + i)*r + j (lq_proj.py:279-285)."""
    c, t, h, w = video.shape
    v = video.reshape(c, t, h // r, r, w // r, r)
    return v.transpose(0, 3, 5, 1, 2, 4).reshape(c * r * r, t, h // r, w // r)


def linear(x, w, b, bf16=True):
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if b is not None:
        y = y + np.asarray(b, np.float64)
    return _r(y, bf16)


def lq_project_stream(video, state, p, bf16=True):
    """LQ4xProj.forward_streaming (lq_proj.py:231-246, 287-302): video [3, T, H, W]
    -> tokens [T' * H/32 * W/32, out]; state = {"conv1": {...}, "conv2": {...}}."""
    x = pixel_unshuffle(_r(video, bf16))
    x = causal_conv_stream(x, state["conv1"], p["conv1_w"], p["conv1_b"], 2, 1, bf16)
    x = silu(channel_rms_norm(x, p["norm1_w"], bf16=bf16), bf16)
    x = causal_conv_stream(x, state["conv2"], p["conv2_w"], p["conv2_b"], 2, 2, bf16)
    x = silu(channel_rms_norm(x, p["norm2_w"], bf16=bf16), bf16)
    tokens = x.reshape(x.shape[0], -1).T
    return linear(tokens, p["out_w"], p["out_b"], bf16)


def new_lq_state():
    return {"conv1": {"history": None, "seen": 0}, "conv2": {"history": None, "seen": 0}}


def patch_embed(lat, w, b, bf16=True):
    """Conv3d kernel = stride = (1, 2, 2) on lat [C, F, h, w] -> tokens [(f, y, x), dim]
    (transformer.py:321, flatten(2).transpose(1, 2))."""
    c, f, h, wd = lat.shape
    x = _r(lat, bf16).reshape(c, f, h // 2, 2, wd // 2, 2).transpose(1, 2, 4, 0, 3, 5)
    rows = x.reshape(f * (h // 2) * (wd // 2), c * 4)
    return linear(rows, np.asarray(w).reshape(w.shape[0], -1), b, bf16)


def embed(noise, lq, recycle, lq_state, p, bf16=True):
    """hidden = patch(noise) + lq_proj(lq) + sr_proj(patch(recycle)) (transformer.py:321-328)."""
    h = patch_embed(noise, p["patch_w"], p["patch_b"], bf16)
    h = _r(h + lq_project_stream(lq, lq_state, p, bf16), bf16)
    rec = patch_embed(recycle, p["patch_w"], p["patch_b"], bf16)
    return _r(h + linear(rec, p["sr_w"], p["sr_b"], bf16), bf16)


def head(hidden, noise, p, recycle_frames=2, bf16=True):
    """transformer.py:338-349: (noise - unpatchify(proj_out(LN(h)*(1+scale)+shift)),
    bf16 copy of its last recycle_frames frames)."""
    c, f, h, w = noise.shape
    y = layer_norm(np.asarray(hidden, np.float32)) * (1 + np.asarray(p["head_scale"], np.float32)) \
        + np.asarray(p["head_shift"], np.float32)
    pred = linear(_r(y, bf16), p["proj_out_w"], p["proj_out_b"], bf16)
    pred = pred.reshape(f, h // 2, w // 2, 2, 2, c).transpose(5, 0, 1, 3, 2, 4).reshape(c, f, h, w)
    result = (np.asarray(noise, np.float32) - pred.astype(np.float32)).astype(np.float32)
    return result, bf16_round(result[:, f - recycle_frames:])
