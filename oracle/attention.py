"""Routed attention oracle (test infrastructure; see oracle/__init__.py).

One restatement covers both reference paths:
* recavsr_infer/kernels/local_attention.py:18-169 (``_paired_local``): per
  query (qy, qx) the visible keys of every visible plane are rows
  [top, top+WH) x cols [left, left+WW) with top = clamp(qy - WH//2, 0, H-WH),
  left = clamp(qx - WW//2, 0, W-WW), WH = min(H, window_h), WW = min(W, window_w)
  (:98-99, :141-148, :213); past planes with slot < 0 are skipped (:118-120).
* :286-325 (``sdpa_attention``): the window covers the grid, so every key of
  every visible plane is seen; empty slots are masked out (:317-318).
Q and K get the temporal rotation of rope.apply_temporal (fp32, bf16 cast) at
their plane positions; scores/softmax are computed in float64 (exact softmax,
no probability rounding) and the output is rounded to bf16.
"""
from __future__ import annotations

import numpy as np

from .numerics import round_to
from .rope import apply_temporal


def window_bounds(coord, extent, window):
    w = min(extent, window)
    return np.clip(coord - w // 2, 0, extent - w), w


def routed_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                     height, width, window_h, window_w, dtype="bf16", compute_dtype=np.float64,
                     query_rows=None):
    """Arrays are [B, tokens, heads, d] float32 holding bf16 (or fp16, with
    dtype="fp16") values; returns the same shape rounded to that dtype.
    query_rows (optional): compute only these query tokens (indices into the
    query block); the result is then [B, len(query_rows), heads, d]."""
    q = np.asarray(q, np.float32)
    span = height * width
    bsz, nq, heads, d = q.shape
    frames = nq // span
    slots = [int(s) for s in np.asarray(slots).reshape(-1)]
    ppos = [int(p) for p in np.asarray(past_positions).reshape(-1)]
    qpos = [int(p) for p in np.asarray(query_positions).reshape(-1)]
    ys, xs = np.divmod(np.arange(span), width)
    top, wh = window_bounds(ys, height, window_h)
    left, ww = window_bounds(xs, width, window_w)
    allowed = ((ys[None, :] >= top[:, None]) & (ys[None, :] < top[:, None] + wh)
               & (xs[None, :] >= left[:, None]) & (xs[None, :] < left[:, None] + ww))
    out = np.zeros_like(q)
    for b in range(bsz):
        qr = apply_temporal(q[b], qpos, cos, sin, span, dtype).astype(compute_dtype)
        keys, vals, masks = [], [], []
        for s, p in zip(slots, ppos):
            if s < 0:
                continue
            k = pk[b, s * span:(s + 1) * span]
            keys.append(apply_temporal(k, [p], cos, sin, span, dtype))
            vals.append(pv[b, s * span:(s + 1) * span])
            masks.append(allowed)
        for f in range(frames):
            keys.append(apply_temporal(ck[b, f * span:(f + 1) * span], [qpos[f]], cos, sin, span, dtype))
            vals.append(cv[b, f * span:(f + 1) * span])
            masks.append(allowed)
        kk = np.concatenate(keys, 0).astype(compute_dtype)   # [nk, heads, d]
        vv = np.concatenate(vals, 0).astype(compute_dtype)
        mm = np.concatenate(masks, 1)                      # [span, nk]
        if query_rows is None:
            mask = np.tile(mm, (frames, 1))                # [nq, nk]
        else:                                              # query token i sees row i % span of mm
            rows = np.asarray(query_rows)
            qr, mask = qr[rows], mm[rows % span]
            if b == 0:
                out = np.zeros((bsz, len(rows), heads, d), np.float32)
        scale = d ** -0.5
        for h in range(heads):
            sc = (qr[:, h] @ kk[:, h].T) * scale
            sc = np.where(mask, sc, -np.inf)
            sc -= sc.max(1, keepdims=True)
            p = np.exp(sc)
            p /= p.sum(1, keepdims=True)
            out[b, :, h] = (p @ vv[:, h]).astype(np.float32)
    return round_to(out, dtype)


def plain_attention(q, k, v, compute_dtype=np.float64):
    """Unmasked SDPA (cross-attention, recavsr_infer/runtime/transformer.py:123-128).
    q [N, heads, d], k/v [L, heads, d] -> bf16-valued [N, heads, d]."""
    q = np.asarray(q, compute_dtype)
    k = np.asarray(k, compute_dtype)
    v = np.asarray(v, compute_dtype)
    out = np.empty(q.shape, np.float32)
    for h in range(q.shape[1]):
        sc = (q[:, h] @ k[:, h].T) * compute_dtype(q.shape[-1] ** -0.5)
        sc -= sc.max(1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(1, keepdims=True)
        out[:, h] = p @ v[:, h]
    return round_to(out, "bf16")
