"""FlashDecoder local GQA attention oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/models/flashdecoder/flashdecoder_wan22.py:38-119
(`_local_attention`, the CPU path) and the visibility of its Triton forward
(models/flashdecoder/_local_attention_triton.py:21-131): queries are the last
QF frames of the NF key frames (frames grouped by `group_size`); a query in
group qg sees the key frames of groups (qg - temporal_window, qg], and within
a frame the keys at dy in [-wh/2, wh/2), dx in [-ww/2, ww/2) around its own
position, truncated at the grid border (no window clamping). Grouped-query
heads: query head h reads key/value head h // (HQ / HK). Softmax in float64
with scale d^-0.5.
"""
from __future__ import annotations

import numpy as np


def visibility(height, width, qf, nf, window, group_size, temporal_window, query_rows=None):
    """Boolean mask [qf*n, nf*n] of flashdecoder_wan22.py:91-107 (only the
    rows `query_rows` when given)."""
    n = height * width
    wh, ww = window
    k = np.arange(nf * n)
    kg, ky, kx = k // (group_size * n), (k % n) // width, k % width
    q = np.arange(qf * n) if query_rows is None else np.asarray(query_rows)
    qg = (q // n + nf - qf) // group_size
    dy = ky[None, :] - ((q % n) // width)[:, None]
    dx = kx[None, :] - (q % width)[:, None]
    return ((kg[None, :] <= qg[:, None]) & (kg[None, :] > qg[:, None] - temporal_window)
            & (dy >= -(wh // 2)) & (dy < wh // 2) & (dx >= -(ww // 2)) & (dx < ww // 2))


def local_gqa_attention(q, k, v, height, width, window, group_size, temporal_window, query_rows=None):
    """q [B, HQ, QF*n, D], k / v [B, HK, NF*n, D] -> [B, HQ, QF*n, D] (float32);
    with `query_rows`, only those query tokens: [B, HQ, len(query_rows), D]."""
    b, hq, tq, d = q.shape
    hk, tk = k.shape[1], k.shape[2]
    n = height * width
    qf, nf = tq // n, tk // n
    if tq % n or tk % n or qf % group_size or nf % group_size or nf < qf or hq % hk:
        raise ValueError("Invalid local grid, GQA heads or temporal group alignment.")
    mask = visibility(height, width, qf, nf, window, group_size, temporal_window, query_rows)
    if query_rows is not None:
        q = q[:, :, np.asarray(query_rows)]
    out = np.empty((b, hq, q.shape[2], d), np.float32)
    q64, k64, v64 = (np.asarray(x, np.float64) for x in (q, k, v))
    for bi in range(b):
        for h in range(hq):
            kv = h // (hq // hk)
            s = q64[bi, h] @ k64[bi, kv].T / np.sqrt(d)
            s = np.where(mask, s, -np.inf)
            s = s - s.max(-1, keepdims=True)
            p = np.exp(s)
            out[bi, h] = (p @ v64[bi, kv] / p.sum(-1, keepdims=True)).astype(np.float32)
    return out
