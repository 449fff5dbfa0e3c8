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


# ---------------------------------------------------------------- decode step
def _linear(x, p, name):
    y = x @ p[name + ".weight"].T
    b = p.get(name + ".bias")
    return y + b if b is not None else y


def _rms_norm(x, weight, eps):
    """torch.nn.RMSNorm: x * rsqrt(mean(x^2) + eps) * weight over the last dim."""
    x64 = x.astype(np.float64)
    r = 1.0 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + eps)
    return (x64 * r * weight).astype(np.float32)


def _silu(x):
    return (x / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


def rope_tables(t_pos, h_pos, w_pos, theta=10000.0, dims=(16, 24, 24)):
    """flashdecoder_wan22.py:158-224 (_RotaryEmbedding3D.frequencies): per token,
    cos / sin [tokens, 64] of (temporal | row | column) angles, every pair
    frequency repeated twice, fp32."""
    cs, sn = [], []
    for pos, d in zip((t_pos, h_pos, w_pos), dims):
        inv = (1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float32) / d))).astype(np.float32)
        ang = pos.astype(np.float32)[:, None] * inv[None, :]
        cs.append(np.repeat(np.cos(ang), 2, axis=-1))
        sn.append(np.repeat(np.sin(ang), 2, axis=-1))
    return np.concatenate(cs, -1).astype(np.float32), np.concatenate(sn, -1).astype(np.float32)


def apply_rope(x, cos, sin):
    """flashdecoder_wan22.py:226-242 on [..., tokens, 64]."""
    even, odd = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = even * cos[..., 0::2] - odd * sin[..., 0::2]
    out[..., 1::2] = even * sin[..., 1::2] + odd * cos[..., 1::2]
    return out


def token_positions(start, frames, height, width):
    t, y, x = np.meshgrid(np.arange(start, start + frames), np.arange(height), np.arange(width), indexing="ij")
    return t.ravel(), y.ravel(), x.ravel()


class DecoderOracle:
    """FlashDecoder's streaming decode (flashdecoder_wan22.py:759-874,
    _StreamingTransformer :380-497, blocks :245-378) as FlashDecoderSession.step
    (runtime/flashdecoder.py:140-175) runs it on the CPU: fp32, no autocast.
    `params` uses the reference's state-dict names; B = 1."""

    def __init__(self, params, *, dim, num_heads, num_kv_groups, depth, refinement_depth,
                 window, mean, std, eps=1e-5, window_size=2):
        self.p, self.dim, self.hq, self.hk = params, dim, num_heads, num_kv_groups
        self.depth, self.rdepth, self.window, self.eps = depth, refinement_depth, tuple(window), eps
        self.mean, self.std = np.asarray(mean, np.float32), np.asarray(std, np.float32)
        self.max_backbone, self.max_refine = window_size, 4 * window_size
        self.caches = {"backbone": [None] * depth, "temporal_refinement": [None] * refinement_depth}
        self.frame_index = 0

    def _block(self, prefix, x, cache, qr, kr, spec):
        p, n_tok = self.p, x.shape[0]
        a = prefix + "attention."
        h = _rms_norm(x, p[prefix + "attention_norm.weight"], self.eps)
        q = _linear(h, p, a + "query").reshape(n_tok, self.hq, 64).transpose(1, 0, 2)
        k = _linear(h, p, a + "key").reshape(n_tok, self.hk, 64).transpose(1, 0, 2)
        v = _linear(h, p, a + "value").reshape(n_tok, self.hk, 64).transpose(1, 0, 2)
        k = _rms_norm(k, p[a + "key_norm.weight"], self.eps)
        v = _rms_norm(v, p[a + "value_norm.weight"], self.eps)
        if cache is not None:
            k, v = np.concatenate([cache[0], k], 1), np.concatenate([cache[1], v], 1)
        q, rk = apply_rope(q, *qr), apply_rope(k, *kr)
        att = local_gqa_attention(q[None], rk[None], v[None], spec["height"], spec["width"], spec["window"],
                                  spec["group_size"], spec["temporal_window"])[0]
        x = x + _linear(att.transpose(1, 0, 2).reshape(n_tok, self.dim), p, a + "output")
        h = _rms_norm(x, p[prefix + "feed_forward_norm.weight"], self.eps)
        f = prefix + "feed_forward."
        x = x + _linear(_silu(_linear(h, p, f + "gate")) * _linear(h, p, f + "up"), p, f + "down")
        return x, (k, v)

    def _stack(self, name, x, cur, height, width):
        n = height * width
        max_frames = self.max_backbone if name == "backbone" else self.max_refine
        keep = (max_frames - cur) * n
        caches = [None if c is None or keep == 0 else (c[0][:, -keep:], c[1][:, -keep:])
                  for c in self.caches[name]]
        prev = 0 if caches[0] is None else caches[0][0].shape[1] // n
        qr = rope_tables(*token_positions(prev, cur, height, width))
        kr = rope_tables(*token_positions(0, prev + cur, height, width))
        spec = dict(height=height, width=width, window=self.window, group_size=cur,
                    temporal_window=max_frames // cur)
        out = []
        for i, c in enumerate(caches):
            x, c2 = self._block(f"{name}.blocks.{i}.", x, c, qr, kr, spec)
            out.append(c2)
        self.caches[name] = out
        return x

    def step(self, latent, lr_up):
        """latent: normalized [48, h, w]; lr_up: [3, F, 16h, 16w] (F = 1 on the
        first step, else 4) -> (rgb [3, F, 16h, 16w] clamped to [-1, 1],
        backbone hidden [n, dim], refinement hidden [4n, dim])."""
        p = self.p
        first = self.frame_index == 0
        _, height, width = latent.shape
        n = height * width
        raw = latent * self.std[:, None, None] + self.mean[:, None, None]
        f_lr = lr_up.shape[1]
        # LR stem: pixel_unshuffle(16) channels (c, i, j) of every 16 x 16 patch
        packed = lr_up.reshape(3, f_lr, height, 16, width, 16).transpose(1, 2, 4, 0, 3, 5).reshape(f_lr, n, 768)
        feats = _linear(packed, p, "lr_stem")                      # [F, n, 48]
        if first:
            feats = np.concatenate([feats[:1]] * 3 + [feats], 0)
        grouped = feats.transpose(1, 0, 2).reshape(n, 4 * 48)
        early = _linear(grouped, p, "lr_early_projection")
        late = _linear(feats.reshape(4 * n, 48), p, "lr_late_projection")
        x = _linear(raw.reshape(48, n).T, p, "latent_projection") + early
        x = self._stack("backbone", x, 1, height, width)
        backbone = x
        x = _linear(x, p, "temporal_projection").reshape(n, 4, self.dim).transpose(1, 0, 2).reshape(4 * n, self.dim)
        x = self._stack("temporal_refinement", x + late, 4, height, width)
        refine = x
        y = _linear(_silu(_linear(x, p, "spatial_projection.0")), p, "spatial_projection.2")   # [4n, 768]
        rgb = y.reshape(4, height, width, 3, 16, 16).transpose(3, 0, 1, 4, 2, 5).reshape(3, 4, 16 * height, 16 * width)
        if first:
            rgb = rgb[:, 3:]
        self.frame_index += 1
        return np.clip(rgb, -1, 1), backbone, refine
