"""RoPE oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/runtime/rope.py:11-82 (tables), :23-30 (apply_rotary)
and :33-47 (apply_temporal). The 1-D table is the standard rotary table the
reference takes from diffusers 0.37.1 ``get_1d_rotary_pos_embed`` (theta
10000, float64 frequencies theta^(-2i/dim), cos/sin of pos*freq, each pair
frequency repeated twice, cast to float32).
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_round, round_to


def rotary_table(dim: int, size: int) -> tuple[np.ndarray, np.ndarray]:
    freqs = 1.0 / (10000.0 ** (np.arange(0, dim, 2, dtype=np.float64)[: dim // 2] / dim))
    ang = np.outer(np.arange(size, dtype=np.float64), freqs)
    return (np.repeat(np.cos(ang), 2, axis=1).astype(np.float32),
            np.repeat(np.sin(ang), 2, axis=1).astype(np.float32))


def rolling_tables(head_dim: int, height: int, width: int, training_frames: int = 22):
    """rope.py:50-82 -> (temporal_cos [22, td/2], temporal_sin, spatial_cos [H*W, d], spatial_sin)."""
    sd = 2 * (head_dim // 6)
    td = head_dim - 2 * sd
    ct, st = rotary_table(td, training_frames)
    ch, sh = rotary_table(sd, height)
    cw, sw = rotary_table(sd, width)
    ones = np.ones((height, width, td), np.float32)
    zeros = np.zeros((height, width, td), np.float32)
    scos = np.concatenate([ones, np.broadcast_to(ch[:, None], (height, width, sd)),
                           np.broadcast_to(cw[None], (height, width, sd))], -1)
    ssin = np.concatenate([zeros, np.broadcast_to(sh[:, None], (height, width, sd)),
                           np.broadcast_to(sw[None], (height, width, sd))], -1)
    return (np.ascontiguousarray(ct[:, ::2]), np.ascontiguousarray(st[:, ::2]),
            scos.reshape(height * width, head_dim).astype(np.float32),
            ssin.reshape(height * width, head_dim).astype(np.float32))


def apply_rotary(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rope.py:23-30: fp32 pair rotation, then bf16 rounding. x [..., d]; cos/sin broadcastable."""
    even, odd = x[..., 0::2].astype(np.float32), x[..., 1::2].astype(np.float32)
    c, s = cos[..., 0::2].astype(np.float32), sin[..., 0::2].astype(np.float32)
    out = np.empty(np.broadcast_shapes(x.shape, cos.shape), np.float32)
    out[..., 0::2] = even * c - odd * s
    out[..., 1::2] = even * s + odd * c
    return bf16_round(out)


def apply_temporal(x: np.ndarray, positions, tcos: np.ndarray, tsin: np.ndarray, span: int,
                   dtype: str = "bf16"):
    """rope.py:33-47: x [planes*span, heads, d]; rotate dims < 2*tcos.shape[1] by plane position."""
    td = tcos.shape[-1] * 2
    planes = len(positions)
    f = x.reshape(planes, span, x.shape[-2], x.shape[-1]).astype(np.float32)
    pos = np.asarray(positions, dtype=np.int64)
    c = tcos[pos][:, None, None, :]
    s = tsin[pos][:, None, None, :]
    even, odd = f[..., :td:2], f[..., 1:td:2]
    out = f.copy()
    out[..., :td:2] = even * c - odd * s
    out[..., 1:td:2] = even * s + odd * c
    out[..., :td] = round_to(out[..., :td], dtype)
    return out.reshape(x.shape)
