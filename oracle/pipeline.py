"""Host-pipeline oracle (test infrastructure; see oracle/__init__.py).

Restates the frame preparation and strip blending around the DiT:

* recavsr_infer/video.py:138-179: `enlarge_block` (cv2.resize INTER_LINEAR of
  uint8 RGB frames to the scaled size, the last frame repeated to fill the
  block) and `block_tensor` (uint8 -> fp32, x / 127.5 - 1, the width then the
  height padded to a multiple of 32 with reflect, or replicate when the pad is
  not smaller than the size).
* recavsr_infer/frames.py:29-40: `scaled_size`; video.py:119-130 `block_schedule`.
* recavsr_infer/strips.py:24-99: `strip_columns`, `column_weights`,
  `blend_strips`' per-frame canvas arithmetic.

cv2.resize's 8-bit bilinear arithmetic (opencv-python-headless 4.13, the
reference's pinned `>=4.13`; its library code is not in the reference and is
restated here from its observable outputs, which tests/test_oracle_pipeline.py
checks against cv2 itself on random geometries):
  per output column x: f = fl32((x + 0.5) * s - 0.5) with s = 1 / (W / w) in
  double; i = floor(f), f -= i; a column left of the image (i < 0) or at / past
  its last column (i >= w - 1) takes i clamped and f = 0; weights
  (rint((1 - f) * 2048), rint(f * 2048)) (round half to even), rows as
  horizontal sums S = src[i] * a0 + src[i + 1] * a1 (int);
  per output row y: the same f, i without the clamp of f (only the two source
  row indices i, i + 1 are clipped to the image), weights b0, b1 likewise;
  out = ((S0 >> 4) * b0 >> 16) + ((S1 >> 4) * b1 >> 16), then (out + 2) >> 2,
  saturated to [0, 255].
"""
from __future__ import annotations

import math

import numpy as np

TOKEN_STRIDE = 32           # recavsr_infer/runtime/constants.py (SPATIAL_TOKEN_STRIDE)
COEF_SCALE = 2048           # 11 fractional bits of the bilinear weights


def scaled_size(height: int, width: int, scale: float = 4.0) -> tuple[int, int]:
    """frames.py:29-40: each dimension times the scale, rounded half up."""
    scale = float(scale)
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("Scale must be a finite positive number.")
    if height < 1 or width < 1:
        raise ValueError("Input dimensions must be positive.")
    out = tuple(math.floor(x * scale + 0.5) for x in (height, width))
    if min(out) < 1:
        raise ValueError("Scale produces an empty output dimension.")
    return out


def block_schedule(total: int, prefix: int = 21, body: int = 8):
    """video.py:119-130: (start, valid RGB frames, padded RGB frames) per block."""
    if total < 1:
        raise ValueError("A video must contain at least one frame.")
    start = 0
    while start < total:
        block = prefix if start == 0 else body
        valid = min(block, total - start)
        yield start, valid, block
        start += valid


def _axis(src: int, dst: int, clamp_fraction: bool):
    scale = 1.0 / (dst / src)
    f = ((np.arange(dst) + 0.5) * scale - 0.5).astype(np.float32)
    i = np.floor(f).astype(np.int64)
    f = (f - i).astype(np.float32)
    if clamp_fraction:
        lo, hi = i < 0, i >= src - 1
        f[lo], i[lo] = 0, 0
        f[hi], i[hi] = 0, src - 1
    w0 = np.rint((np.float32(1) - f) * COEF_SCALE).astype(np.int64)
    w1 = np.rint(f * COEF_SCALE).astype(np.int64)
    return np.clip(i, 0, src - 1), np.clip(i + 1, 0, src - 1), w0, w1


def resize_linear_u8(img: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """cv2.resize(img, (out_w, out_h), interpolation=INTER_LINEAR) of a uint8
    [h, w, c] image (the arithmetic in the module docstring)."""
    h, w, _ = img.shape
    x0, x1, a0, a1 = _axis(w, out_w, True)
    y0, y1, b0, b1 = _axis(h, out_h, False)
    x = img.astype(np.int64)
    rows = x[:, x0] * a0[None, :, None] + x[:, x1] * a1[None, :, None]
    v = ((rows[y0] >> 4) * b0[:, None, None] >> 16) + ((rows[y1] >> 4) * b1[:, None, None] >> 16)
    return np.clip((v + 2) >> 2, 0, 255).astype(np.uint8)


def enlarge_block(chunk: np.ndarray, size, block: int) -> np.ndarray:
    """video.py:153-174: uint8 [valid, h, w, 3] -> uint8 [block, H, W, 3]."""
    frames = [resize_linear_u8(f, size[0], size[1]) for f in chunk]
    return np.stack(frames + frames[-1:] * (block - len(frames)))


def _pad_index(n: int, pad: int) -> np.ndarray:
    """Source index of every position of an axis of n values padded by `pad`
    at the end: reflect when pad < n (torch F.pad reflect), else replicate."""
    idx = np.arange(n + pad)
    tail = idx >= n
    if pad < n:
        idx[tail] = 2 * (n - 1) - idx[tail]
    else:
        idx[tail] = n - 1
    return idx


def block_tensor(enlarged: np.ndarray, reciprocal: bool = False) -> np.ndarray:
    """video.py:165-179 on the enlarged uint8 [block, H, W, 3] frames:
    fp32 [1, 3, block, Hp, Wp], x / 127.5 - 1, padded to the token stride.
    torch divides by the scalar on the CPU but multiplies by its fp32
    reciprocal on CUDA; reciprocal=True restates the CUDA arithmetic."""
    frames, h, w, _ = enlarged.shape
    x = np.transpose(enlarged, (3, 0, 1, 2)).astype(np.float32)
    if reciprocal:
        x = (x * (np.float32(1) / np.float32(127.5)) - np.float32(1.0)).astype(np.float32)
    else:
        x = (x / np.float32(127.5) - np.float32(1.0)).astype(np.float32)
    ph, pw = (-h) % TOKEN_STRIDE, (-w) % TOKEN_STRIDE
    x = x[:, :, _pad_index(h, ph)][:, :, :, _pad_index(w, pw)]
    return x[None]


def strip_columns(width: int, strips: int, overlap: int, scale: float):
    """strips.py:24-46: equal-width LQ column ranges [x0, x1) covering 0..width."""
    if strips < 2:
        return [(0, width)]
    step = 1
    if float(scale).is_integer():
        step = TOKEN_STRIDE // math.gcd(TOKEN_STRIDE, int(scale))
    base = math.ceil((width + (strips - 1) * overlap) / strips)
    strip = min(width, -(-base // step) * step)
    starts = [round(i * (width - strip) / (strips - 1)) for i in range(strips)]
    cols = [(x, x + strip) for x in starts]
    for (_, a1), (b0, _) in zip(cols, cols[1:]):
        if a1 - b0 < 1:
            raise ValueError("Strips do not overlap; increase --strip-overlap.")
    return cols


def column_weights(columns, scale: float, out_width: int):
    """strips.py:48-69: per strip (output x offset, fp32 feather weights)."""
    placed = [(round(x0 * scale), round(x1 * scale)) for x0, x1 in columns]
    weights = []
    for i, (o0, o1) in enumerate(placed):
        w = np.ones(o1 - o0, dtype=np.float32)
        if i > 0:
            ramp = placed[i - 1][1] - o0
            w[:ramp] = np.minimum(w[:ramp], (np.arange(ramp) + 0.5) / ramp)
        if i < len(placed) - 1:
            ramp = o1 - placed[i + 1][0]
            w[-ramp:] = np.minimum(w[-ramp:], (np.arange(ramp)[::-1] + 0.5) / ramp)
        weights.append((o0, w))
    if placed[-1][1] != out_width:
        raise ValueError("Strips must cover the scaled frame exactly.")
    return weights


def feather_total(weights, out_width: int) -> np.ndarray:
    """strips.py:82-84: the per-column sum of the strips' weights, in strip order."""
    total = np.zeros(out_width, dtype=np.float32)
    for o0, w in weights:
        total[o0:o0 + len(w)] += w
    return total


def blend_frame(frames, weights, total, height: int, width: int) -> np.ndarray:
    """strips.py:85-97 for one output frame: fp32 canvas of f * w summed in
    strip order, divided by the total, + 0.5, clipped, truncated to uint8."""
    canvas = np.zeros((height, width, 3), dtype=np.float32)
    for f, (o0, w) in zip(frames, weights):
        canvas[:, o0:o0 + len(w)] += f * w[None, :, None]
    canvas /= total[None, :, None]
    return np.clip(canvas + 0.5, 0, 255).astype(np.uint8)
