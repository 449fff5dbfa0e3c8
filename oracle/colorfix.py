"""Colour-correction oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/color_fix.py:18-117:

* `adain_color_fix` (:58-81): per frame and RGB channel of [B, 3, T, H, W]
  tensors in [-1, 1]: content / reference mapped to [0, 1] by (x + 1) * 0.5,
  spatial mean and variance (sample variance unless the plane has one pixel),
  (content - mean_c) * sqrt((var_r + 1e-5) / (var_c + 1e-5)) + mean_r, back
  by * 2 - 1. Statistics in float64 here (the reference's CUDA reduction order
  is not reproducible; the tolerance covers it).
* `wavelet_color_fix` (:84-117): content = clamp((decoded + 1) * 0.5, 0, 1);
  reference = clamp(bicubic(lq / 255), 0, 1) at the decoded size (torch's
  upsample_bicubic2d, align_corners=False: Keys' cubic convolution with
  A = -0.75, source x = (dst + 0.5) * in / out - 0.5, taps clamped to the
  image); then 5 levels (dilations 1, 2, 4, 8, 16) of the 3x3 kernel
  [1, 2, 1]^T [1, 2, 1] / 16 with replicate padding, high += low - blur per
  level on the content (summed per level, not telescoped) and the reference
  blurred alongside; fixed = clamp(high + low_reference, 0, 1); uint8
  round(fixed * 255) (half to even), [T, H, W, 3]. fp32 arithmetic.
"""
from __future__ import annotations

import numpy as np

A = np.float32(-0.75)


def adain_color_fix(decoded: np.ndarray, reference: np.ndarray) -> np.ndarray:
    """[B, 3, T, H, W] in [-1, 1] (any float) -> fp32 of the same shape."""
    if decoded.ndim != 5 or decoded.shape[1] != 3 or decoded.shape != reference.shape:
        raise ValueError("Color correction expects matching [B,3,T,H,W] tensors.")
    c = (decoded.astype(np.float32) + np.float32(1)) * np.float32(0.5)
    r = (reference.astype(np.float32) + np.float32(1)) * np.float32(0.5)
    hw = c.shape[-2] * c.shape[-1]
    ddof = 1 if hw > 1 else 0
    cm = c.astype(np.float64).mean(axis=(-2, -1), keepdims=True)
    rm = r.astype(np.float64).mean(axis=(-2, -1), keepdims=True)
    cv = c.astype(np.float64).var(axis=(-2, -1), ddof=ddof, keepdims=True)
    rv = r.astype(np.float64).var(axis=(-2, -1), ddof=ddof, keepdims=True)
    gain = np.sqrt((rv + 1e-5) / (cv + 1e-5))
    out = (c.astype(np.float64) - cm) * gain + rm
    return (out * 2 - 1).astype(np.float32)


def _cubic_coeffs(t: np.ndarray) -> np.ndarray:
    """Keys' cubic convolution weights (A = -0.75) of the 4 taps at offsets
    -1, 0, 1, 2 for fractional positions t, fp32: [..., 4]."""
    t = t.astype(np.float32)
    one = np.float32(1)

    def conv1(x):                       # |x| <= 1
        return ((A + 2) * x - (A + 3)) * x * x + one

    def conv2(x):                       # 1 < |x| < 2
        return ((A * x - 5 * A) * x + 8 * A) * x - 4 * A

    return np.stack([conv2(t + one), conv1(t), conv1(one - t), conv2(one - t + one)], -1).astype(np.float32)


def _axis(src: int, dst: int):
    scale = np.float32(src / dst)
    real = (np.arange(dst, dtype=np.float32) + np.float32(0.5)) * scale - np.float32(0.5)
    i0 = np.floor(real).astype(np.int64)
    t = (real - i0).astype(np.float32)
    idx = np.clip(i0[:, None] + np.arange(-1, 3)[None, :], 0, src - 1)
    return idx, _cubic_coeffs(t)


def bicubic(img: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """torch.nn.functional.interpolate(img, (out_h, out_w), mode="bicubic",
    align_corners=False) of [N, C, h, w] fp32: rows first along x, then y."""
    _, _, h, w = img.shape
    yi, yc = _axis(h, out_h)
    xi, xc = _axis(w, out_w)
    x = img.astype(np.float32)
    rows = x[:, :, :, xi]                                    # [N, C, h, out_w, 4]
    horiz = (rows * xc[None, None, None]).sum(-1, dtype=np.float32)
    cols = horiz[:, :, yi]                                   # [N, C, out_h, 4, out_w]
    return (cols * yc[None, None, :, :, None]).sum(-2, dtype=np.float32)


def _blur(x: np.ndarray, r: int) -> np.ndarray:
    """3x3 [1,2,1]x[1,2,1]/16 with dilation r and replicate padding, [N, C, H, W]."""
    _, _, h, w = x.shape
    yy = np.clip(np.arange(h)[:, None] + np.array([-r, 0, r])[None, :], 0, h - 1)
    xx = np.clip(np.arange(w)[:, None] + np.array([-r, 0, r])[None, :], 0, w - 1)
    k = np.array([1, 2, 1], np.float32) / np.float32(4)
    out = np.zeros_like(x, dtype=np.float32)
    for a in range(3):
        for b in range(3):
            out += x[:, :, yy[:, a]][:, :, :, xx[:, b]] * np.float32(k[a] * k[b])
    return out.astype(np.float32)


def wavelet_color_fix(decoded: np.ndarray, input_rgb: np.ndarray) -> np.ndarray:
    """decoded [1, 3, T, H, W] in [-1, 1]; input_rgb uint8 [T, h, w, 3] ->
    uint8 [T, H, W, 3]."""
    if decoded.ndim != 5 or decoded.shape[:2] != (1, 3):
        raise ValueError("Wavelet correction expects decoded [1,3,T,H,W] frames.")
    content = np.clip((decoded[0].transpose(1, 0, 2, 3).astype(np.float32) + np.float32(1)) * np.float32(0.5), 0, 1)
    ref = input_rgb.transpose(0, 3, 1, 2).astype(np.float32) / np.float32(255.0)
    ref = np.clip(bicubic(ref, content.shape[-2], content.shape[-1]), 0, 1)
    low_c, low_r = content, ref
    high = np.zeros_like(content)
    for r in (1, 2, 4, 8, 16):
        nxt = _blur(low_c, r)
        high = (high + (low_c - nxt)).astype(np.float32)
        low_c = nxt
        low_r = _blur(low_r, r)
    fixed = np.clip(high + low_r, 0, 1).astype(np.float32)
    return np.rint(fixed * np.float32(255.0)).astype(np.uint8).transpose(0, 2, 3, 1)
