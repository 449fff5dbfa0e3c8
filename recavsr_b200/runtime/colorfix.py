"""Colour correction on B200 (drop-in for recavsr_infer/color_fix.py:58-117).

`adain_color_fix(decoded, reference)` and `wavelet_color_fix(decoded,
input_rgb)` keep the reference's signatures, validation messages and return
types (an fp32 [B, 3, T, H, W] tensor; a uint8 numpy [T, H, W, 3] array) and
run on the decoded frames' CUDA device through rc_cf_adain and
rc_cf_bicubic_u8 + five rc_cf_wavelet_level launches.
`wavelet_color_fix_device` keeps the uint8 result on the device (for a
pipeline that encodes from device memory). There is no CPU path.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib

RADII = (1, 2, 4, 8, 16)


def _dtype_code(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    if t.dtype == torch.bfloat16:
        return t.contiguous(), 1
    return t.float().contiguous(), 0


def adain_color_fix(decoded: torch.Tensor, reference: torch.Tensor) -> torch.Tensor:
    """color_fix.py:58-81: AdaIN of matching [B, 3, T, H, W] RGB tensors in
    [-1, 1]; returns fp32 [B, 3, T, H, W]."""
    if decoded.ndim != 5 or decoded.shape[1] != 3 or decoded.shape != reference.shape:
        raise ValueError("Color correction expects matching [B,3,T,H,W] tensors.")
    if decoded.device != reference.device:
        raise ValueError("Decoded frames and color reference must share a device.")
    _lib.require_cuda(decoded, "adain_color_fix")
    c, dc = _dtype_code(decoded)
    r, dr = _dtype_code(reference)
    b, ch, t, h, w = decoded.shape
    planes, hw = b * ch * t, h * w
    ws = torch.empty(_lib.library().rc_cf_adain_workspace(planes, hw), dtype=torch.uint8, device=decoded.device)
    out = torch.empty(decoded.shape, dtype=torch.float32, device=decoded.device)
    _lib.call("rc_cf_adain", c.data_ptr(), dc, r.data_ptr(), dr, planes, hw, ws.data_ptr(), ws.numel(),
              out.data_ptr(), _lib.stream(decoded.device))
    return out


def wavelet_color_fix_device(decoded: torch.Tensor, lq: torch.Tensor) -> torch.Tensor:
    """decoded [1, 3, T, H, W] in [-1, 1] (CUDA), lq uint8 [T, h, w, 3] (CUDA)
    -> uint8 [T, H, W, 3] on the device."""
    _lib.require_cuda(decoded, "wavelet_color_fix")
    _, _, t, hh, ww = decoded.shape
    d, dt = _dtype_code(decoded[0])
    lq = lq.to(device=decoded.device).contiguous()
    dev, st = decoded.device, _lib.stream(decoded.device)
    f = lambda: torch.empty((t * 3, hh, ww), dtype=torch.float32, device=dev)
    ref, ref2, low, low2, high = f(), f(), f(), f(), f()
    out = torch.empty((t, hh, ww, 3), dtype=torch.uint8, device=dev)
    _lib.call("rc_cf_bicubic_u8", lq.data_ptr(), t, lq.shape[1], lq.shape[2], hh, ww, ref.data_ptr(), st)
    for i, r in enumerate(RADII):
        first, last = i == 0, i == len(RADII) - 1
        _lib.call("rc_cf_wavelet_level", d.data_ptr(), dt, None if first else low.data_ptr(), ref.data_ptr(),
                  None if last else low2.data_ptr(), None if last else ref2.data_ptr(), high.data_ptr(),
                  out.data_ptr() if last else None, t, hh, ww, r, int(first), int(last), st)
        low, low2 = low2, low
        ref, ref2 = ref2, ref
    return out


@torch.inference_mode()
def wavelet_color_fix(decoded: torch.Tensor, input_rgb: np.ndarray) -> np.ndarray:
    """color_fix.py:84-117: decoded [1, 3, T, H, W] in [-1, 1]; input_rgb the
    matching uint8 LQ frames [T, h, w, 3] -> uint8 [T, H, W, 3] (numpy)."""
    if decoded.ndim != 5 or decoded.shape[:2] != (1, 3):
        raise ValueError("Wavelet correction expects decoded [1,3,T,H,W] frames.")
    if (not isinstance(input_rgb, np.ndarray) or input_rgb.dtype != np.uint8 or input_rgb.ndim != 4
            or input_rgb.shape[0] != decoded.shape[2] or input_rgb.shape[-1] != 3):
        raise ValueError("Wavelet reference must be matching uint8 LQ [T,h,w,3] frames.")
    lq = torch.from_numpy(np.ascontiguousarray(input_rgb))
    return wavelet_color_fix_device(decoded, lq).cpu().numpy()
