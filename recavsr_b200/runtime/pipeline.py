"""Frame preparation and strip blending on the device (drop-in for
recavsr_infer/video.py:119-179 and recavsr_infer/strips.py:24-99).

The reference enlarges every LQ block on the CPU (cv2.resize, video.py:158)
and uploads the enlarged uint8 frames; here the host uploads the LQ frames as
decoded (1/16 of the bytes at x4) and one kernel, rc_enlarge_block, does the
bilinear enlarge with cv2's 8-bit arithmetic, the block padding, the
normalization and the pad to the token stride. Strip blending (the reference's
CPU canvas loop) runs per frame in rc_strip_blend. The column / weight
bookkeeping stays on the host and follows the reference step for step, since
the same columns and ramps must reach the kernels.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from .. import _lib
from .constants import BODY_RGB_FRAMES, PREFIX_RGB_FRAMES, SPATIAL_TOKEN_STRIDE


def scaled_size(height: int, width: int, scale: float = 4.0) -> tuple[int, int]:
    """frames.py:29-40: each scaled dimension rounded half up."""
    if isinstance(scale, bool):
        raise ValueError("Scale must be a finite positive number.")
    scale = float(scale)
    if not math.isfinite(scale) or scale <= 0:
        raise ValueError("Scale must be a finite positive number.")
    if height < 1 or width < 1:
        raise ValueError("Input dimensions must be positive.")
    dims = (height * scale, width * scale)
    if any(not math.isfinite(x) or x > 2 ** 31 - 1 for x in dims):
        raise ValueError("Scaled dimensions exceed the supported integer range.")
    out = tuple(math.floor(x + 0.5) for x in dims)
    if min(out) < 1:
        raise ValueError("Scale produces an empty output dimension.")
    return out


def block_schedule(total: int):
    """video.py:119-130: (start, valid RGB frames, padded RGB frames) per block."""
    if total < 1:
        raise ValueError("A video must contain at least one frame.")
    start = 0
    while start < total:
        block = PREFIX_RGB_FRAMES if start == 0 else BODY_RGB_FRAMES
        valid = min(block, total - start)
        yield start, valid, block
        start += valid


def padded_size(height: int, width: int) -> tuple[int, int]:
    s = SPATIAL_TOKEN_STRIDE
    return -(-height // s) * s, -(-width // s) * s


ENLARGE_BF16, ENLARGE_RECIPROCAL = 1, 2


def enlarge_block(chunk: torch.Tensor, size, *, block: int, dtype=torch.float32,
                  out: torch.Tensor | None = None, normalize: str = "cuda") -> torch.Tensor:
    """enlarge_block + block_tensor (video.py:153-179) of uint8 frames
    [valid, h, w, 3] already on the device: [1, 3, block, Hp, Wp] in `dtype`
    (fp32 as the reference's block_tensor returns; bf16 is what the session
    consumes). normalize="cuda" reproduces block_tensor on a CUDA device (torch
    multiplies by the fp32 reciprocal of 127.5 there), "cpu" on the CPU (a
    true division); the two differ by one fp32 ulp on some byte values."""
    if normalize not in ("cuda", "cpu"):
        raise ValueError("normalize must be 'cuda' or 'cpu'.")
    if chunk.device.type != "cuda" or chunk.dtype != torch.uint8 or chunk.dim() != 4 or chunk.shape[-1] != 3:
        raise ValueError("enlarge_block expects CUDA uint8 frames [valid, h, w, 3].")
    valid, h, w, _ = chunk.shape
    if valid < 1 or valid > block:
        raise ValueError("Invalid temporal block.")
    if chunk.stride(2) != 3 or chunk.stride(3) != 1:
        chunk = chunk.contiguous()
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("enlarge_block writes float32 or bfloat16.")
    srh, srw = size
    hp, wp = padded_size(srh, srw)
    shape = (1, 3, block, hp, wp)
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=chunk.device)
    elif tuple(out.shape) != shape or out.dtype != dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of the padded block shape.")
    flags = (ENLARGE_BF16 if dtype == torch.bfloat16 else 0) | (ENLARGE_RECIPROCAL if normalize == "cuda" else 0)
    _lib.call("rc_enlarge_block", chunk.data_ptr(), chunk.stride(0), chunk.stride(1), valid, block, h, w,
              srh, srw, flags, out.data_ptr(), _lib.stream(chunk.device))
    return out


def prepare_block(frames, start, valid, block, *, device, scale=4.0, size=None, dtype=torch.float32,
                  normalize="cuda"):
    """video.py:138-150: upsample one LQ block to the model raster on the
    device. `frames` is the uint8 [N, h, w, 3] video (numpy, a CPU tensor,
    ideally pinned, or a CUDA tensor); only frames [start, start + valid) are
    uploaded."""
    if start < 0 or valid < 1 or valid > block or start + valid > len(frames):
        raise ValueError("Invalid temporal block.")
    chunk = frames[start:start + valid]
    if isinstance(chunk, np.ndarray):
        chunk = torch.from_numpy(np.ascontiguousarray(chunk))
    chunk = chunk.to(device=device, non_blocking=True)
    height, width = chunk.shape[1:3]
    size = size or scaled_size(height, width, scale)
    return enlarge_block(chunk, size, block=block, dtype=dtype, normalize=normalize)


def strip_columns(width: int, strips: int, overlap: int, scale: float):
    """strips.py:24-46: equal-width LQ column ranges [x0, x1) covering 0..width."""
    if strips < 2:
        return [(0, width)]
    step = 1
    if float(scale).is_integer():
        step = SPATIAL_TOKEN_STRIDE // math.gcd(SPATIAL_TOKEN_STRIDE, int(scale))
    base = math.ceil((width + (strips - 1) * overlap) / strips)
    strip = min(width, -(-base // step) * step)
    starts = [round(i * (width - strip) / (strips - 1)) for i in range(strips)]
    columns = [(x, x + strip) for x in starts]
    for (_, a1), (b0, _) in zip(columns, columns[1:]):
        if a1 - b0 < 1:
            raise ValueError("Strips do not overlap; increase --strip-overlap.")
    return columns


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


class StripBlender:
    """blend_strips (strips.py:72-99) one frame at a time on the device: the
    feather ramps and their per-column total (summed in strip order, :82-84)
    are uploaded once; blend() combines one uint8 frame per strip."""

    MAX_STRIPS = 16

    def __init__(self, columns, scale: float, height: int, width: int, *, device):
        self.weights = column_weights(columns, scale, width)
        if len(self.weights) > self.MAX_STRIPS:
            raise ValueError(f"At most {self.MAX_STRIPS} strips.")
        total = np.zeros(width, dtype=np.float32)
        for o0, w in self.weights:
            total[o0:o0 + len(w)] += w
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.height, self.width, self.device = height, width, device
        self.total = torch.from_numpy(total).to(self.device)
        self.ramps = [torch.from_numpy(w).to(self.device) for _, w in self.weights]

    def blend(self, frames, out: torch.Tensor | None = None) -> torch.Tensor:
        """frames: one CUDA uint8 [height, width_s, 3] frame per strip, left to
        right -> uint8 [height, width, 3]."""
        n = len(self.weights)
        if len(frames) != n:
            raise RuntimeError("Strip videos have different frame counts.")
        for f, (o0, w) in zip(frames, self.weights):
            if f.device != self.device or f.dtype != torch.uint8 or tuple(f.shape) != (self.height, len(w), 3):
                raise RuntimeError(f"Unexpected strip frame size {tuple(f.shape[:2])}.")
            if f.stride(1) != 3 or f.stride(2) != 1:
                raise ValueError("Strip frames need contiguous RGB pixels.")
        if out is None:
            out = torch.empty((self.height, self.width, 3), dtype=torch.uint8, device=self.device)
        ptrs = (C.c_void_p * n)(*[f.data_ptr() for f in frames])
        strides = (C.c_longlong * n)(*[f.stride(0) for f in frames])
        offs = (C.c_int * n)(*[o0 for o0, _ in self.weights])
        widths = (C.c_int * n)(*[len(w) for _, w in self.weights])
        wptr = (C.c_void_p * n)(*[r.data_ptr() for r in self.ramps])
        _lib.call("rc_strip_blend", n, ptrs, strides, offs, widths, wptr, self.total.data_ptr(), self.height,
                  self.width, out.data_ptr(), out.stride(0), _lib.stream(self.device))
        return out
