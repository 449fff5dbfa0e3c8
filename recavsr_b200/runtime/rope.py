"""Rolling RoPE (drop-in for recavsr_infer/runtime/rope.py).

Tables are built once on the host exactly as the reference builds them (the
standard rotary table of diffusers' get_1d_rotary_pos_embed: theta 10000,
float64 frequencies, pair frequencies repeated, cast to float32). The per-token
rotations run on the device: apply_rotary through rc_rmsnorm_rope (norm
skipped) and apply_temporal through rc_temporal_rope.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _lib
from .constants import ROPE_WINDOW_LATENTS


def _rotary_1d(dim: int, size: int) -> tuple[torch.Tensor, torch.Tensor]:
    freqs = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float64)[: dim // 2] / dim))
    ang = torch.outer(torch.arange(size, dtype=torch.float64), freqs)
    return (ang.cos().repeat_interleave(2, dim=1).float(), ang.sin().repeat_interleave(2, dim=1).float())


def rotary_table(dim, size, *, device):
    """rope.py:11-20."""
    c, s = _rotary_1d(dim, size)
    return c.to(device), s.to(device)


def apply_rotary(x, cos, sin):
    """rope.py:23-30 for x [..., span, heads, d] with cos/sin holding span*d values
    (custom op recavsr_b200::rotary, opaque under torch.compile)."""
    return _rotary(x, cos, sin)


@torch.library.custom_op("recavsr_b200::rotary", mutates_args=())
def _rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(x, "apply_rotary")
    d, heads = x.shape[-1], x.shape[-2]
    span = cos.numel() // d
    if cos.numel() != span * d or x.dtype != torch.bfloat16 or x.numel() % (span * heads * d):
        raise ValueError("apply_rotary on B200 expects bf16 x [..., span, heads, d] and per-token tables.")
    rows = x.reshape(-1, heads * d)
    if rows.stride(-1) != 1 or rows.data_ptr() % 16:
        rows = rows.contiguous()
    out = torch.empty((rows.shape[0], heads * d), dtype=x.dtype, device=x.device)
    cc = cos.reshape(span, d).float().contiguous()
    ss = sin.reshape(span, d).float().contiguous()
    _lib.call("rc_rmsnorm_rope", 1, (C.c_void_p * 1)(rows.data_ptr()), (C.c_longlong * 1)(rows.stride(0)),
              (C.c_void_p * 1)(None), (C.c_void_p * 1)(out.data_ptr()), (C.c_longlong * 1)(heads * d),
              rows.shape[0], heads * d, d, span, cc.data_ptr(), ss.data_ptr(), 0.0,
              _lib.stream(x.device))
    return out.reshape(x.shape)


@_rotary.register_fake
def _rotary_fake(x, cos, sin):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def apply_temporal(x, positions, cos, sin, *, span):
    """rope.py:33-47: rotate the first 2*cos.shape[-1] dims of each plane by its
    position (custom op recavsr_b200::temporal, opaque under torch.compile)."""
    return _temporal(x, positions, cos, sin, span)


@torch.library.custom_op("recavsr_b200::temporal", mutates_args=())
def _temporal(x: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
              span: int) -> torch.Tensor:
    _lib.require_cuda(x, "apply_temporal")
    if x.dtype != torch.bfloat16:
        raise ValueError("apply_temporal on B200 supports bf16 inputs.")
    b, tokens, heads, d = x.shape
    planes = positions.numel()
    if tokens != planes * span:
        raise ValueError("apply_temporal: tokens must hold complete planes.")
    rows = x.reshape(b * tokens, heads * d)
    if rows.stride(-1) != 1:
        rows = rows.contiguous()
    out = torch.empty((b * tokens, heads * d), dtype=x.dtype, device=x.device)
    pos = positions.to(device=x.device, dtype=torch.int32).repeat(b).contiguous()
    _lib.call("rc_temporal_rope", rows.data_ptr(), rows.stride(0), out.data_ptr(), heads * d,
              pos.data_ptr(), cos.float().contiguous().data_ptr(), sin.float().contiguous().data_ptr(),
              b * tokens, span, heads, d, cos.shape[-1] * 2, _lib.stream(x.device))
    return out.reshape(x.shape)


@_temporal.register_fake
def _temporal_fake(x, positions, cos, sin, span):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


class RollingRoPE:
    """rope.py:50-107: bounded 22-frame temporal table + fixed spatial tables."""

    def __init__(self, head_dim, height, width, *, device, training_frames=ROPE_WINDOW_LATENTS):
        if min(head_dim, height, width, training_frames) <= 0:
            raise ValueError("RoPE dimensions must be positive.")
        self.height, self.width, self.training_frames = height, width, training_frames
        self.spatial_dim = 2 * (head_dim // 6)
        self.temporal_dim = head_dim - 2 * self.spatial_dim
        ct, st = _rotary_1d(self.temporal_dim, training_frames)
        self.temporal_cos = ct[:, ::2].contiguous().to(device)
        self.temporal_sin = st[:, ::2].contiguous().to(device)
        ch, sh = _rotary_1d(self.spatial_dim, height)
        cw, sw = _rotary_1d(self.spatial_dim, width)
        shape = (height, width, self.temporal_dim)
        self.spatial_cos = torch.cat(
            (torch.ones(shape), ch[:, None].expand(-1, width, -1), cw[None].expand(height, -1, -1)),
            -1).reshape(1, 1, height * width, 1, head_dim).to(device)
        self.spatial_sin = torch.cat(
            (torch.zeros(shape), sh[:, None].expand(-1, width, -1), sw[None].expand(height, -1, -1)),
            -1).reshape(1, 1, height * width, 1, head_dim).to(device)
        self._query_positions = {}

    def positions(self, start: int, frames: int) -> tuple[int, torch.Tensor]:
        """rope.py:85-101."""
        if start < 0 or frames < 1:
            raise ValueError("Latent start must be nonnegative and frame count positive.")
        origin = max(0, start + frames - self.training_frames)
        values = tuple(range(start - origin, start - origin + frames))
        if min(values) < 0 or max(values) >= self.training_frames:
            raise ValueError("A block is larger than the rolling interval.")
        if values not in self._query_positions:
            self._query_positions[values] = torch.tensor(
                values, device=self.temporal_cos.device, dtype=torch.int32)
        return origin, self._query_positions[values]

    def spatial(self, x):
        framed = x.reshape(x.shape[0], -1, self.height * self.width, x.shape[2], x.shape[3])
        return apply_rotary(framed, self.spatial_cos, self.spatial_sin).reshape_as(x)
