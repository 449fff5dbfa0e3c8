"""Cache-routed attention on B200 (drop-in for recavsr_infer/kernels/local_attention.py).

``paired_attention`` keeps the reference signature and custom-op name
("recavsr_local::paired", :172-260) and ``sdpa_attention`` keeps :286-325; both
run rc_paired_attention: a temporal-RoPE gather pre-pass plus the tcgen05
flash-attention kernel that reads the routed cache planes in place through
their slot ids (no gather/cat copies of V). Dense windows (window covering the
grid) give exactly the sdpa path's visibility; smaller windows the clamped
per-query windows of the Triton kernel.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _lib


def _check(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin, height, width,
           window_h, window_w):
    if q.device.type != "cuda" or q.dtype != torch.bfloat16:
        raise ValueError("The B200 attention kernel requires CUDA BF16 tensors.")
    if q.shape != ck.shape or q.shape != cv.shape or pk.shape != pv.shape:
        raise ValueError("Q/current KV and past KV shapes disagree.")
    span = height * width
    if height <= 0 or width <= 0 or q.shape[1] % span:
        raise ValueError("Invalid token geometry.")
    frames = q.shape[1] // span
    if q.shape[-1] != 128:
        raise ValueError("The B200 attention kernel supports head_dim 128.")
    if slots.numel() * span != pk.shape[1] or past_positions.shape != slots.shape:
        raise ValueError("Cache slot metadata mismatch.")
    if query_positions.numel() != frames or cos.shape != sin.shape:
        raise ValueError("Rolling RoPE metadata mismatch.")
    if min(window_h, window_w) <= 0:
        raise ValueError("Spatial windows must be positive.")
    if any(x.stride(-1) != 1 for x in (q, ck, cv, pk, pv) if x.numel()):
        raise ValueError("Head dimensions must be contiguous.")
    return frames


def _i32(t: torch.Tensor, device) -> torch.Tensor:
    if t.dtype == torch.int32 and t.device == device and t.is_contiguous():
        return t
    return t.to(device=device, dtype=torch.int32).contiguous()


def routed_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                     height, width, window_h, window_w, *, out=None):
    """Shared launcher: out [B, QT*H*W, heads, d] bf16 (contiguous unless `out` given)."""
    frames = _check(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                    height, width, window_h, window_w)
    b, tokens, heads, d = q.shape
    cap = slots.numel()
    dev = q.device
    if out is None:
        out = torch.empty((b, tokens, heads, d), dtype=q.dtype, device=dev)
    ws_bytes = _lib.library().rc_paired_attention_workspace(b, frames, cap, height, width, heads, d)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    strides = []
    for t in (q, ck, cv, pk, pv):
        strides += [t.stride(0), t.stride(1), t.stride(2)]
    st = (C.c_longlong * 15)(*strides)
    si = _i32(slots, dev) if cap else None
    pp = _i32(past_positions, dev) if cap else None
    qp = _i32(query_positions, dev)
    cc = cos.to(device=dev, dtype=torch.float32).contiguous()
    ss = sin.to(device=dev, dtype=torch.float32).contiguous()
    _lib.call("rc_paired_attention", q.data_ptr(), ck.data_ptr(), cv.data_ptr(),
              pk.data_ptr() if cap else None, pv.data_ptr() if cap else None, st,
              _lib.ptr(si), _lib.ptr(pp), qp.data_ptr(), cc.data_ptr(), ss.data_ptr(),
              b, frames, cap, height, width, heads, d, cos.shape[-1] * 2, window_h, window_w,
              ws.data_ptr(), ws_bytes, out.data_ptr(), out.stride(1), None, None, _lib.stream(dev))
    return out


@torch.library.custom_op("recavsr_local::paired", mutates_args=())
def paired_attention(
    q: torch.Tensor,
    ck: torch.Tensor,
    cv: torch.Tensor,
    pk: torch.Tensor,
    pv: torch.Tensor,
    slots: torch.Tensor,
    past_positions: torch.Tensor,
    query_positions: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    height: int,
    width: int,
    window_h: int,
    window_w: int,
    query_tile_h: int = 4,
    query_tile_w: int = 8,
    key_tile: int = 64,
) -> torch.Tensor:
    """local_attention.py:172-260 (tile arguments are validated like the
    reference and otherwise ignored: the tcgen05 kernel has its own tiling)."""
    frames = q.shape[1] // max(height * width, 1)
    if height > 0 and width > 0 and q.shape[1] % (height * width) == 0 and frames not in (2, 6):
        raise ValueError("The final kernel supports prefix=6 or block=2, head=32/64/128.")
    if query_tile_h * query_tile_w * 2 not in (32, 64, 128) or key_tile not in (32, 64, 128):
        raise ValueError("Unsupported kernel tile.")
    return routed_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                            height, width, window_h, window_w)


@paired_attention.register_fake
def _fake(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin, height, width,
          window_h, window_w, query_tile_h=4, query_tile_w=8, key_tile=64):
    return torch.empty_like(q, memory_format=torch.contiguous_format)


def sdpa_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                   height, width, window_h, window_w):
    """local_attention.py:286-325: full-spatial attention with the router's sparse
    temporal visibility (the same kernel with a window covering the grid)."""
    if window_h < height or window_w < width:
        raise ValueError("SDPA requires a window covering the full spatial grid.")
    return routed_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                            height, width, height, width)
