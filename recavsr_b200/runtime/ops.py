"""Launchers of the library's kernels that the runtime and the drop-in
modules share. Nothing here registers an operator under the reference's
namespaces (recavsr_local, recavsr_math, recavsr_nvfp4): the drop-in modules
(kernels.local_attention, kernels.native_norm, runtime.nvfp4) do that, so
this module can be imported in the same process as the reference itself."""
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


def rows(x: torch.Tensor) -> torch.Tensor:
    m = x.reshape(-1, x.shape[-1])
    if m.stride(-1) != 1 or m.data_ptr() % 16 or (m.stride(0) * x.element_size()) % 16:
        m = m.contiguous()
    return m


def rms_norm_rope(x: torch.Tensor, weight: torch.Tensor | None, eps: float,
                  cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                  head_dim: int | None = None, span: int = 1) -> torch.Tensor:
    """RMSNorm over the last dim (weight None: skip) then, with cos/sin [span, d],
    the spatial rotary of each head for token row % span."""
    m = rows(x)
    n = m.shape[1]
    d = head_dim or n
    out = torch.empty((m.shape[0], n), dtype=torch.bfloat16, device=x.device)
    w = None if weight is None else weight.to(torch.bfloat16).contiguous()
    xs = (C.c_void_p * 1)(m.data_ptr())
    lx = (C.c_longlong * 1)(m.stride(0))
    ws = (C.c_void_p * 1)(_lib.ptr(w))
    os_ = (C.c_void_p * 1)(out.data_ptr())
    lo = (C.c_longlong * 1)(n)
    _lib.call("rc_rmsnorm_rope", 1, xs, lx, ws, os_, lo, m.shape[0], n, d, span,
              _lib.ptr(cos), _lib.ptr(sin), float(eps), _lib.stream(x.device))
    return out.reshape(x.shape)


def scale_numel(m: int, k: int) -> int:
    return (m + 127) // 128 * 128 * (((k // 16) + 3) // 4 * 4)


def quantize(matrix: torch.Tensor, global_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """nvfp4.py:49-68: (packed E2M1 u8 [M, K/2], swizzled E4M3 scales u8 flat).

    global_scale = 1 is the reference formula bit for bit; another value
    selects the per-tensor global-scale mode (the GEMM then needs
    alpha = 1 / (g_a * g_b)). Runs as the custom op recavsr_b200::nvfp4_quantize,
    so a torch.compile(fullgraph=True) caller traces through it."""
    return _quantize(matrix, float(global_scale))


@torch.library.custom_op("recavsr_b200::nvfp4_quantize", mutates_args=())
def _quantize(matrix: torch.Tensor, global_scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    _lib.require_cuda(matrix, "nvfp4.quantize")
    if matrix.dim() != 2 or matrix.dtype != torch.bfloat16:
        raise ValueError("nvfp4.quantize expects a 2-D bf16 matrix.")
    m, k = matrix.shape
    if k % 16:
        raise ValueError("NVFP4 rows must be a multiple of 16 elements.")
    if matrix.stride(1) != 1 or (matrix.stride(0) * 2) % 16 or matrix.data_ptr() % 16:
        matrix = matrix.contiguous()
    packed = torch.empty((m, k // 2), dtype=torch.uint8, device=matrix.device)
    scales = torch.empty((scale_numel(m, k),), dtype=torch.uint8, device=matrix.device)
    _lib.call("rc_nvfp4_quantize", matrix.data_ptr(), m, k, matrix.stride(0), float(global_scale),
              packed.data_ptr(), scales.data_ptr(), _lib.stream(matrix.device))
    return packed, scales


@_quantize.register_fake
def _quantize_fake(matrix, global_scale):
    m, k = matrix.shape
    return (matrix.new_empty((m, k // 2), dtype=torch.uint8),
            matrix.new_empty((scale_numel(m, k),), dtype=torch.uint8))


_SPLIT_WS: dict = {}


def split_workspace(device: torch.device) -> torch.Tensor:
    """The zero-filled split-K workspace of the NVFP4 GEMM, one per (device,
    stream): calls sharing a workspace must be ordered on one stream."""
    device = torch.device(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), _lib.stream(device))
    ws = _SPLIT_WS.get(key)
    if ws is None:
        ws = torch.zeros((_lib.library().rc_gemm_split_workspace(),), dtype=torch.uint8, device=device)
        _SPLIT_WS[key] = ws
    return ws


def gemm(values, weights, scales, weight_scales, bias=None, *, alpha=1.0,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [M, N] = alpha * A . B^T + bias on the tcgen05 block-scaled path."""
    a = values.view(torch.uint8)
    b = weights.view(torch.uint8)
    m, n, k = a.shape[0], b.shape[0], a.shape[1] * 2
    if b.shape[1] * 2 != k:
        raise ValueError("NVFP4 operand widths disagree.")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    ws = split_workspace(a.device)
    _lib.call("rc_nvfp4_gemm_ws", a.data_ptr(), scales.view(torch.uint8).data_ptr(), b.data_ptr(),
              weight_scales.view(torch.uint8).data_ptr(), _lib.ptr(bias), m, n, k, float(alpha),
              _lib.EPI_BIAS, out.data_ptr(), out.stride(0), None, None, None, 1.0,
              ws.data_ptr(), ws.numel(), _lib.stream(a.device))
    return out


