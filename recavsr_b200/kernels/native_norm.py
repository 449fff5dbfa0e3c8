"""Native norm ops (drop-in for recavsr_infer/kernels/native_norm.py:7-32).

Same custom-op names; the math runs in rc_ln_modulate_quant /
rc_rmsnorm_rope (fp32 statistics, one bf16 rounding)."""
from __future__ import annotations

import torch

from .. import _lib


def _rows(x: torch.Tensor) -> torch.Tensor:
    m = x.reshape(-1, x.shape[-1])
    if m.stride(-1) != 1 or m.data_ptr() % 16 or (m.stride(0) * x.element_size()) % 16:
        m = m.contiguous()
    return m


@torch.library.custom_op("recavsr_math::layer_norm", mutates_args=())
def native_layer_norm(
    x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float
) -> torch.Tensor:
    """native_norm.py:7-17: layer_norm(x.float(), w.float(), b.float(), eps).to(x.dtype)."""
    _lib.require_cuda(x, "native_layer_norm")
    if x.dtype != torch.bfloat16:
        raise ValueError("native_layer_norm on B200 supports bf16 inputs.")
    m = _rows(x)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    w = None if weight is None else weight.to(torch.bfloat16).contiguous()
    b = None if bias is None else bias.to(torch.bfloat16).contiguous()
    _lib.call("rc_ln_modulate_quant", m.data_ptr(), m.stride(0), m.shape[0], m.shape[1],
              _lib.ptr(w), _lib.ptr(b), None, None, float(eps), out.data_ptr(), m.shape[1],
              None, None, 1.0, _lib.stream(x.device))
    return out


@native_layer_norm.register_fake
def _layer_fake(x, weight, bias, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("recavsr_math::rms_norm", mutates_args=())
def native_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """native_norm.py:25-28: F.rms_norm(x, (N,), weight, eps) -- one bf16 rounding."""
    _lib.require_cuda(x, "native_rms_norm")
    if x.dtype != torch.bfloat16:
        raise ValueError("native_rms_norm on B200 supports bf16 inputs.")
    return rms_norm_rope(x, weight, eps)


@native_rms_norm.register_fake
def _rms_fake(x, weight, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


def rms_norm_rope(x: torch.Tensor, weight: torch.Tensor | None, eps: float,
                  cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                  head_dim: int | None = None, span: int = 1) -> torch.Tensor:
    """RMSNorm over the last dim (weight None: skip) then, with cos/sin [span, d],
    the spatial rotary of each head for token row % span."""
    m = _rows(x)
    n = m.shape[1]
    d = head_dim or n
    out = torch.empty((m.shape[0], n), dtype=torch.bfloat16, device=x.device)
    w = None if weight is None else weight.to(torch.bfloat16).contiguous()
    import ctypes as C
    xs = (C.c_void_p * 1)(m.data_ptr())
    lx = (C.c_longlong * 1)(m.stride(0))
    ws = (C.c_void_p * 1)(_lib.ptr(w))
    os_ = (C.c_void_p * 1)(out.data_ptr())
    lo = (C.c_longlong * 1)(n)
    _lib.call("rc_rmsnorm_rope", 1, xs, lx, ws, os_, lo, m.shape[0], n, d, span,
              _lib.ptr(cos), _lib.ptr(sin), float(eps), _lib.stream(x.device))
    return out.reshape(x.shape)
