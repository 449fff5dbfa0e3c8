"""Native norm ops (drop-in for recavsr_infer/kernels/native_norm.py:7-32).

Same custom-op names and the same dtype contract: the norm is computed in
fp32 and returned in x's dtype. PreparedBlock.layer_norm passes fp32 rows
(runtime/transformer.py:91,121,130) and norm_q / norm_k bf16 rows (:99-100,122).
bf16 rows with bf16 (or no) affine parameters take the packed row kernels
(rc_ln_modulate_quant, rc_rmsnorm_rope: fp32 statistics, one bf16 rounding);
every other floating input takes rc_layer_norm (fp32 math with the fp32 affine
parameters, one rounding into x's dtype)."""
from __future__ import annotations

import torch

from .. import _lib
from ..runtime.ops import rms_norm_rope  # noqa: F401  (re-exported)
from ..runtime.ops import rows as _rows

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _fp32(t: torch.Tensor | None, device) -> torch.Tensor | None:
    return None if t is None else t.to(device=device, dtype=torch.float32).contiguous()


def _generic(x: torch.Tensor, weight, bias, eps: float, rms: bool) -> torch.Tensor:
    """rc_layer_norm: any floating x, fp32 affine, output in x's dtype."""
    if x.dtype not in _DTYPES:
        raise ValueError(f"native norms support float32 / bfloat16 / float16 inputs (got {x.dtype}).")
    m = _rows(x)
    n = m.shape[1]
    out = torch.empty((m.shape[0], n), dtype=x.dtype, device=x.device)
    w, b = _fp32(weight, x.device), _fp32(None if rms else bias, x.device)
    for t in (w, b):
        if t is not None and t.numel() != n:
            raise ValueError("Norm affine parameters must match the last dimension.")
    _lib.call("rc_layer_norm", m.data_ptr(), _DTYPES[x.dtype], m.stride(0), m.shape[0], n,
              _lib.ptr(w), _lib.ptr(b), float(eps), int(rms), out.data_ptr(), n, _lib.stream(x.device))
    return out.reshape(x.shape)


def _bf16_or_none(t: torch.Tensor | None) -> bool:
    return t is None or t.dtype == torch.bfloat16


@torch.library.custom_op("recavsr_math::layer_norm", mutates_args=())
def native_layer_norm(
    x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float
) -> torch.Tensor:
    """native_norm.py:7-17: layer_norm(x.float(), w.float(), b.float(), eps).to(x.dtype)."""
    _lib.require_cuda(x, "native_layer_norm")
    n = x.shape[-1]
    if not (x.dtype == torch.bfloat16 and _bf16_or_none(weight) and _bf16_or_none(bias)
            and n % 64 == 0 and n <= 4096):
        return _generic(x, weight, bias, eps, rms=False)
    m = _rows(x)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    w = None if weight is None else weight.contiguous()
    b = None if bias is None else bias.contiguous()
    _lib.call("rc_ln_modulate_quant", m.data_ptr(), m.stride(0), m.shape[0], m.shape[1],
              _lib.ptr(w), _lib.ptr(b), None, None, float(eps), out.data_ptr(), m.shape[1],
              None, None, 1.0, _lib.stream(x.device))
    return out


@native_layer_norm.register_fake
def _layer_fake(x, weight, bias, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("recavsr_math::rms_norm", mutates_args=())
def native_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """native_norm.py:25-28: F.rms_norm(x, (N,), weight, eps)."""
    _lib.require_cuda(x, "native_rms_norm")
    n = x.shape[-1]
    if not (x.dtype == torch.bfloat16 and _bf16_or_none(weight) and n % 8 == 0 and n <= 4096):
        return _generic(x, weight, None, eps, rms=True)
    return rms_norm_rope(x, weight, eps)


@native_rms_norm.register_fake
def _rms_fake(x, weight, eps):
    return torch.empty_like(x, memory_format=torch.contiguous_format)
