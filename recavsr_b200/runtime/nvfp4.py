"""NVFP4 DiT linears on B200 (drop-in for recavsr_infer/runtime/nvfp4.py).

Same public surface: validate_support, nvfp4_mm (custom op
"recavsr_nvfp4::linear"), quantize, NVFP4Linear, quantize_block_linears.
quantize() runs rc_nvfp4_quantize and nvfp4_mm runs the tcgen05 block-scaled
GEMM rc_nvfp4_gemm instead of torch._scaled_mm_v2. Codes, scale layout and
the bf16-typed parameter views are byte-identical to the reference.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import _lib


def validate_support(device: torch.device) -> None:
    """nvfp4.py:14-19: fail before loading the model when the GPU is unsuitable."""
    _lib.library()
    if not torch.cuda.is_available():
        raise RuntimeError("NVFP4 DiT requires a CUDA device.")
    if torch.cuda.get_device_capability(device) < (10, 0):
        raise ValueError("NVFP4 DiT requires an NVIDIA Blackwell GPU or later.")


def scale_numel(m: int, k: int) -> int:
    return (m + 127) // 128 * 128 * (((k // 16) + 3) // 4 * 4)


def quantize(matrix: torch.Tensor, global_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """nvfp4.py:49-68: (packed E2M1 u8 [M, K/2], swizzled E4M3 scales u8 flat).

    global_scale = 1 is the reference formula bit for bit; another value
    selects the per-tensor global-scale mode (the GEMM then needs
    alpha = 1 / (g_a * g_b))."""
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


@torch.library.custom_op("recavsr_nvfp4::linear", mutates_args=())
def nvfp4_mm(
    values: torch.Tensor,
    weights: torch.Tensor,
    scales: torch.Tensor,
    weight_scales: torch.Tensor,
    bias: torch.Tensor | None,
) -> torch.Tensor:
    """nvfp4.py:22-39: block-scaled FP4 GEMM with bias, bf16 [M, N]."""
    return gemm(values, weights, scales, weight_scales, bias)


@nvfp4_mm.register_fake
def _nvfp4_mm_fake(values, weights, scales, weight_scales, bias):
    return torch.empty((values.shape[0], weights.shape[0]), device=values.device,
                       dtype=torch.bfloat16)


class NVFP4Linear(nn.Module):
    """nvfp4.py:71-93: weights quantized once into bf16-typed parameter views."""

    @torch.inference_mode()
    def __init__(self, linear: nn.Linear):
        super().__init__()
        if linear.weight.device.type != "cuda" or linear.weight.dtype != torch.bfloat16:
            raise ValueError("NVFP4 conversion requires loaded CUDA BF16 linears.")
        if linear.in_features % 16 or linear.out_features % 16:
            raise ValueError("NVFP4 linear dimensions must be multiples of 16.")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        weight, scales = quantize(linear.weight.detach())
        self.weight_packed = nn.Parameter(weight.view(torch.bfloat16), requires_grad=False)
        self.scales_packed = nn.Parameter(scales.view(torch.bfloat16), requires_grad=False)
        self.bias = linear.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            raise ValueError("NVFP4 linears require BF16 inputs and produce BF16 outputs.")
        matrix = x.reshape(-1, self.in_features)
        values, scales = quantize(matrix)
        out = nvfp4_mm(values, self.weight_packed, scales, self.scales_packed, self.bias)
        return out.reshape(*x.shape[:-1], self.out_features)


def quantize_block_linears(block: nn.Module) -> None:
    """nvfp4.py:96-101."""
    for module in list(block.modules()):
        for name, child in list(module.named_children()):
            if isinstance(child, nn.Linear):
                setattr(module, name, NVFP4Linear(child))
