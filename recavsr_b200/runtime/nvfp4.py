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
from .ops import gemm, quantize, scale_numel, split_workspace  # noqa: F401  (re-exported)


def validate_support(device: torch.device) -> None:
    """nvfp4.py:14-19: fail before loading the model when the GPU is unsuitable."""
    _lib.library()
    if not torch.cuda.is_available():
        raise RuntimeError("NVFP4 DiT requires a CUDA device.")
    if torch.cuda.get_device_capability(device) < (10, 0):
        raise ValueError("NVFP4 DiT requires an NVIDIA Blackwell GPU or later.")


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
