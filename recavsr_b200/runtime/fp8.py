"""FP8 (E4M3, per-tensor) DiT linears on B200 (drop-in for recavsr_infer/runtime/fp8.py).

Weights and activations use scale = max(amax, 1e-12)/448 computed on the
device (rc_fp8_quantize) and the tcgen05 kind::f8f6f4 GEMM rc_fp8_gemm with
fp32 accumulation (the reference's use_fast_accum=False path).
"""
from __future__ import annotations

import torch
from torch import nn

from .. import _lib

FP8_MAX = 448.0


def quantize(matrix: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp8.py:41-42 on the device: (e4m3 bytes [M, K] as uint8, fp32 scale [] tensor);
    the custom op recavsr_b200::fp8_quantize (opaque under torch.compile)."""
    return _quantize(matrix)


@torch.library.custom_op("recavsr_b200::fp8_quantize", mutates_args=())
def _quantize(matrix: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _lib.require_cuda(matrix, "fp8.quantize")
    if matrix.dim() != 2 or matrix.dtype != torch.bfloat16:
        raise ValueError("fp8.quantize expects a 2-D bf16 matrix.")
    if matrix.stride(1) != 1 or (matrix.stride(0) * 2) % 16 or matrix.data_ptr() % 16:
        matrix = matrix.contiguous()
    m, k = matrix.shape
    q = torch.empty((m, k), dtype=torch.uint8, device=matrix.device)
    scratch = torch.empty((2,), dtype=torch.int32, device=matrix.device)
    scale = torch.empty((), dtype=torch.float32, device=matrix.device)
    _lib.call("rc_fp8_quantize", matrix.data_ptr(), m, k, matrix.stride(0), scratch.data_ptr(),
              scale.data_ptr(), q.data_ptr(), _lib.stream(matrix.device))
    return q, scale


@_quantize.register_fake
def _quantize_fake(matrix):
    return (matrix.new_empty(matrix.shape, dtype=torch.uint8),
            matrix.new_empty((), dtype=torch.float32))


@torch.library.custom_op("recavsr_b200::fp8_mm", mutates_args=())
def fp8_mm(q: torch.Tensor, scale: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
           bias: torch.Tensor | None) -> torch.Tensor:
    """The torch._scaled_mm call of fp8.py:44-47 (e4m3 A [M, K] . B [N, K]^T,
    per-tensor device scales, bias, bf16 out) on the tcgen05 kind::f8f6f4 GEMM."""
    m, k = q.shape
    n = weight.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=q.device)
    _lib.call("rc_fp8_gemm", q.data_ptr(), scale.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(),
              _lib.ptr(bias), m, n, k, 1.0, _lib.EPI_BIAS, out.data_ptr(), out.stride(0), None,
              _lib.stream(q.device))
    return out


@fp8_mm.register_fake
def _fp8_mm_fake(q, scale, weight, weight_scale, bias):
    return q.new_empty((q.shape[0], weight.shape[0]), dtype=torch.bfloat16)


class FP8Linear(nn.Module):
    """fp8.py:16-47."""

    @torch.inference_mode()
    def __init__(self, linear: nn.Linear):
        super().__init__()
        if linear.weight.device.type != "cuda" or linear.weight.dtype != torch.bfloat16:
            raise ValueError("FP8 conversion requires loaded CUDA BF16 linears.")
        if linear.in_features % 16 or linear.out_features % 16:
            raise ValueError("FP8 linear dimensions must be multiples of 16.")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        quantized, scale = quantize(linear.weight.detach())
        self.weight_packed = nn.Parameter(quantized.view(torch.bfloat16), requires_grad=False)
        self.bias = linear.bias
        self.register_buffer("weight_scale", scale)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            raise ValueError("FP8 linears on B200 take BF16 inputs and produce BF16 outputs.")
        matrix = x.reshape(-1, self.in_features)
        q, scale = quantize(matrix)
        out = fp8_mm(q, scale, self.weight_packed.view(torch.uint8), self.weight_scale, self.bias)
        return out.reshape(*x.shape[:-1], self.out_features)


def quantize_block_linears(block: nn.Module) -> None:
    """fp8.py:51-55."""
    for module in list(block.modules()):
        for name, child in list(module.named_children()):
            if isinstance(child, nn.Linear):
                setattr(module, name, FP8Linear(child))
