"""DiT block oracle with NVFP4 linears (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/runtime/transformer.py:81-134 (PreparedBlock.forward)
with every nn.Linear replaced by NVFP4Linear (runtime/nvfp4.py:87-93):
quantize(x) -> dequantized fp32 matmul + bias -> bf16. Norm modules follow
models/transformer_wan.py:793-820 (FP32LayerNorm: norm1/norm3 without affine,
norm2 affine, eps 1e-6; RMSNorm across heads with affine weight, eps 1e-6,
one bf16 rounding of x*rsqrt(mean(x^2)+eps)*w) and the FFN is diffusers
FeedForward(gelu-approximate): Linear -> GELU(tanh) in fp32 -> bf16 -> Linear.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4
from .attention import plain_attention, routed_attention
from .numerics import bf16_round
from .rope import apply_rotary


def layer_norm(x, weight=None, bias=None, eps=1e-6):
    x = np.asarray(x, np.float32)
    mean = x.mean(-1, keepdims=True, dtype=np.float64)
    var = ((x - mean) ** 2).mean(-1, keepdims=True)
    y = ((x - mean) / np.sqrt(var + eps)).astype(np.float32)
    if weight is not None:
        y = y * np.asarray(weight, np.float32)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y.astype(np.float32)


def rms_norm(x, weight, eps=1e-6):
    x = np.asarray(x, np.float32)
    r = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)
    return bf16_round((x * r * np.asarray(weight, np.float64)).astype(np.float32))


def gelu_tanh(x):
    x = np.asarray(x, np.float32)
    return (0.5 * x * (1.0 + np.tanh(np.float32(0.7978845608028654) *
                                     (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


class QuantLinear:
    """NVFP4Linear with the weight quantized once (nvfp4.py:82-84).
    matmul_dtype float64 for parity checks, float32 for the timed CPU baseline.
    quantized=False: the fp32 nn.Linear of the reference's CPU formulation (its
    NVFP4 GEMM needs CUDA), i.e. x @ W^T + b in fp32 without quantization."""

    def __init__(self, weight, bias, matmul_dtype=np.float64, quantized: bool = True):
        self.n, self.k = weight.shape
        self.bias = None if bias is None else np.asarray(bias, np.float32)
        self.dtype = matmul_dtype
        self.quantized = quantized
        if quantized:
            self.codes, self.scales = nvfp4.quantize(np.asarray(weight, np.float32))
            self.w = nvfp4.dequantize(self.codes, self.scales, self.n, self.k).astype(matmul_dtype)
        else:
            self.w = np.ascontiguousarray(np.asarray(weight, np.float32).T)

    def __call__(self, x):
        x = np.asarray(x, np.float32)
        shape = x.shape
        if not self.quantized:
            out = x.reshape(-1, self.k) @ self.w
            if self.bias is not None:
                out += self.bias
            return out.reshape(*shape[:-1], self.n)
        a = x.reshape(-1, self.k)
        ac, asf = nvfp4.quantize(a)
        out = nvfp4.nvfp4_mm(ac, asf, None, None, self.bias, a.shape[0], self.n, self.k,
                             dtype=self.dtype, b_dequantized=self.w)
        return out.reshape(*shape[:-1], self.n)


def block_forward(p, hidden, past_key, past_value, slots, past_positions, query_positions,
                  height, width, window, heads=24, matmul_dtype=np.float64):
    """p: dict of float32 weights (bf16 values) -- modulation [6, dim] fp32,
    {q,k,v,o,cq,co,up,down}_{w,b}, norm_q/norm_k/cnorm_q weights, norm2_{w,b},
    cross_k/cross_v [L, heads, d], temporal_cos/sin, spatial_cos/sin [HW, d].
    hidden [N, dim] bf16 values. Returns (hidden, k_rot [N,heads,d], v [N,heads,d])."""
    lin = p["_linears"]
    shift, scale, gate, cshift, cscale, cgate = p["modulation"]
    n, dim = hidden.shape
    d = dim // heads
    h = np.asarray(hidden, np.float32)
    norm = bf16_round(layer_norm(h) * (1 + scale) + shift)
    q = lin["q"](norm)
    k = lin["k"](norm)
    v = lin["v"](norm)
    span = height * width
    scos = np.tile(p["spatial_cos"], (n // span, 1))[:, None, :]
    ssin = np.tile(p["spatial_sin"], (n // span, 1))[:, None, :]
    q = apply_rotary(rms_norm(q, p["norm_q"]).reshape(n, heads, d), scos, ssin)
    k = apply_rotary(rms_norm(k, p["norm_k"]).reshape(n, heads, d), scos, ssin)
    v = v.reshape(n, heads, d)
    out = routed_attention(q[None], k[None], v[None], past_key[None], past_value[None], slots,
                           past_positions, query_positions, p["temporal_cos"], p["temporal_sin"],
                           height, width, window[0], window[1], compute_dtype=matmul_dtype)[0]
    o = lin["o"](out.reshape(n, dim))
    h = bf16_round(h + o * gate)
    norm = bf16_round(layer_norm(h, p["norm2_w"], p["norm2_b"]))
    cq = rms_norm(lin["cq"](norm), p["cnorm_q"]).reshape(n, heads, d)
    co = plain_attention(cq, p["cross_k"], p["cross_v"], compute_dtype=matmul_dtype).reshape(n, dim)
    h = bf16_round(h + lin["co"](co))
    norm = bf16_round(layer_norm(h) * (1 + cscale) + cshift)
    up = bf16_round(gelu_tanh(lin["up"](norm)))
    h = bf16_round(h + lin["down"](up) * cgate)
    return h, k, v
