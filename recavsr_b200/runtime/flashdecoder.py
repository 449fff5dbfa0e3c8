"""FlashDecoder local grouped-query attention on B200 (drop-in for
recavsr_infer/models/flashdecoder/flashdecoder_wan22.py:25-119,
`_validate_spatial_window` and `_local_attention`, whose CUDA path is the
Triton forward of _local_attention_triton.py:21-131).

Same keyword signature, validation and error messages; the CUDA fp16 / bf16,
head-dim-64 path the reference sends to Triton runs the tcgen05 kernel
rc_local_gqa_attention. There is no CPU path: other inputs raise.
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _lib


def validate_spatial_window(window):
    """flashdecoder_wan22.py:25-35."""
    if (window is None or len(window) != 2
            or any(isinstance(v, bool) or not isinstance(v, int) or v <= 0 or v % 2 for v in window)):
        raise ValueError("spatial_window_size requires two positive even integers.")
    return tuple(window)


def local_attention(query, key, value, *, height, width, window, group_size, temporal_window):
    """flashdecoder_wan22.py:38-119: streaming local attention; queries are the
    last complete group of KV. query [B, HQ, QF*n, 64], key / value
    [B, HK, NF*n, 64] (any strides with the head dim contiguous) ->
    [B, HQ, QF*n, 64] contiguous, in query's dtype."""
    window = validate_spatial_window(window)
    if min(height, width, group_size, temporal_window) < 1:
        raise ValueError("Local attention dimensions must be positive.")
    n = height * width
    if query.ndim != 4 or key.ndim != 4 or key.shape != value.shape:
        raise ValueError("Expected 4D Q and matching 4D K/V.")
    qf, nf = query.shape[2] // n, key.shape[2] // n
    if (query.shape[2] % n or key.shape[2] % n or qf < 1 or nf < qf or qf % group_size
            or nf % group_size or query.shape[0] != key.shape[0] or query.shape[-1] != key.shape[-1]
            or query.shape[1] % key.shape[1]):
        raise ValueError("Invalid local grid, GQA heads or temporal group alignment.")
    if query.device != key.device or query.device != value.device:
        raise ValueError("Q/K/V must share a device.")
    key, value = key.to(query.dtype), value.to(query.dtype)
    if not (query.is_cuda and query.dtype in (torch.float16, torch.bfloat16) and query.shape[-1] == 64):
        raise ValueError("The B200 local attention kernel takes CUDA fp16 / bf16 tensors with head_dim 64.")
    tensors = []
    for t in (query, key, value):
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:3]):
            t = t.contiguous()
        tensors.append(t)
    q, k, v = tensors
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    strides = (C.c_longlong * 9)(*[s for t in (q, k, v) for s in t.stride()[:3]])
    _lib.call("rc_local_gqa_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), strides, q.shape[0],
              q.shape[1], k.shape[1], qf, nf, height, width, q.shape[-1], window[0], window[1], group_size,
              temporal_window, int(q.dtype == torch.float16), out.data_ptr(), None, _lib.stream(q.device))
    return out
