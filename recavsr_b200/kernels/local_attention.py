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

import torch

from ..runtime.ops import routed_attention  # noqa: F401  (re-exported)


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
    temporal visibility (the same kernel with a window covering the grid). Runs
    as the custom op recavsr_b200::sdpa_routed, so a torch.compile(fullgraph=True)
    caller traces through it as it traces the reference's torch formulation."""
    if window_h < height or window_w < width:
        raise ValueError("SDPA requires a window covering the full spatial grid.")
    return _sdpa_routed(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                        height, width)


@torch.library.custom_op("recavsr_b200::sdpa_routed", mutates_args=())
def _sdpa_routed(q: torch.Tensor, ck: torch.Tensor, cv: torch.Tensor, pk: torch.Tensor,
                 pv: torch.Tensor, slots: torch.Tensor, past_positions: torch.Tensor,
                 query_positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, height: int,
                 width: int) -> torch.Tensor:
    return routed_attention(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin,
                            height, width, height, width)


@_sdpa_routed.register_fake
def _sdpa_fake(q, ck, cv, pk, pv, slots, past_positions, query_positions, cos, sin, height, width):
    return torch.empty_like(q, memory_format=torch.contiguous_format)
