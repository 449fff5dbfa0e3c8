"""Fixed-slot KV cache with the static router (drop-in for recavsr_infer/runtime/cache.py).

Routing is host bookkeeping and follows cache.py:11-138 exactly (slot ids,
positions and evictions are bit-identical); the plane copies of commit() run
as one rc_kv_commit launch for K and V together. Cache storage is allocated
zero-filled so that key rows the attention kernel stages but masks (tile
tails past a plane) are finite.
"""
from __future__ import annotations

from functools import lru_cache

import torch

from .. import _lib
from .constants import ROPE_WINDOW_LATENTS

ACTIONS = {
    "none": (0, False),
    "recent_1": (1, False),
    "recent_2": (2, False),
    "recent_4": (4, False),
    "anchor": (0, True),
    "recent_2_anchor": (2, True),
    "recent_4_anchor": (4, True),
}


@lru_cache(maxsize=256)
def _metadata(device: str, slots: tuple, positions: tuple):
    """cache.py:22-28: shared int32 slot ids (-1 = empty) and positions."""
    return (torch.tensor(slots, dtype=torch.int32, device=device),
            torch.tensor(positions, dtype=torch.int32, device=device))


def retained_frames(indices, action, *, initial=5, stride=6, anchors=2):
    """cache.py:31-41: chronological union of recent frames and periodic anchors."""
    recent, use_anchor = ACTIONS[action]
    keep = set(indices[-recent:]) if recent else set()
    if use_anchor:
        keep.update([i for i in indices if i >= initial and (i - initial) % stride == 0][-anchors:])
    return tuple(i for i in indices if i in keep)


class FixedKVCache:
    """cache.py:44-138: bounded KV storage indexed by absolute latent frame."""

    def __init__(self, action, *, initial=5, stride=6, anchors=2):
        if action not in ACTIONS or stride <= 0 or anchors <= 0:
            raise ValueError("Invalid static KV router.")
        self.action, self.initial, self.stride, self.anchors = action, initial, stride, anchors
        recent, use_anchor = ACTIONS[action]
        self.capacity = recent + (anchors if use_anchor else 0)
        self.key = self.value = None
        self.frame_to_slot: dict[int, int] = {}
        self.next_latent_frame = 0
        self.signature = None

    def route(self, origin, *, train_frames=ROPE_WINDOW_LATENTS):
        """Slot ids and positions history() exposes, as Python tuples."""
        if not self.frame_to_slot:
            return (), ()
        ids = tuple(sorted(self.frame_to_slot))
        mapped = tuple(i - origin for i in ids)
        if min(mapped) < 0 or max(mapped) >= train_frames:
            raise ValueError("Selected KV exceeds the rolling RoPE training interval.")
        pad = self.capacity - len(ids)
        return tuple(self.frame_to_slot[i] for i in ids) + (-1,) * pad, mapped + (0,) * pad

    def history(self, current, *, origin, train_frames=ROPE_WINDOW_LATENTS):
        """cache.py:67-83."""
        batch, _, heads, dim = current.shape
        if self.key is None or not self.frame_to_slot:
            empty = current.new_empty((batch, 0, heads, dim))
            slots, positions = _metadata(str(current.device), (), ())
            return empty, empty, slots, positions
        slots, positions = self.route(origin, train_frames=train_frames)
        si, pi = _metadata(str(current.device), slots, positions)
        return self.key, self.value, si, pi

    def plan_commit(self, frames, start):
        """cache.py:100-134 bookkeeping: returns [(plane offset in block, slot)]."""
        current_ids = tuple(range(start, start + frames))
        candidates = tuple(sorted(self.frame_to_slot)) + current_ids
        selected = retained_frames(candidates, self.action, initial=self.initial,
                                   stride=self.stride, anchors=self.anchors)
        self.next_latent_frame += frames
        if not self.capacity:
            return []
        self.frame_to_slot = {i: s for i, s in self.frame_to_slot.items() if i in selected}
        free = iter(sorted(set(range(self.capacity)) - set(self.frame_to_slot.values())))
        copies = []
        for i in selected:
            if i in self.frame_to_slot:
                continue
            slot = next(free)
            if i - start < 0:
                raise RuntimeError("Retention tried to resurrect an evicted KV frame.")
            copies.append((i - start, slot))
            self.frame_to_slot[i] = slot
        return copies

    def commit(self, key, value, *, frames, start):
        """cache.py:85-134: copy only newly retained planes (one device launch)."""
        if key.ndim != 4 or value.ndim != 4:
            raise ValueError("KV tensors must have shape [B,tokens,heads,head_dim].")
        if key.dtype != value.dtype or key.device != value.device:
            raise ValueError("Key and value must share dtype and device.")
        if start != self.next_latent_frame or frames <= 0 or key.shape != value.shape:
            raise ValueError("KV commits must be consecutive, shape-matched blocks.")
        if key.shape[1] % frames:
            raise ValueError("KV length must contain complete spatial planes.")
        span = key.shape[1] // frames
        signature = (key.shape[0], span, key.shape[2:], key.dtype, key.device)
        if self.signature is not None and self.signature != signature:
            raise ValueError("KV geometry changed within a video; reset the state.")
        self.signature = signature
        copies = self.plan_commit(frames, start)
        if not self.capacity:
            return
        if self.key is None:
            shape = (key.shape[0], self.capacity * span, *key.shape[2:])
            self.key = torch.zeros(shape, dtype=key.dtype, device=key.device)
            self.value = torch.zeros(shape, dtype=value.dtype, device=value.device)
        if copies:
            commit_planes(key, value, self.key, self.value, span, copies)

    @property
    def frame_indices(self):
        return tuple(sorted(self.frame_to_slot))


def commit_planes(key, value, cache_k, cache_v, span, copies):
    """Copy block planes into cache slots: copies = [(plane offset, slot)]."""
    import ctypes as C
    _lib.require_cuda(key, "FixedKVCache.commit")
    batch = key.shape[0]
    row = key.shape[2] * key.shape[3] * key.element_size()
    for t in (key, value, cache_k, cache_v):
        if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1] or t.stride(1) * t.element_size() != row:
            raise ValueError("KV tensors must have contiguous [heads, head_dim] rows.")
    n = len(copies)
    if n > 8:
        raise ValueError("At most 8 planes per commit.")
    src = (C.c_int * n)(*[c[0] for c in copies])
    dst = (C.c_int * n)(*[c[1] for c in copies])
    rows_src = key.shape[1]
    rows_dst = cache_k.shape[1]
    for b in range(batch):
        _lib.call("rc_kv_commit",
                  key.data_ptr() + b * key.stride(0) * key.element_size(),
                  value.data_ptr() + b * value.stride(0) * value.element_size(),
                  row,
                  cache_k.data_ptr() + b * cache_k.stride(0) * cache_k.element_size(),
                  cache_v.data_ptr() + b * cache_v.stride(0) * cache_v.element_size(),
                  row, row, span, n, src, dst, _lib.stream(key.device))
    del rows_src, rows_dst
