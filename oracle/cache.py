"""Static KV router oracle (test infrastructure; see oracle/__init__.py).

Restates recavsr_infer/runtime/cache.py:11-19 (ACTIONS), :31-41
(retained_frames) and the slot bookkeeping of FixedKVCache (:44-133) without
tensors: it yields the slot ids / positions history() emits and the
(source plane -> slot) copies commit() performs.
"""
from __future__ import annotations

ACTIONS = {
    "none": (0, False),
    "recent_1": (1, False),
    "recent_2": (2, False),
    "recent_4": (4, False),
    "anchor": (0, True),
    "recent_2_anchor": (2, True),
    "recent_4_anchor": (4, True),
}


def retained_frames(indices, action, *, initial=5, stride=6, anchors=2):
    """cache.py:31-41: chronological union of the last `recent` ids and the last
    `anchors` ids i >= initial with (i - initial) % stride == 0."""
    recent, use_anchor = ACTIONS[action]
    keep = set(indices[-recent:]) if recent else set()
    if use_anchor:
        periodic = [i for i in indices if i >= initial and (i - initial) % stride == 0]
        keep.update(periodic[-anchors:])
    return tuple(i for i in indices if i in keep)


class RouterState:
    """cache.py:44-133 bookkeeping: frame id -> physical slot."""

    def __init__(self, action, *, initial=5, stride=6, anchors=2):
        recent, use_anchor = ACTIONS[action]
        self.action, self.initial, self.stride, self.anchors = action, initial, stride, anchors
        self.capacity = recent + (anchors if use_anchor else 0)
        self.frame_to_slot: dict[int, int] = {}
        self.next_latent_frame = 0

    def history(self, origin, train_frames=22):
        """cache.py:67-83: slots by ascending frame id padded with -1; positions id-origin padded with 0."""
        if not self.frame_to_slot:
            return (), ()
        ids = tuple(sorted(self.frame_to_slot))
        mapped = tuple(i - origin for i in ids)
        if min(mapped) < 0 or max(mapped) >= train_frames:
            raise ValueError("Selected KV exceeds the rolling RoPE training interval.")
        pad = self.capacity - len(ids)
        return (tuple(self.frame_to_slot[i] for i in ids) + (-1,) * pad, mapped + (0,) * pad)

    def commit(self, frames, start):
        """cache.py:85-134: returns [(offset_in_block, slot)] plane copies."""
        if start != self.next_latent_frame or frames <= 0:
            raise ValueError("KV commits must be consecutive, shape-matched blocks.")
        current = tuple(range(start, start + frames))
        candidates = tuple(sorted(self.frame_to_slot)) + current
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


def rope_origin(start, frames, training_frames=22):
    """rope.py:85-101: origin = max(0, start + frames - 22); query positions."""
    origin = max(0, start + frames - training_frames)
    return origin, tuple(range(start - origin, start - origin + frames))
