"""Helpers shared by the tests (numpy <-> torch, tolerances)."""
from __future__ import annotations

import numpy as np
import torch

from oracle.numerics import bf16_round


def dev_bf16(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bf16_round(a))).to(device).bfloat16()


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def dev_u8(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.uint8)).to(device)


def max_rel(a, b) -> float:
    """max |a - b| / max |b| (normwise relative error)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def assert_no_device_error():
    from recavsr_b200 import _lib
    torch.cuda.synchronize()
    word = _lib.read_device_error()
    assert word == 0, f"device error word 0x{word:08x}"
