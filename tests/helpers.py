"""Test helpers: torch <-> numpy bit views and error measures."""
from __future__ import annotations

import numpy as np
import torch


def to_dev(a: np.ndarray, dev, dtype=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def bits(t: torch.Tensor) -> np.ndarray:
    """uint16 bit patterns of a 16-bit tensor."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max |y - ref| / max |ref| (the reference's measure, tests/gpu_dense.py:210-223)."""
    return float(np.abs(y.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


def floor_err(ref: np.ndarray, dtype: torch.dtype) -> float:
    """rounding floor of storing ref in dtype, on the same measure."""
    r = torch.from_numpy(np.ascontiguousarray(ref, dtype=np.float32)).to(dtype).float().numpy()
    return rel_err(r, ref)
