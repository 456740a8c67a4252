"""Numeric helpers shared by the tests."""

from __future__ import annotations

import numpy as np

def normwise(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


# Tolerances (normwise relative error against the oracle), per storage type:
# fp32 1e-5 and bf16 2e-2 as the task specifies; fp16 (10-bit mantissa)
# sits between them.
TOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 2e-2}


def to_np(t) -> np.ndarray:
    """torch tensor (any float dtype, any device) -> float32 numpy."""
    return t.detach().float().cpu().numpy()


def from_np(a: np.ndarray, dtype, device):
    """float32 numpy -> torch tensor of `dtype` (values rounded by torch, RNE)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=device, dtype=dtype)


DT = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}


def torch_dtype(name: str):
    import torch
    return getattr(torch, DT[name])
