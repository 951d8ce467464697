"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch


def dev() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("GPU tests need CUDA")
    return torch.device("cuda", 0)


def t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev(), dtype)


def n(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().numpy()
