"""Shared test helpers: seeded inputs and the oracle comparison bars."""
from __future__ import annotations

import math

import numpy as np
import torch

# Tolerances (stated by the task for this path): bf16 inputs with fp32
# accumulation -> relative L2 <= 5e-3 and max-abs <= 2e-2; fp32 mode -> rel L2 <= 1e-5.
BF16_REL_L2 = 5e-3
BF16_MAX_ABS = 2e-2
F32_REL_L2 = 1e-5


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    n = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (n if n > 0 else 1.0))


def lpm_params(in_dim: int, feat: int, seed: int = 0, dtype=torch.float32):
    """nn.Linear(in_dim, feat) initialised as LearnablePositiveMap does
    (kaiming-uniform a=sqrt(5), bias U(+-1/sqrt(fan_in)), feature_maps.py:224-232)
    from torch.manual_seed(seed)."""
    g = torch.Generator().manual_seed(seed)
    bound_w = math.sqrt(6.0 / ((1 + 5.0) * in_dim))  # gain(a=sqrt5)*sqrt(3/fan_in)
    W = (torch.rand(feat, in_dim, generator=g) * 2 - 1) * bound_w
    bound_b = 1.0 / math.sqrt(in_dim)
    b = (torch.rand(feat, generator=g) * 2 - 1) * bound_b
    return W.to(dtype), b.to(dtype)


def randn(shape, seed: int, scale: float = 1.0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
