"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Inputs are drawn on the CPU from ``torch.Generator().manual_seed(seed)`` so the
fixture generator, the CPU tests and the GPU tests all see identical data; the
fixtures record a sha256 of every generated input so a change in the RNG
stream is caught instead of silently comparing different data.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

D_HEAD = 128
OUTLIER_CHANNELS = 4
OUTLIER_FACTOR = 8.0


def randn(shape, seed: int, dtype=torch.float32) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float32).to(dtype)


def outlier_channels(seed: int, d: int = D_HEAD, n: int = OUTLIER_CHANNELS) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 7919)
    return torch.randperm(d, generator=g)[:n].sort().values


def kivi_k(shape, seed: int, dtype=torch.float32) -> torch.Tensor:
    """K ~ N(0,1) with OUTLIER_CHANNELS of the head dim scaled by OUTLIER_FACTOR."""
    x = randn(shape, seed)
    x[..., outlier_channels(seed, shape[-1])] *= OUTLIER_FACTOR
    return x.to(dtype)


def degenerate_groups(shape, seed: int, axis: int) -> torch.Tensor:
    """Inputs whose quantization groups hit the edge cases of the reference
    arithmetic: constant groups (scale 0 -> 1), tiny ranges (zero point
    overflows float16 to inf), exact ties and sign mixtures.  ``axis`` is the
    grouped axis (2 for K, 3 for V); groups are 32 long."""
    x = randn(shape, seed)
    n = shape[axis] // 32
    for gi in range(n):
        idx = [slice(None)] * 4
        idx[axis] = slice(gi * 32, gi * 32 + 32)
        sl = tuple(idx)
        kind = gi % 4
        if kind == 0:    # constant group
            x[sl] = x[sl].mean()
        elif kind == 1:  # tiny range around a large offset
            x[sl] = 3.0 + 1e-6 * x[sl]
        elif kind == 2:  # values on the 2-bit grid (ties at .5 after scaling)
            x[sl] = torch.round(x[sl] * 1.5) / 1.5
    return x


def sha(t) -> str:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous().numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()
