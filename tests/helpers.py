"""Seeded input generation shared by the tests (CPU generator, then copied to the GPU,
so the oracle and the kernels see identical bytes)."""
from __future__ import annotations

import torch

from oracle import fp8 as ofp8


def gen(seed: int) -> torch.Generator:
    return torch.Generator("cpu").manual_seed(seed)


def randn(shape, g, scale=1.0, mean=0.0):
    return torch.randn(shape, generator=g, dtype=torch.float32) * scale + mean


def fp8_amax(shape, g, scale=1.0):
    """N(0, scale^2) quantised with its per-tensor amax scale -> (e4m3 cpu tensor, scale)."""
    return ofp8.quantize_amax(randn(shape, g, scale))


def e4m3_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|index distance| between two e4m3 tensors along the monotone code ordering."""
    def key(t):
        u = t.view(torch.uint8).to(torch.int32)
        mag = u & 0x7F
        return torch.where(u & 0x80 != 0, -mag, mag)
    return (key(a) - key(b)).abs()
