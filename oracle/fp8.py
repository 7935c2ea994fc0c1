"""FP8 (e4m3) quantisation convention of the reference, restated on CPU.

Reference: tasks/model_gpt2_small_transformer_block_fp8/TASK_REFERENCE.md:14-30 and
``_cute_harness_fp8_tensor`` (tasks/model_gpt2_small_transformer_block_fp8/starter.py:176-188):
a tensor ``x`` with scale ``s`` is stored as ``(x / s).to(float8_e4m3fn)`` (round to nearest
even) and read back as ``stored.float() * s``.
"""
from __future__ import annotations

import torch

FP8_MAX = 448.0


def quantize(x: torch.Tensor, scale: float) -> torch.Tensor:
    """e4m3 bytes of x / scale (torch's RNE cast, as the reference evaluators do)."""
    return (x.float() / scale).to(torch.float8_e4m3fn)


def dequantize(q: torch.Tensor, scale: float) -> torch.Tensor:
    return q.float() * scale


def amax_scale(x: torch.Tensor) -> float:
    """Per-tensor scale amax(|x|) / 448 used for BASELINE's synthetic inputs."""
    a = float(x.abs().max())
    return a / FP8_MAX if a > 0 else 1.0


def quantize_amax(x: torch.Tensor):
    """(e4m3 tensor, scale) with the per-tensor amax scale."""
    s = amax_scale(x)
    return quantize(x, s), s


def quantize_amax_f32(x: torch.Tensor):
    """(e4m3 tensor, f32 scale) with s = amax(|x|) / 448 computed in f32 and q = e4m3(x / s)
    by f32 division: the device quantiser's convention (b2f_quantize_fp8), equal to the torch
    expression ``s = x.abs().max() / 448.0; (x / s).to(float8_e4m3fn)`` on an f32 tensor."""
    xf = x.float()
    s = xf.abs().max() / FP8_MAX
    if float(s) == 0.0:
        s = torch.ones((), dtype=torch.float32)
    return (xf / s).to(torch.float8_e4m3fn), float(s)
