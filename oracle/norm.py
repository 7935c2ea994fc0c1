"""CPU restatement of the residual + RMSNorm / LayerNorm + e4m3 quantisation steps.

References:
  - residual RMSNorm   cute_kernels/fused_residual_rmsnorm_fp8/submission.py:139-145
                       (h = x + r; y = h * rsqrt(mean(h^2) + eps) * w)
  - Qwen RMSNorm       tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:167-171
                       (hidden * rsqrt(mean(hidden^2) + eps) * (1 + w))
  - GPT-2 LayerNorm    tasks/model_gpt2_small_transformer_block_fp8/starter.py:407-416
                       (F.layer_norm(..., eps=1e-5) then (y / NORM_SCALE).to(e4m3))
BASELINE config 3 (bf16 x and residual, gamma, eps 1e-6, per-tensor amax scale) has no
reference evaluator; its convention is defined here and by b2f_norm_quant: h is rounded
to bf16 (it is stored as the updated residual) and normalised from that value, y is
rounded to bf16, s = amax(|y|) / 448 and q = e4m3(y / s).  Parity for that output is
unpinned by any reference fixture.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def residual_norm(x: torch.Tensor, weight: torch.Tensor, *, kind="rms",
                  bias: Optional[torch.Tensor] = None, weight_offset=0.0, eps=1e-6,
                  x_scale=1.0, residual: Optional[torch.Tensor] = None,
                  h_dtype: Optional[torch.dtype] = None):
    """Returns (h, y) in f32; h rounded through h_dtype when given (the stored stream)."""
    h = x.float() * x_scale
    if residual is not None:
        h = h + residual.float()
    if h_dtype is not None:
        h = h.to(h_dtype).float()
    w = weight.float()
    if kind == "rms":
        inv = torch.rsqrt(h.double().square().mean(dim=-1, keepdim=True) + eps).float()
        y = h * inv * (w + weight_offset)
    else:
        y = F.layer_norm(h, (h.shape[-1],), w, None if bias is None else bias.float(), eps)
    return h, y


def residual_rmsnorm_amax_quant(x, residual, gamma, eps=1e-6):
    """(q e4m3, scale, h bf16)."""
    h, y = residual_norm(x, gamma, kind="rms", eps=eps, residual=residual,
                         h_dtype=torch.bfloat16)
    y = y.to(torch.bfloat16).float()
    amax = float(y.abs().max())
    s = amax / 448.0 if amax > 0 else 1.0
    q = (y / s).to(torch.float8_e4m3fn)
    return q, s, h.to(torch.bfloat16)


def layer_norm_rows(x: torch.Tensor, eps: float = 1e-5, weight: Optional[torch.Tensor] = None,
                    bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm over each whole row (tasks/level1_40_layer_norm_fp8/starter.py:134-144:
    F.layer_norm over the normalized shape [64, 256, 256], i.e. one 4,194,304-element row per
    batch item, no affine); statistics in f64.  x: values (already dequantised).  f32 out."""
    xd = x.double()
    mean = xd.mean(dim=-1, keepdim=True)
    var = (xd - mean).square().mean(dim=-1, keepdim=True)
    y = (xd - mean) * torch.rsqrt(var + eps)
    if weight is not None:
        y = y * weight.double()
    if bias is not None:
        y = y + bias.double()
    return y.float()
