"""CPU restatement of the reference's attention steps (fp32 softmax over dequantised FP8).

References:
  - GPT-2 block   tasks/model_gpt2_small_transformer_block_fp8/starter.py:428-453
      q, k, v = dequant(qkv_fp8) reshaped [T, 3, H, D]; scores = q k^T / sqrt(D);
      causal mask (triu, diagonal=1) -> -inf; softmax(dim=-1) in f32; ctx = P v;
      ctx_fp8 = (ctx / CONTEXT_SCALE).to(e4m3)
  - Qwen block    tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:354-392
      GQA via repeat_interleave(H / H_kv); scores / sqrt(D); causal; ctx * sigmoid(gate)
  - vision block  tasks/model_qwen35_4b_vision_block_fp8/starter.py:327-345 (no mask)
Sequences: T = B * S tokens; attention never crosses a sequence boundary.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, batch: int,
              causal: bool = True, gate: Optional[torch.Tensor] = None,
              sm_scale: Optional[float] = None) -> torch.Tensor:
    """q [T, Hq, D], k/v [T, Hkv, D] (f32 values) -> ctx [T, Hq, D] f32.

    ``gate`` [T, Hq, D] multiplies the context by sigmoid(gate)."""
    t, hq, d = q.shape
    hkv = k.shape[1]
    s = t // batch
    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(d)
    out = torch.empty((t, hq, d), dtype=torch.float32)
    g = hq // hkv
    mask = torch.triu(torch.ones((s, s), dtype=torch.bool), diagonal=1) if causal else None
    for b in range(batch):
        sl = slice(b * s, (b + 1) * s)
        qb = q[sl].float()
        kb = k[sl].float().repeat_interleave(g, dim=1)
        vb = v[sl].float().repeat_interleave(g, dim=1)
        scores = torch.einsum("thd,shd->hts", qb, kb) * scale
        if mask is not None:
            scores = scores.masked_fill(mask, float("-inf"))
        p = scores.softmax(dim=-1)
        out[sl] = torch.einsum("hts,shd->thd", p, vb)
    if gate is not None:
        out = out * torch.sigmoid(gate.float())
    return out


def head_rmsnorm_rope(x: torch.Tensor, weight: Optional[torch.Tensor], cos: Optional[torch.Tensor],
                      sin: Optional[torch.Tensor], rotary_dim: int, eps: float = 1e-6) -> torch.Tensor:
    """Per-head RMSNorm with Qwen's (1 + w), then rotate-half RoPE on the first
    ``rotary_dim`` dims.  x [T, H, D] f32; cos/sin [T, rotary_dim].

    References: ``_cute_harness_rms_norm`` and ``_cute_harness_apply_rope``
    (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:167-183)."""
    y = x
    if weight is not None:
        inv = torch.rsqrt(x.double().square().mean(dim=-1, keepdim=True) + eps).float()
        y = x * inv * (1.0 + weight.float())
    if cos is None:
        return y
    rot = y[..., :rotary_dim]
    half = rotary_dim // 2
    rotated = torch.cat((-rot[..., half:], rot[..., :half]), dim=-1)
    emb = rot * cos[:, None, :] + rotated * sin[:, None, :]
    return torch.cat((emb, y[..., rotary_dim:]), dim=-1)


def rope_tables(seq: int, rotary_dim: int, theta: float, batch: int = 1):
    """cos/sin [batch*seq, rotary_dim] with positions restarting per sequence (the
    reference's construction: positions * inverse_frequency, duplicated halves)."""
    pos = torch.arange(seq, dtype=torch.float32)
    idx = torch.arange(0, rotary_dim, 2, dtype=torch.float32)
    inv_freq = 1.0 / (theta ** (idx / rotary_dim))
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().repeat(batch, 1), emb.sin().repeat(batch, 1)
