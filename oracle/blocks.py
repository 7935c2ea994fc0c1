"""CPU restatement of the reference decoder blocks (quantised paths).

GPT-2 block — tasks/model_gpt2_small_transformer_block_fp8/starter.py:393-488:
  x = dequant(hidden); n1 = LN(x) -> e4m3 @ NORM; qkv = scaled_linear(+bias) -> e4m3 @ QKV;
  causal attention over dequant(qkv) -> ctx e4m3 @ CONTEXT; r1 = x + out_proj(ctx) + b;
  n2 = LN(r1) -> e4m3 @ NORM; fc(+b) -> gelu_tanh -> e4m3 @ MLP; out = r1 + proj(mlp) + b.
Qwen full-attention block — tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-416:
  n1 = RMSNorm(1+w)(x) -> e4m3; q/gate, k, v linears -> e4m3 @ QKV; q, k per-head
  RMSNorm(1+w) -> RoPE -> e4m3; causal GQA attention * sigmoid(gate) -> e4m3 @ CONTEXT;
  r1 = x + o_proj(ctx); optional SwiGLU MLP: n2 = RMSNorm(1+w)(r1) -> e4m3; gate/up
  -> e4m3 @ MLP_PROJECTION; silu(gate) * up -> e4m3 @ MLP_ACTIVATION; out = r1 + down(act).

Generalisations used by BASELINE's configs (documented beside each parameter):
  - ``batch``: T = batch * seq tokens; attention and RoPE positions restart per sequence.
  - ``residual_dtype``: the reference keeps the residual stream in f32; BASELINE keeps it in
    bf16, in which case r1 (and the output) are rounded to bf16 where the kernels store them.
  - Qwen: ``q_gate`` interleaved [T, H, 2, D] (reference) or separate q and gate weights;
    ``rotary_dim`` partial (reference: 64 of 256) or full; MLP optional.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.nn.functional as F

from . import attention as oatt
from .gemm import scaled_mm


def _q(x: torch.Tensor, scale: float) -> torch.Tensor:
    return (x / scale).to(torch.float8_e4m3fn)


def _dq(q: torch.Tensor, scale: float) -> torch.Tensor:
    return q.float() * scale


def _round(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return x if dtype == torch.float32 else x.to(dtype).float()


@dataclass
class GPT2Weights:
    """e4m3 weights (stored bytes) with per-tensor scales; f32 biases / LN params."""
    qkv_w: torch.Tensor
    qkv_s: float
    qkv_b: torch.Tensor
    out_w: torch.Tensor
    out_s: float
    out_b: torch.Tensor
    fc_w: torch.Tensor
    fc_s: float
    fc_b: torch.Tensor
    proj_w: torch.Tensor
    proj_s: float
    proj_b: torch.Tensor
    ln1_w: torch.Tensor
    ln1_b: torch.Tensor
    ln2_w: torch.Tensor
    ln2_b: torch.Tensor
    heads: int = 12
    eps: float = 1e-5
    norm_scale: float = 1 / 64.0
    qkv_scale: float = 1 / 64.0
    ctx_scale: float = 1 / 64.0
    mlp_scale: float = 1 / 64.0


def gpt2_block(x: torch.Tensor, w: GPT2Weights, *, batch: int,
               residual_dtype: torch.dtype = torch.float32,
               out_dtype: torch.dtype = torch.float32, causal: bool = True,
               rope_cos: Optional[torch.Tensor] = None,
               rope_sin: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x: f32 values of the hidden input [T, d] (already dequantised).  Returns f32.

    With ``rope_cos/rope_sin`` [T, head_dim] and ``causal=False`` this is the Qwen vision
    block (tasks/model_qwen35_4b_vision_block_fp8/starter.py:303-369): rotate-half RoPE on
    q and k after the QKV requantisation, q/k requantised again, non-causal attention."""
    t, d = x.shape
    hd = d // w.heads
    n1 = F.layer_norm(x, (d,), w.ln1_w.float(), w.ln1_b.float(), w.eps)
    n1_q = _q(n1, w.norm_scale)
    qkv = scaled_mm(n1_q, w.qkv_w, w.norm_scale, w.qkv_s) + w.qkv_b.float()
    qkv_d = _dq(_q(qkv, w.qkv_scale), w.qkv_scale).view(t, 3, w.heads, hd)
    q, k, v = qkv_d[:, 0], qkv_d[:, 1], qkv_d[:, 2]
    if rope_cos is not None:
        q = _dq(_q(oatt.head_rmsnorm_rope(q, None, rope_cos, rope_sin, hd), w.qkv_scale),
                w.qkv_scale)
        k = _dq(_q(oatt.head_rmsnorm_rope(k, None, rope_cos, rope_sin, hd), w.qkv_scale),
                w.qkv_scale)
    ctx = oatt.attention(q, k, v, batch=batch, causal=causal)
    ctx_q = _q(ctx.reshape(t, d), w.ctx_scale)
    r1 = _round(x + scaled_mm(ctx_q, w.out_w, w.ctx_scale, w.out_s) + w.out_b.float(),
                residual_dtype)
    n2 = F.layer_norm(r1, (d,), w.ln2_w.float(), w.ln2_b.float(), w.eps)
    n2_q = _q(n2, w.norm_scale)
    fc = scaled_mm(n2_q, w.fc_w, w.norm_scale, w.fc_s) + w.fc_b.float()
    mlp_q = _q(F.gelu(fc, approximate="tanh"), w.mlp_scale)
    out = r1 + scaled_mm(mlp_q, w.proj_w, w.mlp_scale, w.proj_s) + w.proj_b.float()
    return _round(out, out_dtype)


@dataclass
class QwenWeights:
    """Qwen-style gated full-attention block.  ``q_w`` holds the query rows; with
    ``interleaved`` it holds the reference's q_gate weight [H*2*D, hidden] ordered
    (head, {q, gate}, d) and ``gate_w`` is None."""
    q_w: torch.Tensor
    q_s: float
    gate_w: Optional[torch.Tensor]
    gate_s: float
    k_w: torch.Tensor
    k_s: float
    v_w: torch.Tensor
    v_s: float
    o_w: torch.Tensor
    o_s: float
    in_norm_w: torch.Tensor
    q_norm_w: torch.Tensor
    k_norm_w: torch.Tensor
    cos: torch.Tensor  # [seq, rotary_dim]
    sin: torch.Tensor
    heads: int
    kv_heads: int
    head_dim: int
    rotary_dim: int
    interleaved: bool = False
    # optional SwiGLU MLP
    post_norm_w: Optional[torch.Tensor] = None
    mlp_gate_w: Optional[torch.Tensor] = None
    mlp_gate_s: float = 1.0
    mlp_up_w: Optional[torch.Tensor] = None
    mlp_up_s: float = 1.0
    mlp_down_w: Optional[torch.Tensor] = None
    mlp_down_s: float = 1.0
    eps: float = 1e-6
    norm_scale: float = 1 / 64.0
    qkv_scale: float = 1 / 64.0
    ctx_scale: float = 1 / 64.0
    mlp_proj_scale: float = 1 / 64.0
    mlp_act_scale: float = 1 / 32.0


def _rms(x, w, eps):
    inv = torch.rsqrt(x.double().square().mean(dim=-1, keepdim=True) + eps).float()
    return x * inv * (1.0 + w.float())


def qwen_block(x: torch.Tensor, w: QwenWeights, *, batch: int,
               residual_dtype: torch.dtype = torch.float32,
               out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    t, hidden = x.shape
    h, hk, d = w.heads, w.kv_heads, w.head_dim
    seq = t // batch
    n1_q = _q(_rms(x, w.in_norm_w, w.eps), w.norm_scale)
    qs = w.qkv_scale
    if w.interleaved:
        qg = _dq(_q(scaled_mm(n1_q, w.q_w, w.norm_scale, w.q_s), qs), qs).view(t, h, 2, d)
        q_raw, gate = qg[:, :, 0], qg[:, :, 1]
    else:
        q_raw = _dq(_q(scaled_mm(n1_q, w.q_w, w.norm_scale, w.q_s), qs), qs).view(t, h, d)
        gate = _dq(_q(scaled_mm(n1_q, w.gate_w, w.norm_scale, w.gate_s), qs), qs).view(t, h, d)
    k_raw = _dq(_q(scaled_mm(n1_q, w.k_w, w.norm_scale, w.k_s), qs), qs).view(t, hk, d)
    v = _dq(_q(scaled_mm(n1_q, w.v_w, w.norm_scale, w.v_s), qs), qs).view(t, hk, d)
    cos = w.cos.repeat(batch, 1) if w.cos.shape[0] == seq else w.cos
    sin = w.sin.repeat(batch, 1) if w.sin.shape[0] == seq else w.sin
    q = oatt.head_rmsnorm_rope(q_raw, w.q_norm_w, cos, sin, w.rotary_dim, w.eps)
    k = oatt.head_rmsnorm_rope(k_raw, w.k_norm_w, cos, sin, w.rotary_dim, w.eps)
    q = _dq(_q(q, qs), qs)
    k = _dq(_q(k, qs), qs)
    ctx = oatt.attention(q, k, v, batch=batch, causal=True, gate=gate,
                         sm_scale=1.0 / math.sqrt(d))
    ctx_q = _q(ctx.reshape(t, h * d), w.ctx_scale)
    r1 = _round(x + scaled_mm(ctx_q, w.o_w, w.ctx_scale, w.o_s), residual_dtype)
    if w.mlp_down_w is None:
        return _round(r1, out_dtype)
    n2_q = _q(_rms(r1, w.post_norm_w, w.eps), w.norm_scale)
    g = _q(scaled_mm(n2_q, w.mlp_gate_w, w.norm_scale, w.mlp_gate_s), w.mlp_proj_scale)
    u = _q(scaled_mm(n2_q, w.mlp_up_w, w.norm_scale, w.mlp_up_s), w.mlp_proj_scale)
    act = F.silu(_dq(g, w.mlp_proj_scale)) * _dq(u, w.mlp_proj_scale)
    act_q = _q(act, w.mlp_act_scale)
    out = r1 + scaled_mm(act_q, w.mlp_down_w, w.mlp_act_scale, w.mlp_down_s)
    return _round(out, out_dtype)
