"""Seeded inputs and weights for the block tests (CPU generator, identical bytes on the
GPU).  ``reference_*`` follow the reference evaluators' distributions and fixed scales
(tasks/model_gpt2_small_transformer_block_fp8/starter.py:157-174, 200-223 and
tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:186-229); ``baseline_*`` follow
BASELINE.json configs 4/5 (N(0,1) activations in bf16, N(0,0.02) weights with per-tensor
amax scales)."""
from __future__ import annotations

import torch

from oracle import attention as oatt
from oracle.blocks import GPT2Weights, QwenWeights


def _uq(shape, bound, g):
    """U(-bound, bound) quantised at scale bound/448 (reference weight convention)."""
    s = bound / 448.0
    w = torch.empty(shape).uniform_(-bound, bound, generator=g)
    return (w / s).to(torch.float8_e4m3fn), s


def _nq(shape, std, g):
    """N(0, std^2) quantised with its amax scale (BASELINE weight convention)."""
    w = torch.randn(shape, generator=g) * std
    s = float(w.abs().max()) / 448.0
    return (w / s).to(torch.float8_e4m3fn), s


def gpt2_weights(d=768, heads=12, mlp=3072, g=None, reference=True) -> GPT2Weights:
    mk = (lambda shape, fan: _uq(shape, fan ** -0.5, g)) if reference else \
         (lambda shape, fan: _nq(shape, 0.02, g))
    qkv_w, qkv_s = mk((3 * d, d), d)
    out_w, out_s = mk((d, d), d)
    fc_w, fc_s = mk((mlp, d), d)
    proj_w, proj_s = mk((d, mlp), mlp)
    b = lambda n: torch.randn(n, generator=g) * 0.02  # noqa: E731
    return GPT2Weights(qkv_w, qkv_s, b(3 * d), out_w, out_s, b(d), fc_w, fc_s, b(mlp),
                       proj_w, proj_s, b(d), 1 + b(d), b(d), 1 + b(d), b(d), heads=heads)


def qwen_weights(*, hidden, heads, kv_heads, head_dim, rotary_dim, theta, seq, g,
                 interleaved, mlp=0, reference=True) -> QwenWeights:
    qd, kvd = heads * head_dim, kv_heads * head_dim
    if reference:
        mk = lambda shape, fan: _uq(shape, fan ** -0.5, g)  # noqa: E731
    else:
        mk = lambda shape, fan: _nq(shape, 0.02, g)  # noqa: E731
    n = lambda k: torch.randn(k, generator=g) * 0.02  # noqa: E731
    in_norm, post_norm = n(hidden), n(hidden)
    q_norm, k_norm = n(head_dim), n(head_dim)
    if interleaved:
        q_w, q_s = mk((2 * qd, hidden), hidden)
        gate_w, gate_s = None, 1.0
    else:
        q_w, q_s = mk((qd, hidden), hidden)
        gate_w, gate_s = mk((qd, hidden), hidden)
    k_w, k_s = mk((kvd, hidden), hidden)
    v_w, v_s = mk((kvd, hidden), hidden)
    o_w, o_s = mk((hidden, qd), qd)
    cos, sin = oatt.rope_tables(seq, rotary_dim, theta)
    w = QwenWeights(q_w, q_s, gate_w, gate_s, k_w, k_s, v_w, v_s, o_w, o_s, in_norm, q_norm,
                    k_norm, cos, sin, heads, kv_heads, head_dim, rotary_dim, interleaved)
    if mlp:
        w.post_norm_w = post_norm
        w.mlp_gate_w, w.mlp_gate_s = mk((mlp, hidden), hidden)
        w.mlp_up_w, w.mlp_up_s = mk((mlp, hidden), hidden)
        w.mlp_down_w, w.mlp_down_s = mk((hidden, mlp), mlp)
    return w


def reference_hidden(t, d, g):
    """U(-1, 1) quantised at 1/448 (the block tasks' hidden input) -> (e4m3, scale)."""
    x = torch.empty((t, d)).uniform_(-1.0, 1.0, generator=g)
    return (x * 448.0).to(torch.float8_e4m3fn), 1.0 / 448.0
