"""Regenerates, on CPU, exactly the inputs that the reference evaluators draw.

Each function repeats the draws of one evaluator's ``main()`` (the code after
``# === CUTE_HARNESS_EVALUATOR_V1 ===`` in the reference task's starter.py): same seed, same
calls in the same order, CPU generator.  ``make_golden.py`` runs the evaluators themselves on
CPU and asserts that these regenerated tensors are bit-identical to the ones the evaluator
handed to the kernel, so the GPU tests can use them without the reference tree.

Returned e4m3 tensors are the stored bytes (``float8_e4m3fn``); scales follow the tasks.
"""
from __future__ import annotations

import torch

FP8_MAX = 448.0
E4M3 = torch.float8_e4m3fn


def _fp8(source: torch.Tensor, scale: float) -> torch.Tensor:
    return (source / scale).to(E4M3)


def square_gemm(seed=20260726, n=4096):
    """tasks/level1_01_square_matrix_multiplication_fp8/starter.py:61-99"""
    torch.manual_seed(seed)
    a = torch.rand((n, n), dtype=torch.float32)
    b = torch.rand((n, n), dtype=torch.float32)
    return {"a": (a * FP8_MAX).to(E4M3), "b": (b * FP8_MAX).to(E4M3),
            "scale_a": 1 / FP8_MAX, "scale_b": 1 / FP8_MAX, "source_a": a, "source_b": b}


def gemm_epilogue_task(seed, m=1024, n=8192, k=8192, bias=True, rand_bias=True):
    """tasks/level2_{09,12,40,63,76}_*/starter.py (A ~ U(0,1), B ~ U(+-K^-1/2), bias ~ N(0,1));
    level2_14 has no bias."""
    torch.manual_seed(seed)
    bound = k ** -0.5
    a = torch.rand((m, k), dtype=torch.float32)
    b = torch.empty((n, k), dtype=torch.float32).uniform_(-bound, bound)
    out = {"a": (a * FP8_MAX).to(E4M3), "b": (b * (FP8_MAX / bound)).to(E4M3),
           "scale_a": 1 / FP8_MAX, "scale_b": bound / FP8_MAX, "source_a": a, "source_b": b}
    if bias:
        out["bias"] = torch.randn((n,), dtype=torch.float32)
    return out


def qkv_projection(seed=20260731, m=8192, n=2304, k=768):
    """tasks/model_gpt2_small_qkv_projection_fp8/starter.py:66-110"""
    torch.manual_seed(seed)
    bound = k ** -0.5
    x = torch.empty((m, k), dtype=torch.float32).uniform_(-1.0, 1.0)
    w = torch.empty((n, k), dtype=torch.float32).uniform_(-bound, bound)
    bias = torch.randn((n,), dtype=torch.float32) * 0.02
    return {"a": (x * FP8_MAX).to(E4M3), "b": (w * (FP8_MAX / bound)).to(E4M3), "bias": bias,
            "scale_a": 1 / FP8_MAX, "scale_b": bound / FP8_MAX}


def gpt2_block(seed=20260801, tokens=128, hidden=768, mlp=3072, vision=False):
    """tasks/model_gpt2_small_transformer_block_fp8/starter.py:230-306 (and, with
    ``vision``, tasks/model_qwen35_4b_vision_block_fp8/starter.py:186-247: LN params, biases,
    RoPE tables, then weights in the order qkv, out, fc1, fc2)."""
    torch.manual_seed(seed)
    x = torch.empty((tokens, hidden), dtype=torch.float32).uniform_(-1.0, 1.0)
    r = lambda n: torch.randn((n,), dtype=torch.float32)  # noqa: E731
    ln1_w, ln1_b = 1.0 + 0.02 * r(hidden), 0.02 * r(hidden)
    ln2_w, ln2_b = 1.0 + 0.02 * r(hidden), 0.02 * r(hidden)
    qkv_b, out_b, fc_b, proj_b = 0.02 * r(3 * hidden), 0.02 * r(hidden), 0.02 * r(mlp), 0.02 * r(hidden)
    hb, mb = hidden ** -0.5, mlp ** -0.5
    shapes = [("qkv", 3 * hidden, hidden, hb), ("out", hidden, hidden, hb),
              ("fc", mlp, hidden, hb), ("proj", hidden, mlp, mb)]
    out = {"hidden": _fp8(x, 1 / FP8_MAX), "hidden_scale": 1 / FP8_MAX, "hidden_source": x,
           "ln1_w": ln1_w, "ln1_b": ln1_b, "ln2_w": ln2_w, "ln2_b": ln2_b,
           "qkv_b": qkv_b, "out_b": out_b, "fc_b": fc_b, "proj_b": proj_b}
    if vision:
        heads, hd = 16, hidden // 16
        pos = torch.arange(tokens, dtype=torch.float32)
        idx = torch.arange(0, hd, 2, dtype=torch.float32)
        inv = 1.0 / (10_000.0 ** (idx / hd))
        f = pos[:, None] * inv[None, :]
        emb = torch.cat((f, f), dim=-1)
        out["cos"], out["sin"] = emb.cos(), emb.sin()
    for name, rows, cols, bound in shapes:
        src = torch.empty((rows, cols), dtype=torch.float32).uniform_(-bound, bound)
        s = bound / FP8_MAX
        out[name + "_w"], out[name + "_s"] = _fp8(src, s), s
        out[name + "_source"] = src
    return out


def qwen_block(seed=20260801, tokens=128, hidden=2560, heads=16, kv_heads=4, head_dim=256,
               rotary=64, inter=9216, theta=10_000_000.0):
    """tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:186-236"""
    torch.manual_seed(seed)
    x = torch.empty((tokens, hidden), dtype=torch.float32).uniform_(-1.0, 1.0)
    r = lambda n: torch.randn((n,), dtype=torch.float32)  # noqa: E731
    in_norm, post_norm = 0.02 * r(hidden), 0.02 * r(hidden)
    q_norm, k_norm = 0.02 * r(head_dim), 0.02 * r(head_dim)
    pos = torch.arange(tokens, dtype=torch.float32)
    idx = torch.arange(0, rotary, 2, dtype=torch.float32)
    inv = 1.0 / (theta ** (idx / rotary))
    f = pos[:, None] * inv[None, :]
    emb = torch.cat((f, f), dim=-1)
    out = {"hidden": _fp8(x, 1 / FP8_MAX), "hidden_scale": 1 / FP8_MAX,
           "in_norm_w": in_norm, "post_norm_w": post_norm, "q_norm_w": q_norm,
           "k_norm_w": k_norm, "cos": emb.cos(), "sin": emb.sin()}
    qd, kvd = heads * head_dim, kv_heads * head_dim
    hb, cb, mb = hidden ** -0.5, qd ** -0.5, inter ** -0.5
    specs = [("q_gate", 2 * qd, hidden, hb), ("k", kvd, hidden, hb), ("v", kvd, hidden, hb),
             ("out", hidden, qd, cb), ("gate", inter, hidden, hb), ("up", inter, hidden, hb),
             ("down", hidden, inter, mb)]
    for name, rows, cols, bound in specs:
        src = torch.empty((rows, cols), dtype=torch.float32).uniform_(-bound, bound)
        s = bound / FP8_MAX
        out[name + "_w"], out[name + "_s"] = _fp8(src, s), s
    return out


def gpt2_weights_from(inp, heads=12):
    """Reference-task inputs -> oracle / GPU block weight container."""
    from oracle.blocks import GPT2Weights
    return GPT2Weights(inp["qkv_w"], inp["qkv_s"], inp["qkv_b"], inp["out_w"], inp["out_s"],
                       inp["out_b"], inp["fc_w"], inp["fc_s"], inp["fc_b"], inp["proj_w"],
                       inp["proj_s"], inp["proj_b"], inp["ln1_w"], inp["ln1_b"], inp["ln2_w"],
                       inp["ln2_b"], heads=heads, eps=1e-5 if heads == 12 else 1e-6)


def qwen_weights_from(inp, heads=16, kv_heads=4, head_dim=256, rotary=64):
    from oracle.blocks import QwenWeights
    w = QwenWeights(inp["q_gate_w"], inp["q_gate_s"], None, 1.0, inp["k_w"], inp["k_s"],
                    inp["v_w"], inp["v_s"], inp["out_w"], inp["out_s"], inp["in_norm_w"],
                    inp["q_norm_w"], inp["k_norm_w"], inp["cos"], inp["sin"], heads, kv_heads,
                    head_dim, rotary, interleaved=True)
    w.post_norm_w = inp["post_norm_w"]
    w.mlp_gate_w, w.mlp_gate_s = inp["gate_w"], inp["gate_s"]
    w.mlp_up_w, w.mlp_up_s = inp["up_w"], inp["up_s"]
    w.mlp_down_w, w.mlp_down_s = inp["down_w"], inp["down_s"]
    return w


def layer_norm_task(seed=20260726, batch=16, row=64 * 256 * 256):
    """tasks/level1_40_layer_norm_fp8/starter.py:88-109: U(0,1) * 448 -> e4m3, read at 1/448."""
    torch.manual_seed(seed)
    src = torch.rand((batch, row), dtype=torch.float32)
    return {"x": (src * FP8_MAX).to(E4M3), "x_scale": 1 / FP8_MAX, "eps": 1e-5}


def gated_residual(seed=20260731, m=2048, n=4096, k=4096):
    """cute_kernels/fused_gemm_gated_residual_fp8/submission.py:325-350: A ~ U(-1,1),
    B ~ U(+-K^-1/2), gate and residual ~ N(0,1) f32."""
    torch.manual_seed(seed)
    bound = k ** -0.5
    a = torch.empty((m, k), dtype=torch.float32).uniform_(-1.0, 1.0)
    b = torch.empty((n, k), dtype=torch.float32).uniform_(-bound, bound)
    gate = torch.randn((m, n), dtype=torch.float32)
    residual = torch.randn((m, n), dtype=torch.float32)
    return {"a": (a * FP8_MAX).to(E4M3), "b": (b * (FP8_MAX / bound)).to(E4M3),
            "scale_a": 1 / FP8_MAX, "scale_b": bound / FP8_MAX, "gate": gate,
            "residual": residual}
