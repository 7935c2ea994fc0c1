"""Decoder blocks on the GPU vs the CPU oracle of the reference evaluators' math.

Bars: the reference tasks' own output thresholds — GPT-2 quantised path max-abs 0.05
(tasks/model_gpt2_small_transformer_block_fp8/starter.py:545-547), Qwen 0.08
(tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:418) — at the reference shapes;
BASELINE-style bf16 shapes use the same abs bar plus one bf16 rounding of the output.
"""
from __future__ import annotations

import pytest
import torch

from block_inputs import gpt2_weights, qwen_weights, reference_hidden
from helpers import gen
from oracle import attention as oatt
from oracle import blocks as ob

pytestmark = pytest.mark.gpu


def _blocks():
    from b200fp8 import blocks
    return blocks


def _check(out, ref, tol, rel=0.0):
    err = (out.float().cpu() - ref).abs()
    assert torch.isfinite(out.float()).all()
    bound = tol + rel * ref.abs()
    assert bool((err <= bound).all()), f"max err {float(err.max())}"


def test_gpt2_block_reference_task_shape():
    g = gen(20260801)
    w = gpt2_weights(g=g)
    x_q, xs = reference_hidden(128, 768, g)
    ref = ob.gpt2_block(x_q.float() * xs, w, batch=1)
    blk = _blocks().GPT2Block(w, batch=1, seq=128)
    out = blk.forward(x_q.cuda(), xs)
    torch.cuda.synchronize()
    _check(out, ref, 0.05)


@pytest.mark.parametrize("batch,seq", [(2, 256), (1, 1024)])
def test_gpt2_block_baseline_style_bf16(batch, seq):
    g = gen(20260801 + seq)
    w = gpt2_weights(g=g, reference=False)
    x = (torch.randn((batch * seq, 768), generator=g)).to(torch.bfloat16)
    ref = ob.gpt2_block(x.float(), w, batch=batch, residual_dtype=torch.bfloat16,
                        out_dtype=torch.bfloat16)
    blk = _blocks().GPT2Block(w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                              out_dtype=torch.bfloat16)
    out = blk.forward(x.cuda())
    torch.cuda.synchronize()
    _check(out, ref, 0.05, 2.0 ** -8)
    # CUDA-graph replay reproduces the eager result bit for bit
    eager = out.clone()
    gout = blk.capture(x.cuda())
    blk.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, eager)


def test_qwen_block_reference_task_shape():
    g = gen(20260801)
    w = qwen_weights(hidden=2560, heads=16, kv_heads=4, head_dim=256, rotary_dim=64,
                     theta=1e7, seq=128, g=g, interleaved=True, mlp=9216)
    x_q, xs = reference_hidden(128, 2560, g)
    ref = ob.qwen_block(x_q.float() * xs, w, batch=1)
    blk = _blocks().QwenBlock(w, batch=1, seq=128)
    out = blk.forward(x_q.cuda(), xs)
    torch.cuda.synchronize()
    _check(out, ref, 0.08)


def test_qwen_block_baseline_style_bf16():
    g = gen(20260802)
    batch, seq = 2, 256
    w = qwen_weights(hidden=2560, heads=32, kv_heads=8, head_dim=128, rotary_dim=128,
                     theta=1e6, seq=seq, g=g, interleaved=False, reference=False)
    x = torch.randn((batch * seq, 2560), generator=g).to(torch.bfloat16)
    ref = ob.qwen_block(x.float(), w, batch=batch, residual_dtype=torch.bfloat16,
                        out_dtype=torch.bfloat16)
    blk = _blocks().QwenBlock(w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                              out_dtype=torch.bfloat16)
    out = blk.forward(x.cuda())
    torch.cuda.synchronize()
    _check(out, ref, 0.08, 2.0 ** -8)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_qwen_heads_parallel_partials_sum_to_block(tp):
    """The head slices of the tensor-parallel block, run on one GPU and summed in f32 (what
    the all-reduce does across GPUs), match the unsharded block and the oracle."""
    from b200fp8 import sharding
    g = gen(20260803)
    batch, seq = 2, 256
    w = qwen_weights(hidden=2560, heads=32, kv_heads=8, head_dim=128, rotary_dim=128,
                     theta=1e6, seq=seq, g=g, interleaved=False, reference=False)
    x = torch.randn((batch * seq, 2560), generator=g).to(torch.bfloat16)
    ref = ob.qwen_block(x.float(), w, batch=batch, residual_dtype=torch.bfloat16,
                        out_dtype=torch.bfloat16)
    total = torch.zeros((batch * seq, 2560), device="cuda")
    xd = x.cuda()
    for r in range(tp):
        local = sharding.qwen_tp_weights(w, r, tp)
        blk = _blocks().QwenBlock(local, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                                  out_dtype=torch.bfloat16, add_residual=(r == 0))
        total += blk.forward(xd).float()
    torch.cuda.synchronize()
    _check(total.to(torch.bfloat16), ref, 0.08, 2.0 ** -7)


def _f32_scales(w, names):
    # the C ABI takes f32 scales; round them so both paths form the same GEMM alpha
    for n in names:
        setattr(w, n, float(torch.tensor(getattr(w, n), dtype=torch.float32)))


@pytest.mark.parametrize("vision", [False, True])
def test_gpt2_block_native_entry_matches_python_block(vision):
    """b2f_gpt2_block (one C call) reproduces the Python-composed block bit for bit."""
    g = gen(20260805)
    w = gpt2_weights(g=g, reference=False, d=1024 if vision else 768, heads=16 if vision else 12,
                     mlp=4096 if vision else 3072)
    _f32_scales(w, ("qkv_s", "out_s", "fc_s", "proj_s"))
    batch, seq, d = 2, 256, w.qkv_w.shape[1]
    kw = {}
    if vision:
        cos, sin = oatt.rope_tables(seq, d // 16, 1e4)
        kw = dict(causal=False, rope_cos=cos, rope_sin=sin)
    x = torch.randn((batch * seq, d), generator=g).to(torch.bfloat16).cuda()
    blk = _blocks().GPT2Block(w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                              out_dtype=torch.bfloat16, **kw)
    a = blk.forward(x).clone()
    b = blk.forward_abi(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("mlp", [False, True])
def test_qwen_block_native_entry_matches_python_block(mlp):
    """b2f_qwen_block reproduces the Python-composed block bit for bit (BASELINE geometry
    without the MLP, the reference task's geometry with it)."""
    g = gen(20260806)
    if mlp:
        w = qwen_weights(hidden=2560, heads=16, kv_heads=4, head_dim=256, rotary_dim=64,
                         theta=1e7, seq=128, g=g, interleaved=True, mlp=9216)
        batch, seq = 1, 128
        _f32_scales(w, ("o_s", "mlp_down_s"))
    else:
        batch, seq = 2, 256
        w = qwen_weights(hidden=2560, heads=32, kv_heads=8, head_dim=128, rotary_dim=128,
                         theta=1e6, seq=seq, g=g, interleaved=False, reference=False)
        _f32_scales(w, ("o_s",))
    x = torch.randn((batch * seq, 2560), generator=g).to(torch.bfloat16).cuda()
    blk = _blocks().QwenBlock(w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                              out_dtype=torch.bfloat16)
    a = blk.forward(x).clone()
    b = blk.forward_abi(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
