"""GPU kernels on the reference evaluators' own inputs vs the golden vectors.

Inputs come from tests/golden/task_inputs.py (bit-identical to what each reference
evaluator draws, checked by make_golden.py); expected values are the oracle outputs that the
reference evaluators themselves accepted (tests/golden/<task>.pt).  Bars are each task's
own threshold from its task.json ``validation`` block, plus one f16 rounding of the stored
block outputs (|x| < 8 -> 2^-9 relative)."""
from __future__ import annotations

import os

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(ROOT, "tests", "golden")


def _fixture(task):
    path = os.path.join(GOLDEN, task + ".pt")
    if not os.path.exists(path):
        pytest.skip(f"fixture {task}.pt not generated")
    return torch.load(path)


def _ti():
    import sys
    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    import task_inputs
    return task_inputs


GEMM = {
    # task: (inputs, epilogue kwargs for ops.gemm_fp8, threshold)
    "level1_01_square_matrix_multiplication_fp8": (lambda t: t.square_gemm(), {}, 0.125),
    "level2_76_gemm_add_relu_fp8": (lambda t: t.gemm_epilogue_task(20260726),
                                    {"act": "relu"}, 0.01),
    "level2_09_matmul_subtract_multiply_relu_fp8": (
        lambda t: t.gemm_epilogue_task(20260727), {"pre_mul": 1.5, "pre_add": -3.0, "act": "relu"}, 0.01),
    "level2_12_gemm_multiply_leaky_relu_fp8": (
        lambda t: t.gemm_epilogue_task(20260727),
        {"pre_mul": 2.0, "act": "leaky_relu", "act_param": 0.1}, 0.01),
    "level2_14_gemm_divide_sum_scaling_fp8": (
        lambda t: t.gemm_epilogue_task(20260727, bias=False),
        {"post_mul": 0.5, "rowsum": True, "out_scale": 1 / 1.5}, 0.05),
    "level2_40_matmul_scaling_residual_add_fp8": (
        lambda t: t.gemm_epilogue_task(20260727), {"pre_mul": 1.5}, 0.01),
    "level2_63_gemm_relu_divide_fp8": (
        lambda t: t.gemm_epilogue_task(20260727), {"act": "relu", "post_mul": 0.5}, 0.01),
    "model_gpt2_small_qkv_projection_fp8": (lambda t: t.qkv_projection(), {}, 0.01),
}


@pytest.mark.parametrize("task", sorted(GEMM))
def test_gemm_task_golden(task):
    from b200fp8 import ops
    make, kw, thr = GEMM[task]
    fix = _fixture(task)
    inp = make(_ti())
    bias = inp.get("bias")
    out = ops.gemm_fp8(inp["a"].cuda(), inp["b"].cuda(), scale_a=inp["scale_a"],
                       scale_b=inp["scale_b"], bias=None if bias is None else bias.cuda(),
                       out_dtype=torch.float32, **kw)
    torch.cuda.synchronize()
    got = out.cpu().reshape(-1)[fix["index"]]
    err = (got - fix["value"]).abs().max().item()
    assert err <= thr, err
    assert abs(float(out.abs().max()) - fix["max_abs"]) <= thr


def _block_check(out, fix, thr):
    want = fix["output_f16"].float()
    err = (out.float().cpu() - want).abs()
    bound = thr + want.abs() * 2.0 ** -9
    assert torch.isfinite(out).all()
    assert bool((err <= bound).all()), float(err.max())


def test_gpt2_block_golden():
    from b200fp8 import blocks
    t = _ti()
    fix = _fixture("model_gpt2_small_transformer_block_fp8")
    inp = t.gpt2_block()
    blk = blocks.GPT2Block(t.gpt2_weights_from(inp), batch=1, seq=128)
    out = blk.forward(inp["hidden"].cuda(), inp["hidden_scale"])
    torch.cuda.synchronize()
    _block_check(out, fix, 0.05)


def test_vision_block_golden():
    from b200fp8 import blocks
    t = _ti()
    fix = _fixture("model_qwen35_4b_vision_block_fp8")
    inp = t.gpt2_block(hidden=1024, mlp=4096, vision=True)
    w = t.gpt2_weights_from(inp, heads=16)
    blk = blocks.GPT2Block(w, batch=1, seq=128, causal=False, rope_cos=inp["cos"],
                           rope_sin=inp["sin"])
    out = blk.forward(inp["hidden"].cuda(), inp["hidden_scale"])
    torch.cuda.synchronize()
    _block_check(out, fix, 0.06)


def test_qwen_block_golden():
    from b200fp8 import blocks
    t = _ti()
    fix = _fixture("model_qwen35_4b_full_attention_block_fp8")
    inp = t.qwen_block()
    blk = blocks.QwenBlock(t.qwen_weights_from(inp), batch=1, seq=128)
    out = blk.forward(inp["hidden"].cuda(), inp["hidden_scale"])
    torch.cuda.synchronize()
    _block_check(out, fix, 0.08)
