"""The oracle is pinned: every reference evaluator, executed on CPU by make_golden.py with the
oracle standing in for its kernel, printed PASS; and the committed fixtures agree with a
fresh oracle evaluation of the regenerated evaluator inputs (small tasks, CPU only)."""
from __future__ import annotations

import json
import os
import sys

import pytest
import torch

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

TASKS = [
    "level1_01_square_matrix_multiplication_fp8", "level2_09_matmul_subtract_multiply_relu_fp8",
    "level2_12_gemm_multiply_leaky_relu_fp8", "level2_14_gemm_divide_sum_scaling_fp8",
    "level2_40_matmul_scaling_residual_add_fp8", "level2_63_gemm_relu_divide_fp8",
    "level2_76_gemm_add_relu_fp8", "model_gpt2_small_qkv_projection_fp8",
    "model_gpt2_small_transformer_block_fp8", "model_qwen35_4b_full_attention_block_fp8",
    "model_qwen35_4b_vision_block_fp8", "level1_40_layer_norm_fp8",
    "fused_gemm_gated_residual_fp8",
]


def _results():
    path = os.path.join(GOLDEN, "reference_pass.json")
    if not os.path.exists(path):
        pytest.skip("golden fixtures not generated")
    return json.load(open(path))


@pytest.mark.parametrize("task", TASKS)
def test_reference_evaluator_accepted_oracle(task):
    res = _results()
    assert task in res, f"{task} missing from reference_pass.json"
    line = res[task]["evaluator_line"]
    assert line.startswith(("task=", "kernel=")) and line.endswith(" PASS"), line
    assert res[task]["inputs_regenerated"]
    assert os.path.exists(os.path.join(GOLDEN, task + ".pt"))


def test_gpt2_block_fixture_matches_fresh_oracle():
    import task_inputs as ti
    from oracle import blocks as ob
    fix = torch.load(os.path.join(GOLDEN, "model_gpt2_small_transformer_block_fp8.pt"))
    inp = ti.gpt2_block()
    y = ob.gpt2_block(inp["hidden"].float() * inp["hidden_scale"], ti.gpt2_weights_from(inp),
                      batch=1)
    assert torch.allclose(y.to(torch.float16).float(), fix["output_f16"].float(), atol=1e-3)


def test_qkv_projection_fixture_matches_fresh_oracle_samples():
    import task_inputs as ti
    from oracle import gemm as og
    fix = torch.load(os.path.join(GOLDEN, "model_gpt2_small_qkv_projection_fp8.pt"))
    inp = ti.qkv_projection()
    idx = fix["index"]
    rows = torch.unique(idx // fix["shape"][1])[:64]
    sub = og.gemm_epilogue(inp["a"][rows], inp["b"], inp["scale_a"], inp["scale_b"],
                           bias=inp["bias"])
    full = torch.full(fix["shape"], float("nan"))
    full[rows] = sub
    got = full.reshape(-1)[idx]
    m = ~torch.isnan(got)
    assert m.any()
    assert torch.allclose(got[m], fix["value"][m], atol=1e-5)


def test_layer_norm_fixture_matches_fresh_oracle_samples():
    import task_inputs as ti
    from oracle import norm as onorm
    fix = torch.load(os.path.join(GOLDEN, "level1_40_layer_norm_fp8.pt"))
    inp = ti.layer_norm_task()
    y = onorm.layer_norm_rows(inp["x"].float() * inp["x_scale"], inp["eps"])
    assert list(y.shape) == fix["shape"]
    assert torch.allclose(y.reshape(-1)[fix["index"]], fix["value"], atol=1e-5)


def test_gated_residual_fixture_matches_fresh_oracle_samples():
    import task_inputs as ti
    from oracle import gemm as og
    fix = torch.load(os.path.join(GOLDEN, "fused_gemm_gated_residual_fp8.pt"))
    inp = ti.gated_residual()
    n = fix["shape"][1]
    rows = torch.unique(fix["index"] // n)[:48]
    sub = og.gemm_epilogue(inp["a"][rows], inp["b"], inp["scale_a"], inp["scale_b"],
                           gate=inp["gate"][rows], residual=inp["residual"][rows])
    full = torch.full(fix["shape"], float("nan"))
    full[rows] = sub
    got = full.reshape(-1)[fix["index"]]
    m = ~torch.isnan(got)
    assert m.any()
    assert torch.allclose(got[m], fix["value"][m], atol=1e-5)
