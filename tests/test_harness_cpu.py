"""Evaluator-compatible entry points (b200fp8.harness) and the reporting record, on CPU.

The hosting test runs a reference task's own evaluator (read from the reference checkout
when it is present; skipped otherwise) under the CPU shims of tests/golden/make_golden.py,
with ``harness.make_entry`` built from the evaluator's namespace as the candidate: the
evaluator hands the entry point its exact positional arguments (inputs, workspaces,
output), which are checked against the entry's layout, and the values come from the CPU
oracle (the kernels need a GPU).  The evaluator must print its PASS line."""
from __future__ import annotations

import json
import os
import re
import sys

import pytest
import torch

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")
REFERENCE = os.environ.get("B2F_REFERENCE", "")


def _mg():
    if GOLDEN not in sys.path:
        sys.path.insert(0, GOLDEN)
    import make_golden
    return make_golden


def test_task_table_names_and_patterns():
    from b200fp8 import harness
    names = {s["entry"] for s in harness.TASKS.values()}
    assert len(names) == len(harness.TASKS)  # one entry point per task
    for tid in harness.TASKS:
        e = harness.make_entry(tid)
        assert e.__name__ == harness.TASKS[tid]["entry"]
        assert re.match(harness.success_pattern(tid), f"task={tid.rsplit('_fp8', 1)[0] if not tid.startswith('model_') else tid} x=1 kernel_time_ms=0.1 PASS")
    if REFERENCE and os.path.isdir(os.path.join(REFERENCE, "tasks")):
        for tid, spec in harness.TASKS.items():
            with open(os.path.join(REFERENCE, "tasks", tid, "task.json")) as f:
                tj = json.load(f)
            assert tj["validation"]["success_pattern"] == harness.success_pattern(tid)
            want = tj.get("policy", {}).get("entrypoint_jit")
            if want:
                assert want == spec["entry"], tid


# positional layout of each evaluator call: (inputs before the workspaces, total args)
_LAYOUT = {
    "level2_76_gemm_add_relu_fp8": (3, 4),
    "model_gpt2_small_qkv_projection_fp8": (3, 4),
    "model_gpt2_small_transformer_block_fp8": (13, 22),
    "model_qwen35_4b_vision_block_fp8": (15, 25),
}
# (the Qwen full-attention evaluator, 14 inputs + 14 workspaces + output, takes minutes on
# CPU; its entry point is driven with the same inputs by tests/test_harness_gpu.py)


@pytest.mark.skipif(not (REFERENCE and os.path.isdir(os.path.join(REFERENCE, "tasks"))),
                    reason="set B2F_REFERENCE to a reference checkout to run the evaluators")
@pytest.mark.parametrize("task", sorted(_LAYOUT))
def test_reference_evaluator_hosts_the_entry_point(task):
    from b200fp8 import harness
    mg = _mg()
    seed = harness.TASKS[task]["seed"]
    entry_name = harness.TASKS[task]["entry"]
    n_in, n_total = _LAYOUT[task]
    seen = {}

    def make_candidate(ns):
        entry = harness.make_entry(task, ns)       # built from the evaluator's constants
        assert entry.__name__ == entry_name and entry_name in ns
        fam = harness.TASKS[task]["family"]
        if fam == "gemm":
            oracle = mg.gemm_candidate(ns, harness.TASKS[task]["epilogue"])
        elif fam == "qwen":
            oracle = mg.qwen_candidate(ns)
        else:
            oracle = mg.gpt2_candidate(ns, vision=fam == "vision")

        def cand(*args):
            seen["n"] = len(args)
            assert len(args) == n_total
            assert args[0].dtype == torch.uint8            # e4m3 storage of the first input
            assert args[-1].dtype == torch.float32          # the evaluator's output buffer
            oracle(*args)
        return cand

    line, _, _ = mg._run_with_ns_candidate(
        os.path.join(REFERENCE, "tasks", task, "starter.py"), seed, entry_name, make_candidate)
    assert seen["n"] == n_total
    assert re.search(harness.success_pattern(task), line), line


def test_reporting_record_and_table(tmp_path):
    from b200fp8 import reporting
    stdout = ("task=level2_76_gemm_add_relu full_max_abs=0.001 sample_max_abs=0.01 "
              "kernel_time_ms=0.120000 PASS\n")
    res = reporting.evaluation_result(
        "level2_76_gemm_add_relu_fp8",
        {"stdout": stdout, "success": True, "exit_code": 0, "timed_out": False})
    assert res.passed and res.kernel_time_ms == pytest.approx(0.12)
    assert res.tflops == pytest.approx(2 * 1024 * 8192 * 8192 / 0.12e-3 / 1e12)
    assert 0 < res.roofline_frac < 1.5 and res.n_gpus == 1
    assert res.ncu_summary.startswith("profiles/")
    bad = reporting.evaluation_result(
        "level2_76_gemm_add_relu_fp8",
        {"stdout": "validation failed", "success": False, "exit_code": 1, "timed_out": False})
    assert not bad.passed and bad.kernel_time_ms is None
    rows = [reporting.comparison_row("001:b200fp8", "level2_76_gemm_add_relu_fp8",
                                     status="PASS", baseline_ms=0.3, candidate_ms=0.12,
                                     result=res)]
    assert rows[0]["speedup"] == pytest.approx(2.5)
    txt = reporting.render_comparison_table(rows)
    assert "TFLOP/s" in txt and "Roofline" in txt and "2.500x" in txt
    reporting.write_comparison_reports(tmp_path, metadata={"task": "x"}, rows=rows)
    assert json.loads((tmp_path / "comparison.json").read_text())["rows"][0]["status"] == "PASS"
    assert (tmp_path / "comparison.csv").read_text().startswith("candidate,task_id")
