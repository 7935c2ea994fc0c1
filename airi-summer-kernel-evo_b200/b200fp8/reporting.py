"""Harness-side reporting with throughput and roofline columns.

Mirrors the reference's evaluation record and comparison table
(``experiment/evaluation.py:13-43`` ``EvaluationResult``, ``cute_harness/compare.py:20-147``
``comparison_row`` / ``render_comparison_table`` / ``write_comparison_reports``) and adds,
per run: TFLOP/s, GB/s, the fraction of the measured B200 roofline, the GPU count and the
path of the ncu summary that explains the number.  Field names of the reference's record
(``exit_code``, ``record.acceptance.passed``, ``record.benchmark.kernel_time_ms``) are kept,
so a record written here reads the same through the reference's accessors.
"""
from __future__ import annotations

import csv
import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Optional

_TIME_RE = re.compile(r"(?<![A-Za-z0-9_])kernel_time_ms=([0-9]+(?:\.[0-9]+)?)")
_ROOT = Path(__file__).resolve().parents[2]

# ncu summaries committed for the kernels behind each task family
NCU_SUMMARIES = {
    "gemm": "profiles/gemm_fp8_pair_qwen_square8192.md",
    "gpt2": "profiles/blocks_launch_lists.md",
    "vision": "profiles/blocks_launch_lists.md",
    "qwen": "profiles/blocks_launch_lists.md",
    "layer_norm": "profiles/memory_bound_kernels.md",
}


def measured_peaks() -> dict:
    """HBM GB/s and e4m3 dense TFLOP/s (2 x the measured bf16 burst) of this pool's B200s
    from MEASURED_PEAKS.json at the repository root; the earlier measurement otherwise."""
    try:
        with open(_ROOT / "MEASURED_PEAKS.json") as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "fp8_tflops": 2.0 * float(d["bf16_tflops"]),
                "basis": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "fp8_tflops": 3180.0, "basis": "fallback"}


def kernel_time_from_stdout(stdout: str) -> Optional[float]:
    """The last ``kernel_time_ms=`` value of an evaluator's output (cute_harness/cli.py:122-133)."""
    m = _TIME_RE.findall(stdout or "")
    if not m:
        return None
    v = float(m[-1])
    return v if v > 0 else None


def benchmark_record(task_id: str, stdout: str, n_gpus: int = 1,
                     ncu_summary: Optional[str] = None) -> dict:
    """``record["benchmark"]`` of one evaluated task: the evaluator's kernel time plus the
    task's algorithmic work, achieved TFLOP/s and GB/s and the roofline fraction."""
    from .harness import TASKS, task_work
    t_ms = kernel_time_from_stdout(stdout)
    work = task_work(task_id)
    peaks = measured_peaks()
    rec = {"kernel_time_ms": t_ms, "n_gpus": n_gpus, "flops": work["flops"],
           "bytes": work["bytes"], "bound": work["bound"], "peak_basis": peaks["basis"],
           "ncu_summary": ncu_summary or NCU_SUMMARIES.get(TASKS[task_id]["family"])}
    if t_ms:
        s = t_ms * 1e-3
        rec["tflops"] = work["flops"] / s / 1e12 if work["flops"] else None
        rec["gbs"] = work["bytes"] / s / 1e9
        if work["bound"] == "tensor":
            rec["roofline_frac"] = rec["tflops"] / peaks["fp8_tflops"]
        else:
            rec["roofline_frac"] = rec["gbs"] / peaks["hbm_gbs"]
    return rec


@dataclass(frozen=True)
class EvaluationResult:
    """The reference's evaluation result (experiment/evaluation.py:13-43) with the
    throughput and roofline fields of ``record["benchmark"]`` exposed."""

    exit_code: int
    record: Optional[dict]
    error: Optional[str]

    @property
    def passed(self) -> bool:
        if not self.record:
            return False
        acceptance = self.record.get("acceptance")
        return isinstance(acceptance, dict) and acceptance.get("passed") is True

    def _bench(self, key):
        if not self.record or not isinstance(self.record.get("benchmark"), dict):
            return None
        v = self.record["benchmark"].get(key)
        return v

    @property
    def kernel_time_ms(self) -> Optional[float]:
        v = self._bench("kernel_time_ms")
        return float(v) if isinstance(v, (int, float)) else None

    @property
    def tflops(self) -> Optional[float]:
        return self._bench("tflops")

    @property
    def gbs(self) -> Optional[float]:
        return self._bench("gbs")

    @property
    def roofline_frac(self) -> Optional[float]:
        return self._bench("roofline_frac")

    @property
    def n_gpus(self) -> Optional[int]:
        return self._bench("n_gpus")

    @property
    def ncu_summary(self) -> Optional[str]:
        return self._bench("ncu_summary")

    def to_dict(self) -> dict:
        return {"exit_code": self.exit_code, "passed": self.passed,
                "kernel_time_ms": self.kernel_time_ms, "tflops": self.tflops, "gbs": self.gbs,
                "roofline_frac": self.roofline_frac, "n_gpus": self.n_gpus,
                "ncu_summary": self.ncu_summary, "error": self.error, "record": self.record}


def evaluation_result(task_id: str, response: dict, n_gpus: int = 1) -> EvaluationResult:
    """Builds the result from a ``run_reference_evaluator`` response: acceptance as the
    reference decides it (exit 0, no timeout, ``success_pattern`` in stdout,
    cute_harness/cli.py:104-119) plus the benchmark record."""
    from .harness import TASKS, success_pattern
    stdout = response.get("stdout") or ""
    family_task = TASKS[task_id]
    pattern = response.get("success_pattern") or success_pattern(task_id)
    matched = re.search(pattern, stdout) is not None
    server_ok = (response.get("success") is True and response.get("exit_code") == 0
                 and response.get("timed_out") is not True)
    record = {"task_id": task_id, "entry": family_task["entry"],
              "acceptance": {"server_success": server_ok, "success_pattern_matched": matched,
                             "passed": server_ok and matched},
              "benchmark": benchmark_record(task_id, stdout, n_gpus)}
    return EvaluationResult(response.get("exit_code", 1), record, response.get("error"))


TABLE_FIELDS = (
    ("candidate", "Candidate"), ("task_id", "Task"), ("status", "Status"),
    ("baseline_ms", "Baseline ms"), ("candidate_ms", "Candidate ms"), ("speedup", "Speedup"),
    ("tflops", "TFLOP/s"), ("gbs", "GB/s"), ("roofline_frac", "Roofline"),
    ("n_gpus", "GPUs"), ("ncu_summary", "ncu summary"),
)


def comparison_row(candidate: str, task_id: str, *, status: str,
                   baseline_ms: Optional[float], candidate_ms: Optional[float],
                   result: Optional[EvaluationResult] = None,
                   error: Optional[str] = None) -> dict:
    """compare.py's row (cute_harness/compare.py:50-75) plus the throughput columns."""
    speedup = None
    if status == "PASS" and baseline_ms is not None and candidate_ms and candidate_ms > 0:
        speedup = baseline_ms / candidate_ms
    row = {"candidate": candidate, "task_id": task_id, "status": status,
           "baseline_ms": baseline_ms, "candidate_ms": candidate_ms, "speedup": speedup,
           "tflops": None, "gbs": None, "roofline_frac": None, "n_gpus": None,
           "ncu_summary": None, "error": error}
    if result is not None:
        row.update(tflops=result.tflops, gbs=result.gbs, roofline_frac=result.roofline_frac,
                   n_gpus=result.n_gpus, ncu_summary=result.ncu_summary)
    return row


def _display(field: str, value: Any) -> str:
    if value is None:
        return "-"
    if field in {"baseline_ms", "candidate_ms"}:
        return f"{float(value):.6f}"
    if field == "speedup":
        return f"{float(value):.3f}x"
    if field in {"tflops", "gbs"}:
        return f"{float(value):.1f}"
    if field == "roofline_frac":
        return f"{100.0 * float(value):.1f}%"
    return str(value)


def render_comparison_table(rows: list) -> str:
    headers = [h for _, h in TABLE_FIELDS]
    rendered = [[_display(f, r.get(f)) for f, _ in TABLE_FIELDS] for r in rows]
    widths = [max(len(headers[i]), *(len(r[i]) for r in rendered)) if rendered else
              len(headers[i]) for i in range(len(headers))]
    line = " | ".join(h.ljust(widths[i]) for i, h in enumerate(headers))
    sep = "-+-".join("-" * w for w in widths)
    body = [" | ".join(v.ljust(widths[i]) for i, v in enumerate(r)) for r in rendered]
    return "\n".join((line, sep, *body))


def write_comparison_reports(output_dir, *, metadata: dict, rows: list) -> None:
    """comparison.json / .csv / .txt as compare.py writes them, with the new columns."""
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    payload = dict(metadata)
    payload["rows"] = rows
    (out / "comparison.json").write_text(json.dumps(payload, indent=2) + "\n", encoding="utf-8")
    fields = [f for f, _ in TABLE_FIELDS] + ["error"]
    with (out / "comparison.csv").open("w", newline="", encoding="utf-8") as fh:
        w = csv.DictWriter(fh, fieldnames=fields)
        w.writeheader()
        for r in rows:
            w.writerow({f: r.get(f) for f in fields})
    (out / "comparison.txt").write_text(render_comparison_table(rows) + "\n", encoding="utf-8")
