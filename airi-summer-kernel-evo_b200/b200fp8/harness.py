"""Evaluator-compatible entry points: every reference task's ``@cute.jit`` entry, on b200fp8.

The reference scores a candidate by appending the task's own evaluator (the code after
``# === CUTE_HARNESS_EVALUATOR_V1 ===`` in ``tasks/<id>/starter.py``) to it; the evaluator
draws seeded inputs, calls ``cute.compile(<entry>, *arguments)`` and then the compiled
entry with the same positional arguments (inputs, then evaluator-owned workspaces, then
``output``), times ``_CUTE_HARNESS_REPEATS`` calls with CUDA events, checks the output
against its Torch reference and prints ``task=<id> ... kernel_time_ms=<t> PASS``
(``cute_harness/assembly.py:87-106``, ``cute_harness/cli.py:104-133``).

This module gives each task's entry point with that exact name and positional signature,
running on the b200fp8 kernels (``make_entry``), and ``run_reference_evaluator``, which
executes a task's own evaluator, read from a reference checkout, with the entry point in
place of the compiled CuTe kernel: the evaluator's input generation, reference math,
thresholds, timing loop and PASS line all run unchanged, so ``cute_harness``'s
``_acceptance`` / ``_kernel_time_ms`` and ``compare.py`` consume its output as they would a
CuTe candidate's.  Only the DSL's three calls are substituted: ``cute.compile`` returns the
entry point, ``from_dlpack(t).mark_layout_dynamic(...)`` hands back ``t``, and
``create_cute_tensor_for_fp8(storage, dtype, 1, source)`` stores ``source`` rounded to e4m3
(round to nearest even, as the DSL's conversion) into the uint8 ``storage``.

Arguments are torch CUDA tensors: e4m3 operands as their uint8 storage, the rest f32.
Evaluator workspaces are accepted and left untouched (the evaluators allow it); the entry
points keep their own intermediates, cached per weight set.

    python -m b200fp8.harness list
    python -m b200fp8.harness run <task_id> --reference <checkout> [--seed S]
                                  [--warmup W] [--repeats R]
"""
from __future__ import annotations

import argparse
import builtins
import contextlib
import io
import json
import os
import sys
import types
from types import SimpleNamespace
from typing import Callable, Dict, Optional

import torch

E4M3 = torch.float8_e4m3fn
FP8_MAX = 448.0
MARKER = "# === CUTE_HARNESS_EVALUATOR_V1 ==="


def _e(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == E4M3 else t.view(E4M3)


def _c(ns: dict, name: str):
    return ns["_CUTE_HARNESS_" + name]


# ------------------------------------------------------------------------- task table
# task id: (entry name, family, epilogue of the GEMM family, evaluator seed, default
# evaluator constants used when no evaluator namespace is given)
def _gemm_consts(k: int) -> dict:
    return {"_CUTE_HARNESS_SCALE_A": 1.0 / FP8_MAX,
            "_CUTE_HARNESS_SCALE_B": k ** -0.5 / FP8_MAX}


def _block_consts(hidden, heads, mlp, eps, **extra) -> dict:
    d = {"_CUTE_HARNESS_HIDDEN": hidden, "_CUTE_HARNESS_HEADS": heads,
         "_CUTE_HARNESS_EPSILON": eps, "_CUTE_HARNESS_INPUT_SCALE": 1.0 / FP8_MAX,
         "_CUTE_HARNESS_NORM_SCALE": 1.0 / 64.0, "_CUTE_HARNESS_QKV_SCALE": 1.0 / 64.0,
         "_CUTE_HARNESS_CONTEXT_SCALE": 1.0 / 64.0,
         "_CUTE_HARNESS_WEIGHT_H_SCALE": hidden ** -0.5 / FP8_MAX,
         "_CUTE_HARNESS_WEIGHT_MLP_SCALE": mlp ** -0.5 / FP8_MAX}
    d.update(extra)
    return d


TASKS: Dict[str, dict] = {
    "level1_01_square_matrix_multiplication_fp8": dict(
        entry="square_gemm", family="gemm", epilogue={}, seed=20260726,
        consts={"_CUTE_HARNESS_INPUT_SCALE": 1.0 / FP8_MAX}, shape=(4096, 4096, 4096)),
    "level2_76_gemm_add_relu_fp8": dict(
        entry="gemm_add_relu", family="gemm", epilogue={"bias": True, "act": "relu"},
        seed=20260726, consts=_gemm_consts(8192), shape=(1024, 8192, 8192)),
    "level2_09_matmul_subtract_multiply_relu_fp8": dict(
        entry="matmul_subtract_multiply_relu", family="gemm",
        epilogue={"bias": True, "pre_mul": 1.5, "pre_add": -3.0, "act": "relu"},
        seed=20260727, consts=_gemm_consts(8192), shape=(1024, 8192, 8192)),
    "level2_12_gemm_multiply_leaky_relu_fp8": dict(
        entry="gemm_multiply_leaky_relu", family="gemm",
        epilogue={"bias": True, "pre_mul": 2.0, "act": "leaky_relu", "act_param": 0.1},
        seed=20260727, consts=_gemm_consts(8192), shape=(1024, 8192, 8192)),
    "level2_14_gemm_divide_sum_scaling_fp8": dict(
        entry="gemm_divide_sum_scaling", family="gemm",
        epilogue={"post_mul": 0.5, "rowsum": True, "out_scale": 1 / 1.5},
        seed=20260727, consts=_gemm_consts(8192), shape=(1024, 8192, 8192)),
    "level2_40_matmul_scaling_residual_add_fp8": dict(
        entry="matmul_scaling_residual_add", family="gemm",
        epilogue={"bias": True, "pre_mul": 1.5}, seed=20260727, consts=_gemm_consts(8192),
        shape=(1024, 8192, 8192)),
    "level2_63_gemm_relu_divide_fp8": dict(
        entry="gemm_relu_divide", family="gemm",
        epilogue={"bias": True, "act": "relu", "post_mul": 0.5}, seed=20260727,
        consts=_gemm_consts(8192), shape=(1024, 8192, 8192)),
    "model_gpt2_small_qkv_projection_fp8": dict(
        entry="gpt2_qkv_projection", family="gemm", epilogue={"bias": True},
        seed=20260731, consts={"_CUTE_HARNESS_SCALE_X": 1.0 / FP8_MAX,
                               "_CUTE_HARNESS_SCALE_W": 768 ** -0.5 / FP8_MAX},
        shape=(8192, 2304, 768)),
    "model_gpt2_small_transformer_block_fp8": dict(
        entry="gpt2_transformer_block", family="gpt2", seed=20260801,
        consts=_block_consts(768, 12, 3072, 1e-5, _CUTE_HARNESS_MLP_SCALE=1.0 / 64.0,
                             _CUTE_HARNESS_TOKENS=128)),
    "model_qwen35_4b_vision_block_fp8": dict(
        entry="qwen35_vision_block", family="vision", seed=20260801,
        consts=_block_consts(1024, 16, 4096, 1e-6, _CUTE_HARNESS_MLP_SCALE=1.0 / 64.0,
                             _CUTE_HARNESS_TOKENS=128)),
    "model_qwen35_4b_full_attention_block_fp8": dict(
        entry="qwen35_full_attention_block", family="qwen", seed=20260801,
        consts=_block_consts(
            2560, 16, 9216, 1e-6, _CUTE_HARNESS_KV_HEADS=4, _CUTE_HARNESS_HEAD_DIM=256,
            _CUTE_HARNESS_ROTARY=64, _CUTE_HARNESS_TOKENS=128,
            _CUTE_HARNESS_MLP_PROJECTION_SCALE=1.0 / 64.0,
            _CUTE_HARNESS_MLP_ACTIVATION_SCALE=1.0 / 32.0,
            _CUTE_HARNESS_WEIGHT_CONTEXT_SCALE=4096 ** -0.5 / FP8_MAX)),
    "level1_40_layer_norm_fp8": dict(
        entry="layer_norm", family="layer_norm", seed=20260726,
        consts={"_CUTE_HARNESS_INPUT_SCALE": 1.0 / FP8_MAX, "_CUTE_HARNESS_EPSILON": 1.0e-5,
                "_CUTE_HARNESS_BATCH_SIZE": 16,
                "_CUTE_HARNESS_ROW_SIZE": 64 * 256 * 256}),
}


# ------------------------------------------------------------------------- entry points
def _gemm_entry(name: str, epilogue: dict, ns: dict) -> Callable:
    from . import ops
    sa = ns.get("_CUTE_HARNESS_SCALE_A", ns.get("_CUTE_HARNESS_SCALE_X",
                                                  ns.get("_CUTE_HARNESS_INPUT_SCALE")))
    sb = ns.get("_CUTE_HARNESS_SCALE_B", ns.get("_CUTE_HARNESS_SCALE_W",
                                                  ns.get("_CUTE_HARNESS_INPUT_SCALE")))
    kw = {k: v for k, v in epilogue.items() if k != "bias"}

    def entry(matrix_a, matrix_b_nk, *rest):
        output = rest[-1]
        bias = rest[0] if (epilogue.get("bias") and len(rest) == 2) else None
        if kw.get("rowsum"):
            output.zero_()  # the row sums accumulate into the output
            ops.gemm_fp8(_e(matrix_a), _e(matrix_b_nk), scale_a=sa, scale_b=sb,
                         out=output.view(-1), **kw)
        else:
            ops.gemm_fp8(_e(matrix_a), _e(matrix_b_nk), scale_a=sa, scale_b=sb, bias=bias,
                         out=output, out_dtype=output.dtype, **kw)

    entry.__name__ = entry.__qualname__ = name
    return entry


class _BlockCache:
    """One block object per weight set (keyed by the weights' device addresses): the
    evaluator calls the entry repeatedly with the same tensors."""

    def __init__(self, build):
        self.build = build
        self.key = None
        self.blk = None

    def get(self, tensors, output):
        key = tuple(t.data_ptr() for t in tensors) + (output.data_ptr(),)
        if key != self.key:
            self.blk = self.build()
            self.key = key
        return self.blk


def _gpt2_entry(name: str, ns: dict, vision: bool) -> Callable:
    from . import blocks
    hs, ms = _c(ns, "WEIGHT_H_SCALE"), _c(ns, "WEIGHT_MLP_SCALE")
    heads, eps, in_scale = _c(ns, "HEADS"), _c(ns, "EPSILON"), _c(ns, "INPUT_SCALE")
    state = {}

    def entry(*args):
        (hidden, ln1_w, ln1_b, qkv_w, qkv_b, out_w, out_b, ln2_w, ln2_b, fc_w, fc_b,
         proj_w, proj_b) = args[:13]
        cos, sin = (args[13], args[14]) if vision else (None, None)
        output = args[-1]

        def build():
            w = SimpleNamespace(
                heads=heads, eps=eps, norm_scale=_c(ns, "NORM_SCALE"),
                qkv_scale=_c(ns, "QKV_SCALE"), ctx_scale=_c(ns, "CONTEXT_SCALE"),
                mlp_scale=ns.get("_CUTE_HARNESS_MLP_SCALE", 1.0 / 64.0),
                qkv_w=_e(qkv_w), qkv_s=hs, qkv_b=qkv_b, out_w=_e(out_w), out_s=hs,
                out_b=out_b, fc_w=_e(fc_w), fc_s=hs, fc_b=fc_b, proj_w=_e(proj_w), proj_s=ms,
                proj_b=proj_b, ln1_w=ln1_w, ln1_b=ln1_b, ln2_w=ln2_w, ln2_b=ln2_b)
            blk = blocks.GPT2Block(w, batch=1, seq=hidden.shape[0], residual_dtype=torch.float32,
                                   out_dtype=output.dtype, device=hidden.device,
                                   causal=not vision, rope_cos=cos, rope_sin=sin)
            blk.out = output  # the last GEMM stores straight into the evaluator's buffer
            return blk

        cache = state.setdefault("c", _BlockCache(build))
        blk = cache.get(args[:15] if vision else args[:13], output)
        blk.forward(_e(hidden), in_scale)

    entry.__name__ = entry.__qualname__ = name
    return entry


def _qwen_entry(name: str, ns: dict) -> Callable:
    from . import blocks
    hs = _c(ns, "WEIGHT_H_SCALE")
    state = {}

    def entry(*args):
        (hidden, in_norm, q_norm, k_norm, q_gate, k_w, v_w, out_w, post_norm, gate_w, up_w,
         down_w, cos, sin) = args[:14]
        output = args[-1]

        def build():
            w = SimpleNamespace(
                heads=_c(ns, "HEADS"), kv_heads=_c(ns, "KV_HEADS"), head_dim=_c(ns, "HEAD_DIM"),
                rotary_dim=_c(ns, "ROTARY"), interleaved=True, eps=_c(ns, "EPSILON"),
                norm_scale=_c(ns, "NORM_SCALE"), qkv_scale=_c(ns, "QKV_SCALE"),
                ctx_scale=_c(ns, "CONTEXT_SCALE"),
                mlp_proj_scale=_c(ns, "MLP_PROJECTION_SCALE"),
                mlp_act_scale=_c(ns, "MLP_ACTIVATION_SCALE"),
                q_w=_e(q_gate), q_s=hs, gate_w=None, gate_s=1.0, k_w=_e(k_w), k_s=hs,
                v_w=_e(v_w), v_s=hs, o_w=_e(out_w), o_s=_c(ns, "WEIGHT_CONTEXT_SCALE"),
                in_norm_w=in_norm, q_norm_w=q_norm, k_norm_w=k_norm, cos=cos, sin=sin,
                post_norm_w=post_norm, mlp_gate_w=_e(gate_w), mlp_gate_s=hs,
                mlp_up_w=_e(up_w), mlp_up_s=hs, mlp_down_w=_e(down_w),
                mlp_down_s=_c(ns, "WEIGHT_MLP_SCALE"))
            blk = blocks.QwenBlock(w, batch=1, seq=hidden.shape[0],
                                   residual_dtype=torch.float32, out_dtype=output.dtype,
                                   device=hidden.device)
            blk.out = output
            return blk

        cache = state.setdefault("c", _BlockCache(build))
        blk = cache.get(args[:14], output)
        blk.forward(_e(hidden), _c(ns, "INPUT_SCALE"))

    entry.__name__ = entry.__qualname__ = name
    return entry


def _layer_norm_entry(name: str, ns: dict) -> Callable:
    from . import ops
    scale, eps = _c(ns, "INPUT_SCALE"), _c(ns, "EPSILON")

    def entry(input_tensor, output):
        ops.layer_norm_rows(_e(input_tensor), out=output, x_scale=scale, eps=eps)

    entry.__name__ = entry.__qualname__ = name
    return entry


def make_entry(task_id: str, ns: Optional[dict] = None) -> Callable:
    """The task's entry point (its ``entrypoint_jit`` name and positional signature) on the
    b200fp8 kernels.  ``ns`` is the evaluator's namespace (its ``_CUTE_HARNESS_*``
    constants); without it the task's published constants are used."""
    spec = TASKS[task_id]
    consts = dict(spec["consts"])
    if ns is not None:
        consts.update({k: v for k, v in ns.items() if k.startswith("_CUTE_HARNESS_")})
    fam = spec["family"]
    if fam == "gemm":
        return _gemm_entry(spec["entry"], spec["epilogue"], consts)
    if fam in ("gpt2", "vision"):
        return _gpt2_entry(spec["entry"], consts, vision=fam == "vision")
    if fam == "qwen":
        return _qwen_entry(spec["entry"], consts)
    if fam == "layer_norm":
        return _layer_norm_entry(spec["entry"], consts)
    raise KeyError(task_id)


def success_pattern(task_id: str) -> str:
    """The task's ``validation.success_pattern``: the evaluators print ``task=<name>`` with
    the ``_fp8`` suffix dropped for the KernelBench-derived tasks."""
    name = task_id if task_id.startswith("model_") else task_id.rsplit("_fp8", 1)[0]
    return r"(?m)^task=" + name + r" .* PASS$"


def task_work(task_id: str) -> dict:
    """Algorithmic FLOPs and compulsory HBM bytes of one call (roofline of the reporting)."""
    spec = TASKS[task_id]
    fam = spec["family"]
    if fam == "gemm":
        m, n, k = spec["shape"]
        out_b = 4 * (m if spec["epilogue"].get("rowsum") else m * n)
        return {"flops": 2.0 * m * n * k, "bytes": float(m * k + n * k + out_b),
                "bound": "tensor"}
    if fam == "layer_norm":
        c = spec["consts"]
        n = c["_CUTE_HARNESS_BATCH_SIZE"] * c["_CUTE_HARNESS_ROW_SIZE"]
        return {"flops": 0.0, "bytes": float(n * (1 + 4)), "bound": "hbm"}
    c = spec["consts"]
    t, d, h = 128, c["_CUTE_HARNESS_HIDDEN"], c["_CUTE_HARNESS_HEADS"]
    if fam in ("gpt2", "vision"):
        mlp = 3072 if fam == "gpt2" else 4096
        fl = 2.0 * t * (4 * d * d + 2 * d * mlp) + (2 if fam == "gpt2" else 4) * h * t * t * (d // h)
        by = 4 * d * d + 2 * d * mlp + 12.0 * t * d
    else:
        hd, hk, inter = 256, 4, 9216
        fl = (2.0 * t * d * (2 * h * hd + 2 * hk * hd) + 2.0 * t * h * hd * d +
              2.0 * t * d * 3 * inter + 2.0 * h * t * t * hd)
        by = d * (2 * h * hd + 2 * hk * hd) + h * hd * d + 3.0 * d * inter + 12.0 * t * d
    return {"flops": fl, "bytes": by, "bound": "tensor"}


# ------------------------------------------------------------------------- evaluator runner
class _Wrapped:
    """What ``from_dlpack(t)`` returns under the runner: ``mark_layout_dynamic`` hands back
    the torch tensor the evaluator wrapped."""

    def __init__(self, t):
        self.t = t

    def mark_layout_dynamic(self, leading_dim=None):
        return self.t


def _dsl_shims(compile_fn) -> Dict[str, types.ModuleType]:
    cutlass = types.ModuleType("cutlass")
    cutlass.Float8E4M3FN = type("Float8E4M3FN", (), {})
    cute = types.ModuleType("cutlass.cute")
    cute.compile = compile_fn
    runtime = types.ModuleType("cutlass.cute.runtime")
    runtime.from_dlpack = lambda t, **kw: _Wrapped(t)
    utils = types.ModuleType("cutlass.utils")

    def create_fp8(storage, dtype, leading_dim, source):
        storage.copy_(source.to(E4M3).view(torch.uint8))
        return storage

    utils.create_cute_tensor_for_fp8 = create_fp8
    cutlass.cute, cute.runtime, cutlass.utils = cute, runtime, utils
    return {"cutlass": cutlass, "cutlass.cute": cute, "cutlass.cute.runtime": runtime,
            "cutlass.utils": utils}


def run_reference_evaluator(task_id: str, reference_root: str, *, seed: Optional[int] = None,
                            warmup: int = 2, repeats: int = 5,
                            entry_factory: Optional[Callable] = None) -> dict:
    """Executes ``tasks/<task_id>/starter.py``'s own evaluator from the reference checkout
    at ``reference_root`` with this library's entry point as the candidate, in this
    process, on the current CUDA device.  Returns the response record that the reference's
    acceptance step reads: ``stdout`` (with the evaluator's PASS line), ``exit_code``,
    ``success``, ``timed_out`` and ``error``.  ``entry_factory(task_id, ns)`` replaces
    ``make_entry`` (tests use it to wrap the entry)."""
    spec = TASKS[task_id]
    starter = os.path.join(reference_root, "tasks", task_id, "starter.py")
    with open(starter, encoding="utf-8") as f:
        text = f.read()
    if MARKER not in text:
        raise ValueError(f"{starter} has no evaluator marker")
    suffix = text.split(MARKER, 1)[1].rstrip()
    if not suffix.endswith("main()"):
        raise ValueError("evaluator suffix must end with main()")
    factory = entry_factory or make_entry
    holder = {}

    def compile_fn(fn, *args):
        return holder["entry"]

    mods = _dsl_shims(compile_fn)
    real_import = builtins.__import__

    def _import(name, globals=None, locals=None, fromlist=(), level=0):
        if name == "cutlass" or name.startswith("cutlass."):
            return mods[name] if fromlist else mods["cutlass"]
        return real_import(name, globals, locals, fromlist, level)

    ns = {"__builtins__": dict(builtins.__dict__, __import__=_import),
          "__name__": "__cute_harness_eval__",
          "_CUTE_HARNESS_SEED": spec["seed"] if seed is None else seed,
          "_CUTE_HARNESS_WARMUP": warmup, "_CUTE_HARNESS_REPEATS": repeats,
          spec["entry"]: None}
    out = io.StringIO()
    rec = {"task_id": task_id, "stdout": "", "exit_code": 1, "success": False,
           "timed_out": False, "error": None}
    try:
        exec(compile(suffix[: -len("main()")], starter + "::evaluator", "exec"), ns)
        holder["entry"] = factory(task_id, ns)
        with contextlib.redirect_stdout(out):
            ns["main"]()
        rec.update(exit_code=0, success=True)
    except Exception as exc:  # the evaluator's RuntimeError("validation failed: ...") etc.
        rec["error"] = f"{type(exc).__name__}: {exc}"
    rec["stdout"] = out.getvalue()
    return rec


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m b200fp8.harness", description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("list")
    rp = sub.add_parser("run")
    rp.add_argument("task")
    rp.add_argument("--reference", default=os.environ.get("B2F_REFERENCE"),
                    help="reference checkout holding tasks/<task>/starter.py")
    rp.add_argument("--seed", type=int, default=None)
    rp.add_argument("--warmup", type=int, default=2)
    rp.add_argument("--repeats", type=int, default=5)
    rp.add_argument("--record", default=None, help="write the response record (JSON) here")
    args = ap.parse_args(argv)
    if args.cmd == "list":
        for tid, spec in TASKS.items():
            print(f"{tid}\t{spec['entry']}")
        return 0
    if not args.reference:
        ap.error("run needs --reference PATH (or B2F_REFERENCE)")
    rec = run_reference_evaluator(args.task, args.reference, seed=args.seed,
                                  warmup=args.warmup, repeats=args.repeats)
    sys.stdout.write(rec["stdout"])
    if rec["error"]:
        print(rec["error"], file=sys.stderr)
    if args.record:
        from .reporting import benchmark_record
        rec["benchmark"] = benchmark_record(args.task, rec["stdout"])
        with open(args.record, "w") as f:
            json.dump(rec, f, indent=2)
    return rec["exit_code"]


if __name__ == "__main__":
    sys.exit(main())
