#!/usr/bin/env python
"""Benchmark of the b200fp8 hot path: one JSON line on rank 0.

Headline (every N): BASELINE configs[4], the Qwen-style FP8 gated full-attention block at
B4 x S2048 (hidden 2560, 32 q / 8 kv heads x 128, RoPE theta 1e6, separate gate
projection), one CUDA graph per forward, bf16 residual.  Under torchrun the SAME global
batch is split over the ranks (strong scaling): whole sequences per batch group first, the
rest by heads (column-parallel q / gate / k / v, row-parallel o-projection, one NCCL SUM
all-reduce of the bf16 output per head group).

With ``--workload all`` (the default) the line also carries a ``workloads`` list with every
other BASELINE config measured in the same run, each with its roofline, e2e, parity check
of the timed output and (N=1) CPU baseline:
  N=1: GEMM+bias+ReLU 128x8192x8192; square GEMM n = 4096 / 8192 / 16384
       (configs[1]); residual RMSNorm + amax quant 16384x4096; GPT-2 block
       B8 x S1024; the reference tasks' long-row LayerNorm (level1_40,
       [16 x 4194304]) and gated-residual GEMM (2048 x 4096 x 4096).
  N>1: the same global problems split over the ranks (strong scaling): GEMM 8192^3 along N
       (no communication), norm by rows (one f32 MAX all-reduce), GPT-2 by sequences (no
       communication), Qwen with every rank in one head group (tp = N).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload all|qwen|gpt2|norm|gemm|gemm_bias_relu] [--n 8192]

--impl reference times the reference's own computation of the headline on the host cores:
the Torch math of the Qwen block evaluator
(tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-416), restated on CPU by
oracle.blocks.qwen_block, one sequence of the batch per step.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "airi-summer-kernel-evo_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "basis": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "basis": "fallback"}


PEAKS = _peaks()
FP8_PEAK = 2.0 * PEAKS["bf16_tflops"]        # e4m3 dense rate is 2x bf16
BF16_PEAK = PEAKS["bf16_tflops"]
# attention: QK^T in e4m3 and P.V in bf16, half of the FLOPs each
ATTN_PEAK = 2.0 / (1.0 / FP8_PEAK + 1.0 / BF16_PEAK)
HBM = PEAKS["hbm_gbs"]


class ClockSampler:
    """nvidia-smi clock / throttle sampling over the whole run; ``window`` summarises the
    samples taken between two host timestamps (a workload's soak + timed region)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu=timestamp,{self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                self.rows.append({"t": ts, "sm": float(parts[2]), "max": float(parts[3]),
                                  "hw": parts[6], "hwt": parts[7], "swt": parts[8],
                                  "pcap": parts[9]})
            except ValueError:
                continue

    def window(self, t0: float, t1: float):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r for r in self.rows if t0 - 0.15 <= r["t"] <= t1 + 0.15]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        under = [r for r in rows if r["sm"] > 0.5 * r["max"]] or rows
        reasons = set()
        for r in under:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key] == "Active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in under),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": sorted(reasons),
                "samples": len(under)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _threads() -> int:
    return len(os.sched_getaffinity(0))


def _fp8_inputs(shape, gen, scale=1.0):
    x = torch.randn(shape, generator=gen, dtype=torch.float32) * scale
    amax = float(x.abs().max())
    s = amax / 448.0
    return (x / s).to(torch.float8_e4m3fn), s


def _close_bf16(out_f32_cpu, ref, k):
    """bf16 output within one bf16 rounding (2^-7 relative, with margin for the f32
    accumulation order) of the f64-accumulated oracle."""
    err = (out_f32_cpu - ref).abs()
    tol = ref.abs() * 2.0 ** -7 + 1e-5 * math.sqrt(k)
    bad = int((err > tol).sum())
    return {"status": "pass" if bad == 0 else "fail", "max_abs_err": float(err.max()),
            "mismatches": bad, "bar": "|err| <= 2^-7 |ref| + 1e-5 sqrt(K)"}


def _e4m3_codes(t):
    u = t.view(torch.uint8).to(torch.int32)
    mag = u & 0x7F
    return torch.where(u & 0x80 != 0, -mag, mag)


# ------------------------------------------------------------------ workloads
class GemmWorkload:
    """BASELINE configs[1] (square FP8 GEMM, bf16 out) or configs[0] (GEMM+bias+ReLU at
    M=128).  At N>1 the global n x n problem is split along N: rank r computes the column
    block of C from its rows of B (no communication)."""

    scaling = "strong"

    def __init__(self, n: int, rank: int, world: int = 1, bias_relu: bool = False, m=None):
        self.m = m if m is not None else n
        self.k = n
        self.n_global = n
        self.world, self.rank = world, rank
        self.bias_relu = bias_relu
        g = torch.Generator("cpu").manual_seed(20260726 + n)
        xscale = 0.1 if bias_relu else 1.0
        a, self.sa = _fp8_inputs((self.m, self.k), g, xscale)
        b, self.sb = _fp8_inputs((n, self.k), g, xscale)
        bias = (torch.randn((n,), generator=g) * 0.02) if bias_relu else None
        lo, hi = n * rank // world, n * (rank + 1) // world
        self.n = hi - lo
        self.a_cpu, self.b_cpu = a, b[lo:hi].contiguous()
        self.bias_cpu = bias[lo:hi].contiguous() if bias_relu else None
        self.work = 2.0 * self.m * self.n * self.k          # this rank's FLOPs
        self.unit = "TFLOP/s"
        self.bound = "tensor" if self.m > 128 else "hbm"
        self.algo_bytes = float(self.m * self.k + self.n * self.k + self.m * self.n * 2 +
                                (4 * self.n if bias_relu else 0))
        per_set = self.m * self.k + self.n * self.k
        self.nsets = 1 if per_set >= 2 * L2_BYTES else min(8, -(-3 * L2_BYTES // per_set))
        self.sets = [(self.a_cpu.cuda(), self.b_cpu.cuda()) for _ in range(self.nsets)]
        self.bias = self.bias_cpu.cuda() if bias_relu else None
        self.out = torch.empty((self.m, self.n), device="cuda", dtype=torch.bfloat16)
        self.i = 0
        self.last_set = 0
        self.name = (f"gemm_bias_relu_fp8_{self.m}x{n}x{n}" if bias_relu
                     else f"square_gemm_fp8_{n}")
        self.launches = 1

    def kernel(self):
        from b200fp8 import ops
        if self.bias_relu:
            return "gemm_fp8_kernel<128> (2 K slices)" if ops._auto_split(
                self.m, self.n, self.k, "cuda") else "gemm_fp8_kernel<128>"
        if self.m > 128 and ((self.m + 255) // 256) * ((self.n + 255) // 256) >= 74 and self.k >= 2048:
            return "gemm_fp8_pair_kernel"
        return "gemm_fp8_kernel"

    def config(self):
        c = {"workload": f"{self.name} M={self.m} N={self.n_global} K={self.k} e4m3->bf16"
                         + (" +bias, ReLU" if self.bias_relu else ""),
             "M": self.m, "N": self.n_global, "K": self.k, "out_dtype": "bf16",
             "inputs": "N(0,1)" + ("x0.1" if self.bias_relu else "") + " amax-scaled e4m3",
             "l2": (f"{self.nsets} rotating input sets "
                    f"({self.nsets * (self.m * self.k + self.n * self.k) / 2**20:.0f} MiB) > 126 MiB L2")}
        return c

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        return (f"N-split x{self.world}: each rank computes {self.n} of {self.n_global} output "
                "columns from its rows of B (no communication)")

    def step(self):
        from b200fp8 import ops
        self.last_set = self.i % self.nsets
        a, b = self.sets[self.last_set]
        self.i += 1
        if self.bias_relu:
            ops.gemm_fp8(a, b, scale_a=self.sa, scale_b=self.sb, bias=self.bias, act="relu",
                         out=self.out)
        else:
            ops.gemm_fp8(a, b, scale_a=self.sa, scale_b=self.sb, out=self.out)
        return 1

    def roofline(self, per_launch_ms):
        if self.bound == "tensor":
            return self.kernel(), self.work / 1e12, "TFLOP/s", FP8_PEAK, (
                f"2 x {PEAKS['basis']} cuBLAS bf16 burst ({BF16_PEAK} TFLOP/s); e4m3 dense "
                "rate is 2x bf16")
        return self.kernel(), self.algo_bytes / 1e9, "GB/s", HBM, (
            f"{PEAKS['basis']} HBM copy bandwidth")

    def parity(self):
        """Rows of the output of the last timed step against the f64 oracle."""
        from oracle import gemm as og
        rows = sorted({0, 1, 77, self.m // 2, self.m - 1} |
                      ({255, 256, self.m - 129} if self.m > 512 else set()))
        ref = og.gemm_epilogue(self.a_cpu[rows], self.b_cpu, self.sa, self.sb,
                               bias=self.bias_cpu, act="relu" if self.bias_relu else None)
        r = _close_bf16(self.out[rows].float().cpu(), ref, self.k)
        r["check"] = f"{len(rows)} rows x all {self.n} columns of the timed output vs f64 oracle"
        return r

    # ---------------- end-to-end through the public API with host buffers
    def e2e_setup(self):
        self.h_a = self.a_cpu.view(torch.uint8).pin_memory()
        self.h_b = self.b_cpu.view(torch.uint8).pin_memory()
        self.h_out = torch.empty((self.m, self.n), dtype=torch.bfloat16).pin_memory()
        self.d_a = [torch.empty_like(self.h_a, device="cuda") for _ in range(2)]
        self.d_b = [torch.empty_like(self.h_b, device="cuda") for _ in range(2)]
        self.d_out = [torch.empty((self.m, self.n), dtype=torch.bfloat16, device="cuda")
                      for _ in range(2)]

    def e2e_h2d(self, slot):
        self.d_a[slot].copy_(self.h_a, non_blocking=True)
        self.d_b[slot].copy_(self.h_b, non_blocking=True)

    def e2e_compute(self, slot):
        from b200fp8 import ops
        a = self.d_a[slot].view(torch.float8_e4m3fn)
        b = self.d_b[slot].view(torch.float8_e4m3fn)
        if self.bias_relu:
            ops.gemm_fp8(a, b, scale_a=self.sa, scale_b=self.sb, bias=self.bias, act="relu",
                         out=self.d_out[slot])
        else:
            ops.gemm_fp8(a, b, scale_a=self.sa, scale_b=self.sb, out=self.d_out[slot])

    def e2e_d2h(self, slot):
        self.h_out.copy_(self.d_out[slot], non_blocking=True)

    def e2e_bytes(self):
        return self.h_a.numel() + self.h_b.numel(), self.h_out.numel() * 2

    def e2e_release(self):
        del self.d_a, self.d_b, self.d_out

    def cpu_sample(self, target_s: float):
        from oracle import gemm as og
        threads = _threads()
        torch.set_num_threads(threads)
        rows = 16
        while True:
            t0 = time.perf_counter()
            v = og.cpu_fast_scaled_mm(self.a_cpu[:rows], self.b_cpu, self.sa, self.sb)
            if self.bias_relu:
                v = torch.relu(v + self.bias_cpu)
            v.to(torch.bfloat16)
            t = time.perf_counter() - t0
            if t > target_s / 4 or rows >= self.m:
                break
            rows = min(self.m, rows * 4)
        return {"value": 2.0 * rows * self.n * self.k / t / 1e12, "unit": "TFLOP/s",
                "cores": threads, "kind": "port",
                "sample": f"{rows} of {self.m} rows of the same GEMM "
                          f"({2.0 * rows * self.n * self.k / 1e9:.1f} GFLOP), f32 dequantise + "
                          f"torch.matmul on CPU, {t:.2f} s"}


class NormWorkload:
    """residual-add + RMSNorm + per-tensor amax e4m3 quantisation,
    bf16 x / residual [16384, 4096], gamma 1+N(0,0.02), eps 1e-6.  At N>1 the rows are
    split over the ranks and one MAX all-reduce of the f32 amax joins the two passes."""

    unit = "GB/s"
    bound = "hbm"
    scaling = "strong"
    name = "residual_rmsnorm_amax_quant_16384x4096"
    launches = 2

    def __init__(self, rank: int, world: int = 1, rows: int = 16384, cols: int = 4096):
        g = torch.Generator("cpu").manual_seed(20260731)
        self.world, self.rank = world, rank
        self.sharded = None
        if world > 1:
            from b200fp8.sharding import RowShardedNorm
            self.sharded = RowShardedNorm()
        self.rows_global, self.cols = rows, cols
        x = torch.randn((rows, cols), generator=g).to(torch.bfloat16)
        r = torch.randn((rows, cols), generator=g).to(torch.bfloat16)
        self.g_cpu = (1 + 0.02 * torch.randn((cols,), generator=g)).to(torch.bfloat16)
        lo, hi = rows * rank // world, rows * (rank + 1) // world
        self.rows = hi - lo
        self.x_full, self.r_full = x, r
        self.x_cpu, self.r_cpu = x[lo:hi].contiguous(), r[lo:hi].contiguous()
        self.x, self.r, self.gamma = self.x_cpu.cuda(), self.r_cpu.cuda(), self.g_cpu.cuda()
        self.h = torch.empty_like(self.x)
        self.q = torch.empty((self.rows, cols), device="cuda", dtype=torch.float8_e4m3fn)
        self.amax = torch.zeros(1, device="cuda")
        self.scale = torch.zeros(1, device="cuda")
        # compulsory traffic: read x, r; write h (bf16) and q (e4m3)
        self.work = float(self.rows * cols * (2 + 2 + 2 + 1))
        self.algo_bytes = self.work

    def config(self):
        return {"workload": f"residual RMSNorm + amax e4m3 quant [{self.rows_global} x "
                            f"{self.cols}] bf16", "rows": self.rows_global, "cols": self.cols,
                "eps": 1e-6, "l2": "inputs 268 MB > 126 MB L2"}

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        return (f"row-split x{self.world}: each rank {self.rows} of {self.rows_global} rows; "
                "one f32 MAX all-reduce (NCCL) of the amax between pass 1 and pass 2")

    def step(self):
        from b200fp8 import ops
        kw = dict(residual=self.r, h_out=self.h, q_out=self.q, amax=self.amax,
                  scale_out=self.scale)
        if self.sharded is not None:
            self.sharded(self.x, self.gamma, **kw)
        else:
            ops.norm_quant(self.x, self.gamma, **kw)
        return 2

    def roofline(self, per_launch_ms):
        return ("norm_stream_kernel (stats + apply passes)", self.algo_bytes / 1e9, "GB/s", HBM,
                f"{PEAKS['basis']} HBM copy bandwidth")

    def parity(self):
        """h bit-exact, the scale against the oracle's global amax, q within one e4m3 code
        (<= 0.5 % of the codes may differ by one: f32 reduction order of the row norms)."""
        from oracle import norm as onorm
        q_ref, s_ref, h_ref = onorm.residual_rmsnorm_amax_quant(self.x_full, self.r_full,
                                                                self.g_cpu)
        lo = self.rows_global * self.rank // self.world
        h_ok = torch.equal(self.h.cpu(), h_ref[lo:lo + self.rows])
        s = float(self.scale.cpu())
        s_ok = abs(s - s_ref) <= 1e-6 * s_ref
        d = (_e4m3_codes(self.q.cpu()) - _e4m3_codes(q_ref[lo:lo + self.rows])).abs()
        q_ok = int(d.max()) <= 1 and float((d > 0).float().mean()) <= 0.005
        return {"status": "pass" if (h_ok and s_ok and q_ok) else "fail",
                "h_bit_exact": h_ok, "scale_rel_err": abs(s - s_ref) / s_ref,
                "q_max_code_diff": int(d.max()), "q_frac_differing": float((d > 0).float().mean()),
                "check": "all rows of the timed output vs the CPU oracle (global amax)"}

    def e2e_setup(self):
        self.hx, self.hr = self.x_cpu.pin_memory(), self.r_cpu.pin_memory()
        self.hq = torch.empty((self.rows, self.cols), dtype=torch.uint8).pin_memory()
        self.hh = torch.empty((self.rows, self.cols), dtype=torch.bfloat16).pin_memory()
        self.sx = [self.x, torch.empty_like(self.x)]
        self.sr = [self.r, torch.empty_like(self.r)]
        self.sh = [self.h, torch.empty_like(self.h)]
        self.sq = [self.q, torch.empty_like(self.q)]

    def e2e_h2d(self, slot):
        self.sx[slot].copy_(self.hx, non_blocking=True)
        self.sr[slot].copy_(self.hr, non_blocking=True)

    def e2e_compute(self, slot):
        from b200fp8 import ops
        kw = dict(residual=self.sr[slot], h_out=self.sh[slot], q_out=self.sq[slot],
                  amax=self.amax, scale_out=self.scale)
        if self.sharded is not None:
            self.sharded(self.sx[slot], self.gamma, **kw)
        else:
            ops.norm_quant(self.sx[slot], self.gamma, **kw)

    def e2e_d2h(self, slot):
        self.hq.copy_(self.sq[slot].view(torch.uint8), non_blocking=True)
        self.hh.copy_(self.sh[slot], non_blocking=True)

    def e2e_bytes(self):
        n = self.rows * self.cols
        return 4 * n, 3 * n

    def e2e_release(self):
        del self.sx, self.sr, self.sh, self.sq

    def cpu_sample(self, target_s: float):
        from oracle import norm as onorm
        threads = _threads()
        torch.set_num_threads(threads)
        rows = 256
        while True:
            t0 = time.perf_counter()
            onorm.residual_rmsnorm_amax_quant(self.x_cpu[:rows], self.r_cpu[:rows], self.g_cpu)
            t = time.perf_counter() - t0
            if t > target_s / 4 or rows >= self.rows:
                break
            rows = min(self.rows, rows * 4)
        return {"value": rows * self.cols * 7 / t / 1e9, "unit": "GB/s", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {self.rows} rows, oracle residual RMSNorm + amax quant "
                          f"on CPU, {t:.2f} s"}


class LayerNormRowsWorkload:
    """The reference task level1_40 (tasks/level1_40_layer_norm_fp8): LayerNorm over each of
    16 rows of 4,194,304 e4m3 values read at 1/448, eps 1e-5, f32 output
    (b2f_layer_norm_rows: every row split over 64 CTAs).  Inputs U(0,1) * 448 as the task's
    evaluator draws them, from a CPU generator."""

    unit = "GB/s"
    bound = "hbm"
    scaling = "strong"
    name = "layer_norm_rows_16x4194304"
    launches = 2

    def __init__(self, rank: int, world: int = 1, rows: int = 16, cols: int = 64 * 256 * 256):
        g = torch.Generator("cpu").manual_seed(20260726)
        self.world, self.rank = world, rank
        self.rows, self.cols = rows, cols
        self.x_cpu = (torch.rand((rows, cols), generator=g) * 448.0).to(torch.float8_e4m3fn)
        self.x = self.x_cpu.cuda()
        self.out = torch.empty((rows, cols), device="cuda")
        self.work = float(rows * cols * (1 + 4))
        self.algo_bytes = self.work

    def config(self):
        return {"workload": f"layer norm [{self.rows} x {self.cols}] e4m3 (1/448) -> f32",
                "rows": self.rows, "cols": self.cols, "eps": 1e-5,
                "l2": "output 268 MB > 126 MB L2 (the 67 MB input is re-read from L2 by "
                      "the second pass)"}

    def parallelism(self):
        return "single GPU"

    def step(self):
        from b200fp8 import ops
        ops.layer_norm_rows(self.x, out=self.out, x_scale=1 / 448.0, eps=1e-5)
        return 2

    def roofline(self, per_launch_ms):
        return ("ln_rows_stats_kernel + ln_rows_apply_kernel", self.algo_bytes / 1e9, "GB/s",
                HBM, f"{PEAKS['basis']} HBM copy bandwidth")

    def parity(self):
        from oracle import norm as onorm
        ref = onorm.layer_norm_rows(self.x_cpu.float() / 448.0, 1e-5)
        err = float((self.out.cpu() - ref).abs().max())
        return {"status": "pass" if err <= 0.01 else "fail", "max_abs_err": err,
                "bar": "0.01 (task level1_40's full_max_absolute_error_vs_torch)",
                "check": "every element of the timed output vs the f64 oracle"}

    def e2e_setup(self):
        self.hx = self.x_cpu.view(torch.uint8).pin_memory()
        self.ho = torch.empty((self.rows, self.cols)).pin_memory()
        self.sx = [self.x, torch.empty_like(self.x)]
        self.so = [self.out, torch.empty_like(self.out)]

    def e2e_h2d(self, slot):
        self.sx[slot].view(torch.uint8).copy_(self.hx, non_blocking=True)

    def e2e_compute(self, slot):
        from b200fp8 import ops
        ops.layer_norm_rows(self.sx[slot], out=self.so[slot], x_scale=1 / 448.0, eps=1e-5)

    def e2e_d2h(self, slot):
        self.ho.copy_(self.so[slot], non_blocking=True)

    def e2e_bytes(self):
        return self.rows * self.cols, self.rows * self.cols * 4

    def e2e_release(self):
        del self.sx, self.so

    def cpu_sample(self, target_s: float):
        from oracle import norm as onorm
        threads = _threads()
        torch.set_num_threads(threads)
        t0 = time.perf_counter()
        onorm.layer_norm_rows(self.x_cpu[:2].float() / 448.0, 1e-5)
        t = time.perf_counter() - t0
        return {"value": 2 * self.cols * 5 / t / 1e9, "unit": "GB/s", "cores": threads,
                "kind": "port", "sample": f"2 of {self.rows} rows through the f64 oracle, {t:.2f} s"}


class GatedGemmWorkload:
    """The gated-residual GEMM of cute_kernels/fused_gemm_gated_residual_fp8 (2048 x 4096 x
    4096, out = A.B^T * scale * gate + residual, f32 gate / residual / output), inputs drawn
    as that submission draws them, from a CPU generator."""

    unit = "TFLOP/s"
    bound = "tensor"
    scaling = "strong"
    name = "gemm_gated_residual_fp8_2048x4096x4096"
    launches = 1

    def __init__(self, rank: int, world: int = 1, m=2048, n=4096, k=4096):
        g = torch.Generator("cpu").manual_seed(20260731)
        bound = k ** -0.5
        a = torch.empty((m, k)).uniform_(-1.0, 1.0, generator=g)
        b = torch.empty((n, k)).uniform_(-bound, bound, generator=g)
        self.gate_cpu = torch.randn((m, n), generator=g)
        self.res_cpu = torch.randn((m, n), generator=g)
        self.a_cpu, self.b_cpu = (a * 448.0).to(torch.float8_e4m3fn), (b * (448.0 / bound)).to(torch.float8_e4m3fn)
        self.sa, self.sb = 1 / 448.0, bound / 448.0
        self.m, self.n, self.k = m, n, k
        self.a, self.b = self.a_cpu.cuda(), self.b_cpu.cuda()
        self.gate, self.res = self.gate_cpu.cuda(), self.res_cpu.cuda()
        self.out = torch.empty((m, n), device="cuda")
        self.work = 2.0 * m * n * k
        self.world, self.rank = world, rank

    def config(self):
        return {"workload": f"gated-residual GEMM M={self.m} N={self.n} K={self.k} e4m3 -> f32",
                "M": self.m, "N": self.n, "K": self.k,
                "l2": "A, B, gate, residual and output: 109 MB per call, about the L2 size"}

    def parallelism(self):
        return "single GPU"

    def step(self):
        from b200fp8 import ops
        ops.gemm_fp8(self.a, self.b, scale_a=self.sa, scale_b=self.sb, gate=self.gate,
                     residual=self.res, out=self.out, out_dtype=torch.float32)
        return 1

    def roofline(self, per_launch_ms):
        return ("gemm_fp8 (gate + residual epilogue)", self.work / 1e12, "TFLOP/s", FP8_PEAK,
                f"2 x {PEAKS['basis']} cuBLAS bf16 burst ({BF16_PEAK} TFLOP/s)")

    def parity(self):
        from oracle import gemm as og
        rows = [0, 1, 511, 1024, 2047]
        ref = og.gemm_epilogue(self.a_cpu[rows], self.b_cpu, self.sa, self.sb,
                               gate=self.gate_cpu[rows], residual=self.res_cpu[rows])
        err = float((self.out[rows].cpu() - ref).abs().max())
        return {"status": "pass" if err <= 0.002 else "fail", "max_abs_err": err,
                "bar": "0.002 (the submission's own check)",
                "check": "5 rows x all columns of the timed output vs the f64 oracle"}

    def e2e_setup(self):
        self.ha = self.a_cpu.view(torch.uint8).pin_memory()
        self.hb = self.b_cpu.view(torch.uint8).pin_memory()
        self.hg, self.hr = self.gate_cpu.pin_memory(), self.res_cpu.pin_memory()
        self.ho = torch.empty((self.m, self.n)).pin_memory()
        self.s = [[torch.empty_like(t) for t in (self.a, self.b, self.gate, self.res, self.out)]
                  for _ in range(2)]

    def e2e_h2d(self, slot):
        a, b, gt, r, _ = self.s[slot]
        a.view(torch.uint8).copy_(self.ha, non_blocking=True)
        b.view(torch.uint8).copy_(self.hb, non_blocking=True)
        gt.copy_(self.hg, non_blocking=True)
        r.copy_(self.hr, non_blocking=True)

    def e2e_compute(self, slot):
        from b200fp8 import ops
        a, b, gt, r, o = self.s[slot]
        ops.gemm_fp8(a, b, scale_a=self.sa, scale_b=self.sb, gate=gt, residual=r, out=o,
                     out_dtype=torch.float32)

    def e2e_d2h(self, slot):
        self.ho.copy_(self.s[slot][4], non_blocking=True)

    def e2e_bytes(self):
        mk, nk, mn = self.m * self.k, self.n * self.k, self.m * self.n
        return mk + nk + 8 * mn, 4 * mn

    def e2e_release(self):
        del self.s

    def cpu_sample(self, target_s: float):
        from oracle import gemm as og
        threads = _threads()
        torch.set_num_threads(threads)
        rows = 256
        t0 = time.perf_counter()
        v = og.cpu_fast_scaled_mm(self.a_cpu[:rows], self.b_cpu, self.sa, self.sb)
        v = v * self.gate_cpu[:rows] + self.res_cpu[:rows]
        t = time.perf_counter() - t0
        return {"value": 2.0 * rows * self.n * self.k / t / 1e12, "unit": "TFLOP/s",
                "cores": threads, "kind": "port",
                "sample": f"{rows} of {self.m} rows, f32 dequantise + torch.matmul + gate + "
                          f"residual on CPU, {t:.2f} s"}


def _nq(shape, g, std=0.02):
    w = torch.randn(shape, generator=g) * std
    s = float(w.abs().max()) / 448.0
    return (w / s).to(torch.float8_e4m3fn), s


def _gpt2_weights(g, d=768, mlp=3072):
    """BASELINE configs[3] weights: N(0, 0.02) e4m3 with per-tensor amax scales."""
    from types import SimpleNamespace
    w = SimpleNamespace(heads=12, eps=1e-5, norm_scale=1 / 64.0, qkv_scale=1 / 64.0,
                        ctx_scale=1 / 64.0, mlp_scale=1 / 64.0)
    w.qkv_w, w.qkv_s = _nq((3 * d, d), g)
    w.out_w, w.out_s = _nq((d, d), g)
    w.fc_w, w.fc_s = _nq((mlp, d), g)
    w.proj_w, w.proj_s = _nq((d, mlp), g)
    b = lambda n: torch.randn(n, generator=g) * 0.02  # noqa: E731
    w.qkv_b, w.out_b, w.fc_b, w.proj_b = b(3 * d), b(d), b(mlp), b(d)
    w.ln1_w, w.ln1_b, w.ln2_w, w.ln2_b = 1 + b(d), b(d), 1 + b(d), b(d)
    return w


def _qwen_weights(g, seq, hidden=2560, heads=32, kv_heads=8, hd=128, theta=1e6):
    """BASELINE configs[4] weights: separate q / gate / k / v / o projections, RMSNorm
    weights N(0, 0.02) used as (1 + w), full-dimension RoPE with theta 1e6."""
    from types import SimpleNamespace
    w = SimpleNamespace(heads=heads, kv_heads=kv_heads, head_dim=hd, rotary_dim=hd,
                        interleaved=False, eps=1e-6, norm_scale=1 / 64.0, qkv_scale=1 / 64.0,
                        ctx_scale=1 / 64.0, mlp_proj_scale=1 / 64.0, mlp_act_scale=1 / 32.0,
                        post_norm_w=None, mlp_gate_w=None, mlp_up_w=None, mlp_down_w=None,
                        mlp_gate_s=1.0, mlp_up_s=1.0, mlp_down_s=1.0)
    w.q_w, w.q_s = _nq((heads * hd, hidden), g)
    w.gate_w, w.gate_s = _nq((heads * hd, hidden), g)
    w.k_w, w.k_s = _nq((kv_heads * hd, hidden), g)
    w.v_w, w.v_s = _nq((kv_heads * hd, hidden), g)
    w.o_w, w.o_s = _nq((hidden, heads * hd), g)
    n = lambda k: torch.randn(k, generator=g) * 0.02  # noqa: E731
    w.in_norm_w, w.q_norm_w, w.k_norm_w = n(hidden), n(hd), n(hd)
    pos = torch.arange(seq, dtype=torch.float32)
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    f = pos[:, None] * inv[None, :]
    emb = torch.cat((f, f), dim=-1)
    w.cos, w.sin = emb.cos(), emb.sin()
    return w


def _stage_model(kind, blk):
    """Algorithmic FLOPs, HBM bytes and peak of each stage of one forward of ``blk`` (the
    rank-local block): {stage: (flops, bytes, peak TFLOP/s)}."""
    if kind == "gpt2":
        t, d, m, s, b, h, hd = blk.t, blk.d, blk.mlp, blk.seq, blk.batch, blk.heads, blk.hd
        return {
            "ln1": (0.0, t * d * 3.0, FP8_PEAK),
            "qkv_gemm": (2.0 * t * d * 3 * d, t * d + 3 * d * d + 3 * t * d + 0.0, FP8_PEAK),
            # QKV GEMM writing q, k (e4m3) and the 16-bit V image from its epilogue
            "qkv_gemm_v": (2.0 * t * d * 3 * d, t * d + 3 * d * d + 4 * t * d + 0.0, FP8_PEAK),
            "v_convert": (0.0, t * d * 3.0, FP8_PEAK),
            "attention": (2.0 * b * h * s * s * hd, t * d * 5.0, ATTN_PEAK),
            "out_gemm": (2.0 * t * d * d, t * d + d * d + 4.0 * t * d, FP8_PEAK),
            "ln2": (0.0, t * d * 3.0, FP8_PEAK),
            "fc_gemm": (2.0 * t * d * m, t * d + m * d + t * m + 0.0, FP8_PEAK),
            "proj_gemm": (2.0 * t * m * d, t * m + d * m + 4.0 * t * d, FP8_PEAK),
        }
    t, hid, h, hk, dh, s, b = blk.t, blk.hidden, blk.h, blk.hk, blk.dh, blk.seq, blk.batch
    nc = blk.n_cat
    return {
        "in_norm": (0.0, t * hid * 3.0, FP8_PEAK),
        "qgkv_gemm": (2.0 * t * hid * nc, t * hid + nc * hid + t * nc + 0.0, FP8_PEAK),
        # projection with the q / k norm + RoPE and the V copy in its epilogue: reads A and
        # the weights, writes the gate (e4m3), q and k (e4m3) and V (16-bit)
        "qgkv_gemm_prep": (2.0 * t * hid * nc,
                           t * hid + nc * hid + t * (nc - hk * dh) + 2.0 * t * hk * dh, FP8_PEAK),
        # projection writing q / gate / k (e4m3) and the 16-bit V image from its epilogue
        "qgkv_gemm_v": (2.0 * t * hid * nc,
                        t * hid + nc * hid + t * (nc - hk * dh) + 2.0 * t * hk * dh, FP8_PEAK),
        "qkv_prep": (0.0, 2.0 * t * (h + hk) * dh + 3.0 * t * hk * dh, FP8_PEAK),
        # q / k head norm + RoPE only (V came from the projection)
        "qk_prep": (0.0, 2.0 * t * (h + hk) * dh, FP8_PEAK),
        "qk_norm_rope": (0.0, 2.0 * t * (h + hk) * dh, FP8_PEAK),
        "v_convert": (0.0, 3.0 * t * hk * dh, FP8_PEAK),
        "attention": (2.0 * b * h * s * s * dh, t * dh * (3.0 * h + 4.0 * hk), ATTN_PEAK),
        "o_gemm": (2.0 * t * h * dh * hid, t * h * dh + hid * h * dh + 4.0 * t * hid, FP8_PEAK),
    }


class BlockWorkload:
    """BASELINE configs[3] (GPT-2 block, B8 x S1024) or configs[4] (Qwen gated attention
    block, B4 x S2048, 32q/8kv x 128, RoPE 1e6, separate gate projection), bf16 residual,
    random-init e4m3 weights with per-tensor amax scales; the block runs as a CUDA graph.
    At N>1 the global batch is split: batch groups first, then heads (``tp``)."""

    unit = "TFLOP/s"
    bound = "tensor"
    scaling = "strong"

    def __init__(self, kind: str, rank: int, world: int = 1, tp=None):
        from b200fp8 import blocks, sharding
        g = torch.Generator("cpu").manual_seed(20260801)
        self.kind, self.world, self.rank = kind, world, rank
        if kind == "gpt2":
            self.batch, self.seq, self.hidden = 8, 1024, 768
            self.w = _gpt2_weights(g)
            self.dp, self.tp = sharding.plan_block_parallel(world, self.batch, 12, 12, tp=tp or 1)
            self.name = "gpt2_block_fp8_b8_s1024"
        else:
            self.batch, self.seq, self.hidden = 4, 2048, 2560
            self.w = _qwen_weights(g, self.seq)
            self.dp, self.tp = sharding.plan_block_parallel(world, self.batch, 32, 8, tp=tp)
            self.name = "qwen_gated_attention_block_fp8_b4_s2048" + (
                f"_heads_tp{self.tp}" if tp else "")
        if world > 1:
            d, self.tp_rank, self.group = sharding.tp_groups(world, self.tp)
        else:
            d, self.tp_rank, self.group = 0, 0, None
        self.local_batch = self.batch // self.dp
        gx = torch.Generator("cpu").manual_seed(20260802)
        x_all = torch.randn((self.batch * self.seq, self.hidden), generator=gx).to(torch.bfloat16)
        t = self.local_batch * self.seq
        self.x_cpu = x_all[d * t:(d + 1) * t].contiguous()
        kw = dict(batch=self.local_batch, seq=self.seq, residual_dtype=torch.bfloat16,
                  out_dtype=torch.bfloat16)
        if kind == "gpt2":
            self.blk = blocks.GPT2Block(self.w, **kw)
            self.local = self.blk
        elif self.tp > 1:
            self.blk = sharding.QwenBlockTP(self.w, group=self.group, tp_rank=self.tp_rank,
                                            tp=self.tp, **kw)
            self.local = self.blk.blk
        else:
            self.blk = blocks.QwenBlock(self.w, **kw)
            self.local = self.blk
        self.launches = self.local.launches_per_forward
        self.x = self.x_cpu.cuda()
        self.blk.capture(self.x)
        self.blk.graph_input.copy_(self.x)
        self.work = self.local.flops()
        self.comm_ms = []
        self.flush = None
        if kind == "gpt2":
            # weights + activations of a forward (~110 MB) fit in L2: flush between steps
            self.flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def config(self):
        c = {"workload": f"{self.name} B={self.batch} S={self.seq} hidden={self.hidden}",
             "batch": self.batch, "seq": self.seq, "hidden": self.hidden,
             "dp": self.dp, "tp": self.tp, "residual": "bf16",
             "graph": "one CUDA graph per forward"}
        if self.kind == "gpt2":
            c.update(d_model=768, heads=12, head_dim=64, mlp=3072,
                     l2="a 252 MiB buffer is written between timed steps (L2 flush); the "
                        "flush is outside the per-step events")
        else:
            c.update(heads=32, kv_heads=8, head_dim=128, rope_theta=1e6,
                     l2="weights 33 MB + activations ~310 MB per forward > 126 MB L2")
        return c

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        p = f"{self.dp} batch groups ({self.local_batch} of {self.batch} sequences each, no communication)"
        if self.tp > 1:
            p += (f" x {self.tp}-way heads (column-parallel q/gate/k/v, row-parallel o-proj, "
                  "one NCCL SUM all-reduce of the bf16 [T x hidden] output per head group)")
        return p

    def pre_step(self):
        if self.flush is not None:
            self.flush.zero_()

    def step(self, ev=None):
        if self.tp > 1:
            import torch.distributed as dist
            out = self.local.replay()
            if ev is not None:
                ev[0].record()
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
            if ev is not None:
                ev[1].record()
        else:
            self.blk.replay()
        return self.launches

    def stages(self):
        times = self.local.stage_times(self.x, reps=5)
        model = _stage_model(self.kind, self.local)
        out = {}
        for name, ms in times.items():
            fl, by, pk = model.get(name, (0.0, 0.0, FP8_PEAK))
            roof_ms = max(fl / (pk * 1e12), by / (HBM * 1e9)) * 1e3
            out[name] = {"ms": round(ms, 5), "roofline_ms": round(roof_ms, 5),
                         "frac": round(roof_ms / ms, 3) if ms > 0 else None,
                         "tflops": round(fl / (ms * 1e-3) / 1e12, 1) if fl else None,
                         "gbs": round(by / (ms * 1e-3) / 1e9, 1)}
        return out

    def roofline(self, per_launch_ms):
        return None  # from the stage breakdown (dominant kernel)

    def snapshot(self):
        """Keeps the first sequence of the last timed step's output (after the head group's
        all-reduce): the eager stage timings that follow reuse the output buffer and, with
        heads parallelism, leave only this rank's partial in it."""
        out = self.local._g_out if self.tp > 1 else self.blk._g_out
        self._snap = out[:self.seq].float().cpu()

    def parity(self):
        """The timed graph's output for the first sequence of this rank's batch group
        against the CPU oracle block (reference thresholds: 0.05 GPT-2, 0.08 Qwen, plus one
        bf16 rounding of the output)."""
        from oracle import blocks as ob
        out0 = getattr(self, "_snap", None)
        if out0 is None:
            out = self.local._g_out if self.tp > 1 else self.blk._g_out
            out0 = out[:self.seq].float().cpu()
        x = self.x_cpu[:self.seq].float()
        t0 = time.perf_counter()
        if self.kind == "gpt2":
            ref = ob.gpt2_block(x, self.w, batch=1, residual_dtype=torch.bfloat16,
                                out_dtype=torch.bfloat16)
            tol = 0.05
        else:
            ref = ob.qwen_block(x, self.w, batch=1, residual_dtype=torch.bfloat16,
                                out_dtype=torch.bfloat16)
            tol = 0.08
        self.oracle_s = time.perf_counter() - t0
        err = (out0 - ref).abs()
        bound = tol + 2.0 ** -8 * ref.abs()
        ok = bool((err <= bound).all()) and bool(torch.isfinite(out0).all())
        return {"status": "pass" if ok else "fail", "max_abs_err": float(err.max()),
                "bar": f"|err| <= {tol} + 2^-8 |ref| (reference task threshold)",
                "check": f"sequence 0 of this rank's group ({self.seq} tokens x {self.hidden}) "
                         "of the timed output vs the CPU oracle block"}

    def e2e_setup(self):
        self.hx = self.x_cpu.pin_memory()
        self.ho = torch.empty_like(self.x_cpu).pin_memory()
        self.sin = [torch.empty_like(self.x) for _ in range(2)]
        self.sout = [torch.empty_like(self.x) for _ in range(2)]

    def e2e_h2d(self, slot):
        self.sin[slot].copy_(self.hx, non_blocking=True)

    def e2e_compute(self, slot):
        self.blk.graph_input.copy_(self.sin[slot])
        self.sout[slot].copy_(self.blk.replay())

    def e2e_d2h(self, slot):
        self.ho.copy_(self.sout[slot], non_blocking=True)

    def e2e_bytes(self):
        n = self.x_cpu.numel() * 2
        return n, n

    def e2e_release(self):
        del self.sin, self.sout

    def cpu_sample(self, target_s: float):
        """The oracle block on one sequence (timed inside ``parity``, which runs first)."""
        threads = _threads()
        t = getattr(self, "oracle_s", None)
        if t is None:
            self.parity()
            t = self.oracle_s
        return {"value": self.work / self.local_batch / t / 1e12, "unit": "TFLOP/s",
                "cores": threads, "kind": "port",
                "sample": f"1 of {self.batch} sequences through the CPU oracle block "
                          f"(f64-accumulated FP8 products), {t:.2f} s"}


def make_workload(name: str, rank: int, world: int = 1, tp=None, n: int = 8192):
    if name == "gemm":
        return GemmWorkload(n, rank, world)
    if name == "gemm_bias_relu":
        return GemmWorkload(8192, rank, world, bias_relu=True, m=128)
    if name == "norm":
        return NormWorkload(rank, world)
    if name in ("gpt2", "qwen"):
        return BlockWorkload(name, rank, world, tp)
    if name == "qwen_heads":
        return BlockWorkload("qwen", rank, world, tp=world)
    if name == "layer_norm_rows":
        return LayerNormRowsWorkload(rank, world)
    if name == "gated_gemm":
        return GatedGemmWorkload(rank, world)
    raise SystemExit(f"unknown workload {name}")


def _run_e2e(wl, steps: int) -> float:
    """End-to-end steps through the public API: step i copies its inputs host -> device,
    runs, and copies its result device -> host.  Three streams and two buffer slots
    pipeline the work (inputs of step i+1 and the result of step i-1 cross PCIe while step i
    computes); every step still moves all of its bytes.  Returns ms per step, timed with
    CUDA events on the current stream around the whole pipeline."""
    cur = torch.cuda.current_stream()
    s_in, s_c, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_c = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for st in (s_in, s_c, s_out):
        st.wait_event(e0)
    for i in range(steps + 2):
        if i < steps:
            slot = i % 2
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_c[slot])
                wl.e2e_h2d(slot)
                ev_in[slot].record(s_in)
        j = i - 1
        if 0 <= j < steps:
            slot = j % 2
            with torch.cuda.stream(s_c):
                s_c.wait_event(ev_in[slot])
                if j >= 2:
                    s_c.wait_event(ev_out[slot])
                wl.e2e_compute(slot)
                ev_c[slot].record(s_c)
        k = i - 2
        if 0 <= k < steps:
            slot = k % 2
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c[slot])
                wl.e2e_d2h(slot)
                ev_out[slot].record(s_out)
    for st in (s_in, s_c, s_out):
        cur.wait_stream(st)
    e1.record(cur)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _traffic(name):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(name)
    except Exception:
        return None


def measure(wl, args, world, rank, sampler, soak_s, steps, cpu_s):
    """Warm-up, soak, timed steps, stage breakdown, e2e, parity and (N=1) CPU baseline of
    one workload.  Returns its JSON entry (rank 0) or None."""
    from b200fp8 import device_status
    for _ in range(args.warmup):
        if hasattr(wl, "pre_step"):
            wl.pre_step()
        wl.step()
    torch.cuda.synchronize()
    t_window0 = time.time()
    # Untimed soak so the timed region runs at the sustained (power-capped) clock; every
    # rank runs the same number of soak steps (steps may hold collectives).
    t_est = time.time()
    for _ in range(2):
        wl.step()
    torch.cuda.synchronize()
    per_step_s = max((time.time() - t_est) / 2, 1e-6)
    n_soak = int(_max_over_ranks(float(min(20000, soak_s / per_step_s)), world))
    for i in range(n_soak):
        wl.step()
        if i % 64 == 63:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    has_comm = isinstance(wl, BlockWorkload) and wl.tp > 1
    # Host time to enqueue one step (no synchronisation): the timed steps are queued behind a
    # device-side wait at least that long, so the device runs them back to back and the
    # events time device work, not the Python launch path (which e2e covers).
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    for _ in range(3):
        if hasattr(wl, "pre_step"):
            wl.pre_step()
        wl.step()
    host_ms = (time.perf_counter() - h0) / 3 * 1e3
    torch.cuda.synchronize()
    host_ms = _max_over_ranks(host_ms, world)
    _barrier(world)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int((1.5 * steps * host_ms + 0.5) * 2.0e6))  # ~2 GHz clock cycles
    t0.record(stream)
    launches = 0
    # Per-step events only where the steps are separated by untimed work (the L2 flush of
    # the GPT-2 block): an event between two launches serialises them and stops the next
    # kernel's programmatic early launch, which costs the short GEMMs up to a third of a
    # step.  Otherwise the K steps run back to back between t0 and t1.
    per_step = getattr(wl, "flush", None) is not None
    for i in range(steps):
        if hasattr(wl, "pre_step"):
            wl.pre_step()
        if per_step:
            ev[i][0].record(stream)
        launches += wl.step(cev[i]) if has_comm else wl.step()
        if per_step:
            ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    t_window1 = time.time()
    _barrier(world)
    if per_step:
        step_ms = [e[0].elapsed_time(e[1]) for e in ev]
        ms_per_step = statistics.mean(step_ms)  # flushes between steps are not timed
    else:
        ms_per_step = t0.elapsed_time(t1) / steps
        step_ms = [ms_per_step]
    ms_per_step = _max_over_ranks(ms_per_step, world)
    per_launch_ms = _max_over_ranks(statistics.mean(step_ms), world)
    comm = None
    if has_comm:
        c_ms = _max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in cev), world)
        comm = {"collective": "NCCL all_reduce SUM, bf16 [T x hidden]",
                "comm_nranks": wl.tp, "bytes": wl.x.numel() * 2,
                "ms_per_step": round(c_ms, 5), "share_of_step": round(c_ms / ms_per_step, 4)}
    status = device_status()
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = wl.work * world / (ms_per_step * 1e-3) / scale  # whole job (all ranks)

    if hasattr(wl, "snapshot"):
        wl.snapshot()  # the timed output, before the stage timings overwrite its buffer
    stages = wl.stages() if hasattr(wl, "stages") else None
    if stages is not None:
        stages = {k: v for k, v in stages.items()}
        dom = max(stages, key=lambda k: stages[k]["ms"])
        model = _stage_model(wl.kind, wl.local)
        fl, by, pk = model[dom]
        dms = stages[dom]["ms"]
        if fl > 0:
            roof = {"bound": "tensor", "achieved": round(fl / (dms * 1e-3) / 1e12, 1),
                    "peak": round(pk, 1), "unit": "TFLOP/s",
                    "peak_basis": ("blend of e4m3 (2 x bf16) and bf16 peaks for the QK^T / "
                                   "P.V halves" if dom == "attention" else "2 x bf16 burst"),
                    "algorithmic_work_per_launch": fl}
        else:
            roof = {"bound": "hbm", "achieved": round(by / (dms * 1e-3) / 1e9, 1),
                    "peak": HBM, "unit": "GB/s", "algorithmic_work_per_launch": by}
        roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
        roof["kernel"] = dom
        roof["per_launch_ms"] = dms
        roof["per_launch_source"] = ("CUDA events between the stages of eager forwards "
                                     "(launches queued behind a device sleep)")
        combined = sum(v["roofline_ms"] for v in stages.values())
        block_roof = {"stage_roofline_sum_ms": round(combined, 5),
                      "measured_ms": round(ms_per_step, 5),
                      "ratio_to_roofline": round(ms_per_step / combined, 3)}
    else:
        kname, work, unit, peak, basis = wl.roofline(per_launch_ms)
        achieved = work / (per_launch_ms * 1e-3)
        roof = {"bound": wl.bound, "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": unit, "frac": round(achieved / peak, 4), "peak_basis": basis,
                "kernel": kname, "per_launch_ms": round(per_launch_ms, 5),
                "algorithmic_work_per_launch": work * (1e12 if unit == "TFLOP/s" else 1e9)}
        block_roof = None
    tr = _traffic(wl.name)
    roof["traffic"] = tr.get("traffic_bytes_per_launch") if tr else None
    if tr:
        roof["traffic_source"] = tr.get("source")
    roof["peak_note"] = "of measured" if PEAKS["basis"] == "measured" else "of fallback"

    parity = wl.parity() if rank == 0 else None

    wl.e2e_setup()
    _run_e2e(wl, 2)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_steps = max(3, min(steps, 20))
    e2e_ms = _max_over_ranks(_run_e2e(wl, e2e_steps), world)
    h2d, d2h = wl.e2e_bytes()
    wl.e2e_release()

    entry = None
    if rank == 0:
        entry = {
            "workload": wl.name, "metric": f"{wl.unit} ({wl.name}, whole job)",
            "value": round(value, 2), "unit": wl.unit, "ms_per_step": round(ms_per_step, 5),
            "scaling": wl.scaling, "config": dict(wl.config(), parallelism=wl.parallelism()),
            "roofline": roof,
            "e2e": {"value": round(wl.work * world / (e2e_ms * 1e-3) / scale, 3),
                    "unit": wl.unit, "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "path": "public b200fp8 API; every step copies its inputs from pinned host "
                            "memory and its result back; copies of neighbouring steps overlap "
                            "the compute (3 streams, 2 buffer slots)"},
            "parity": parity, "gpu_launches": launches, "device_status": status,
            "window": (t_window0, t_window1),
        }
        if stages is not None:
            entry["stages"] = stages
            entry["block_roofline"] = block_roof
        if comm is not None:
            entry["comm"] = comm
        if world == 1 and cpu_s > 0:
            entry["cpu_baseline"] = wl.cpu_sample(target_s=cpu_s)
    return entry


def _cublaslt_same_shape(n, soak_s: float, steps: int):
    """cuBLASLt FP8 (torch._scaled_mm) at the square shape, a library reference point timed
    the way our kernel is: the same soak at the sustained (power-capped) clock, then
    `steps` calls back to back behind a device-side wait, rotating input sets larger than
    L2 where they fit."""
    try:
        g = torch.Generator("cpu").manual_seed(1)
        a, sa = _fp8_inputs((n, n), g)
        b, sb = _fp8_inputs((n, n), g)
        nsets = 1 if 2 * n * n >= 2 * L2_BYTES else min(8, -(-3 * L2_BYTES // (2 * n * n)))
        sets = [(a.cuda(), b.cuda()) for _ in range(nsets)]
        sa_t = torch.tensor(sa, device="cuda")
        sb_t = torch.tensor(sb, device="cuda")
        run = lambda j: torch._scaled_mm(sets[j % nsets][0], sets[j % nsets][1].t(),  # noqa: E731
                                         scale_a=sa_t, scale_b=sb_t, out_dtype=torch.bfloat16)
        for j in range(3):
            run(j)
        torch.cuda.synchronize()
        t_end = time.time() + soak_s
        j = 0
        while time.time() < t_end:
            run(j)
            j += 1
            if j % 16 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(2.0e6))
        c0.record()
        for j in range(steps):
            run(j)
        c1.record()
        torch.cuda.synchronize()
        return round(2.0 * n ** 3 / (c0.elapsed_time(c1) / steps * 1e-3) / 1e12, 1)
    except Exception as exc:  # a side measurement never fails the bench
        return f"unavailable: {type(exc).__name__}"


def run_ours(args):
    world, rank, local = _dist()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=180))
    else:
        torch.cuda.set_device(0)
    from b200fp8 import _lib  # noqa: F401  (fails loudly without the .so)

    sampler = ClockSampler(torch.cuda.current_device())
    if rank == 0:
        sampler.start()
        time.sleep(0.3)

    headline_name = "qwen" if args.workload == "all" else args.workload
    plan = [(headline_name, args.tp, args.soak_seconds, args.steps, args.cpu_seconds)]
    if args.workload == "all":
        side_cpu = min(args.cpu_seconds, 3.0)
        side_soak = min(args.soak_seconds, 0.5)
        if world == 1:
            plan += [("gemm_bias_relu", None, side_soak, args.steps, side_cpu)]
            plan += [(("gemm", n), None, side_soak, args.steps, side_cpu)
                     for n in (4096, 8192, 16384)]
            plan += [("norm", None, side_soak, args.steps, side_cpu),
                     ("gpt2", None, side_soak, args.steps, side_cpu),
                     ("layer_norm_rows", None, side_soak, args.steps, side_cpu),
                     ("gated_gemm", None, side_soak, args.steps, side_cpu)]
        else:
            plan += [("qwen_heads", None, side_soak, args.steps, 0),
                     (("gemm", 8192), None, side_soak, args.steps, 0),
                     ("norm", None, side_soak, args.steps, 0),
                     ("gpt2", None, side_soak, args.steps, 0)]
    entries = []
    for name, tp, soak, steps, cpu_s in plan:
        n = args.n
        if isinstance(name, tuple):
            name, n = name
        if name == "qwen_heads" and (8 % world or 32 % world):
            continue
        wl = make_workload(name, rank, world, tp, n)
        e = measure(wl, args, world, rank, sampler, soak, steps, cpu_s)
        if e is not None and name == "gemm" and world == 1:
            e["cublaslt_fp8_tflops_same_shape"] = _cublaslt_same_shape(n, soak, steps)
        entries.append(e)
        del wl
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        _barrier(world)
    if rank == 0:
        sampler.stop()
        for e in entries:
            w0, w1 = e.pop("window")
            e["clocks"] = sampler.window(w0, w1)
        head = entries[0]
        out = {
            "metric": head["metric"], "value": head["value"], "unit": head["unit"],
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": head["scaling"], "vs_baseline": None,
            "dtype": "e4m3 operands, f32 accumulate, bf16 residual / outputs",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init e4m3 weights "
                    "with per-tensor amax scales)",
        }
        for k in ("config", "roofline", "e2e", "cpu_baseline", "parity", "stages",
                  "block_roofline", "comm", "gpu_launches", "clocks", "device_status"):
            if k in head:
                out[k] = head[k]
        if len(entries) > 1:
            out["workloads"] = entries[1:]
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_reference(args):
    """Reference arm: the reference evaluator's Torch math of the headline (the Qwen gated
    full-attention block, tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-416,
    restated by oracle.blocks.qwen_block) on the host cores, one of the batch's sequences
    per step, BASELINE configs[4]'s shapes and weights."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    from oracle import blocks as ob
    threads = _threads()
    torch.set_num_threads(threads)
    g = torch.Generator("cpu").manual_seed(20260801)
    batch, seq, hidden = 4, 2048, 2560
    w = _qwen_weights(g, seq)
    gx = torch.Generator("cpu").manual_seed(20260802)
    x = torch.randn((batch * seq, hidden), generator=gx).to(torch.bfloat16)
    t, hd, h, hk, dh = seq, hidden, 32, 8, 128
    n_cat = 2 * h * dh + 2 * hk * dh
    flops = 2.0 * t * hd * n_cat + 2.0 * t * h * dh * hd + 2.0 * h * seq * seq * dh
    times = []
    for i in range(args.warmup + args.steps):
        xs = x[(i % batch) * seq:(i % batch + 1) * seq].float()
        t0 = time.perf_counter()
        ob.qwen_block(xs, w, batch=1, residual_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    dt = statistics.mean(times)
    value = flops / dt / 1e12
    out = {
        "impl": "reference", "metric": "TFLOP/s (qwen_gated_attention_block_fp8_b4_s2048, whole job)",
        "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 * batch, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 operands, f32/f64 accumulate, bf16 residual / outputs",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init e4m3 weights)",
        "config": {"workload": f"qwen_gated_attention_block_fp8_b4_s2048 B={batch} S={seq} "
                               f"hidden={hidden}", "batch": batch, "seq": seq, "hidden": hidden,
                   "parallelism": "host cores of rank 0"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port",
                         "sample": "1 of 4 sequences per step through the Torch math of the "
                                   "reference's Qwen block evaluator on CPU (oracle.blocks."
                                   "qwen_block; ms_per_step scaled to the 4-sequence batch)"},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="all")
    ap.add_argument("--n", type=int, default=8192, help="square GEMM size for --workload gemm")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--soak-seconds", type=float, default=1.0)
    ap.add_argument("--tp", type=int, default=None,
                    help="qwen: head-parallel group size (default: batch groups first)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
