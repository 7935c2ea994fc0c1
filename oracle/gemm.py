"""CPU restatement of the reference's scaled FP8 GEMM and its epilogues.

The reference computes every FP8 linear with ``torch._scaled_mm(a_fp8, b_fp8.t(),
scale_a, scale_b, out_dtype=float32)``:
  - square GEMM     tasks/level1_01_square_matrix_multiplication_fp8/starter.py:125-138
  - GEMM+bias+ReLU  tasks/level2_76_gemm_add_relu_fp8/starter.py:148-169
  - epilogues       tasks/level2_09_*/starter.py:126  relu((lin - 2) * 1.5)
                    tasks/level2_12_*/starter.py:126  leaky_relu(lin * 2, 0.1)
                    tasks/level2_14_*/starter.py:116-121  (mm / 2).sum(1, keepdim) * 1.5
                    tasks/level2_40_*/starter.py:125  lin * 0.5 + lin
                    tasks/level2_63_*/starter.py:125  relu(lin) / 2
  - block linears   ``_cute_harness_scaled_linear`` in the block tasks' starter.py.
  - gated residual  cute_kernels/fused_gemm_gated_residual_fp8/submission.py:383-394
                    (_scaled_mm(a, b.t()) * gate + residual)
e4m3 x e4m3 products are exact in f32; this oracle accumulates them in f64 and rounds
once, so it is at least as accurate as any f32 accumulation order.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def scaled_mm(a_fp8: torch.Tensor, b_nk_fp8: torch.Tensor, scale_a: float,
              scale_b: float) -> torch.Tensor:
    """f32 (A . B_nk^T) * scale_a * scale_b, f64-accumulated."""
    acc = a_fp8.double() @ b_nk_fp8.double().t()
    return (acc * (float(scale_a) * float(scale_b))).float()


def activation(v: torch.Tensor, act: Optional[str], act_param: float = 0.0) -> torch.Tensor:
    if act is None or act == "none":
        return v
    if act == "relu":
        return torch.relu(v)
    if act == "gelu_tanh":
        return F.gelu(v, approximate="tanh")
    if act == "leaky_relu":
        return F.leaky_relu(v, negative_slope=act_param)
    if act == "silu":
        return F.silu(v)
    raise ValueError(act)


def gemm_epilogue(a_fp8, b_nk_fp8, scale_a=1.0, scale_b=1.0, bias=None, pre_mul=1.0,
                  pre_add=0.0, act=None, act_param=0.0, post_mul=1.0, residual=None,
                  residual_scale=1.0, rowsum=False, out_scale=1.0, gate=None) -> torch.Tensor:
    """f32 value of the fused epilogue before the output cast (see b2f_gemm_fp8)."""
    v = scaled_mm(a_fp8, b_nk_fp8, scale_a, scale_b)
    if bias is not None:
        v = v + bias.float()
    v = v * pre_mul + pre_add
    v = activation(v, act, act_param) * post_mul
    if gate is not None:
        v = v * gate.float()
    if residual is not None:
        v = v + residual.float() * residual_scale
    if rowsum:
        return v.double().sum(dim=1).float() / out_scale
    return v / out_scale


def cpu_fast_scaled_mm(a_fp8, b_nk_fp8, scale_a, scale_b) -> torch.Tensor:
    """Fastest CPU form of the same math (f32 dequantise + multithreaded matmul); the
    timed CPU baseline of bench.py."""
    return (a_fp8.float() @ b_nk_fp8.float().t()) * (float(scale_a) * float(scale_b))


def reference_scaled_mm_cpu(a_fp8, b_nk_fp8, scale_a, scale_b) -> torch.Tensor:
    """The reference evaluator's own call, ``torch._scaled_mm(a, b.t(), scale_a, scale_b,
    out_dtype=float32)`` (tasks/level1_01_square_matrix_multiplication_fp8/starter.py:125-138),
    executed on CPU."""
    sa = torch.tensor(float(scale_a), dtype=torch.float32)
    sb = torch.tensor(float(scale_b), dtype=torch.float32)
    return torch._scaled_mm(a_fp8, b_nk_fp8.t(), scale_a=sa, scale_b=sb,
                            out_dtype=torch.float32)
