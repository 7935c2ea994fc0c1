"""torch.library registrations of the b200fp8 ops (namespace ``b200fp8``).

Registering the ops as torch custom ops lets torch's graph machinery see them:
``torch.cuda.graphs`` capture them like any other kernel launch, and ``torch.compile`` /
``torch.export`` trace through them as opaque nodes (the fake implementations below give
output shapes and dtypes without running anything).  The real implementations call the
C ABI through ``b200fp8.ops``; there is no CPU implementation.

  torch.ops.b200fp8.gemm_fp8(a, b_nk, scale_a, scale_b, bias, act, out_dtype, out_scale,
                              residual, residual_scale) -> Tensor
  torch.ops.b200fp8.quantize_fp8(x) -> (q, scale)
  torch.ops.b200fp8.residual_rmsnorm_quant(x, residual, gamma, eps) -> (q, scale, h)
  torch.ops.b200fp8.attention_fp8(q, k, v, batch, heads, kv_heads, head_dim, causal,
                                   q_scale, k_scale, v_scale, ctx_scale, gate,
                                   gate_scale) -> Tensor
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.library import custom_op

from . import ops

_E4M3 = torch.float8_e4m3fn


@custom_op("b200fp8::gemm_fp8", mutates_args=(), device_types="cuda")
def gemm_fp8(a: Tensor, b_nk: Tensor, scale_a: float, scale_b: float, bias: Optional[Tensor],
             act: str, out_dtype: torch.dtype, out_scale: float, residual: Optional[Tensor],
             residual_scale: float) -> Tensor:
    return ops.gemm_fp8(a, b_nk, scale_a=scale_a, scale_b=scale_b, bias=bias,
                        act=None if act == "none" else act, out_dtype=out_dtype,
                        out_scale=out_scale, residual=residual, residual_scale=residual_scale)


@gemm_fp8.register_fake
def _gemm_fp8_fake(a, b_nk, scale_a, scale_b, bias, act, out_dtype, out_scale, residual,
                   residual_scale):
    return a.new_empty((a.shape[0], b_nk.shape[0]), dtype=out_dtype)


@custom_op("b200fp8::quantize_fp8", mutates_args=(), device_types="cuda")
def quantize_fp8(x: Tensor) -> Tuple[Tensor, Tensor]:
    q, s = ops.quantize_fp8(x)
    return q, s


@quantize_fp8.register_fake
def _quantize_fp8_fake(x):
    return x.new_empty(x.shape, dtype=_E4M3), x.new_empty((1,), dtype=torch.float32)


@custom_op("b200fp8::residual_rmsnorm_quant", mutates_args=(), device_types="cuda")
def residual_rmsnorm_quant(x: Tensor, residual: Tensor, gamma: Tensor,
                           eps: float) -> Tuple[Tensor, Tensor, Tensor]:
    h = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
    q, s = ops.norm_quant(x, gamma, residual=residual, h_out=h, eps=eps)
    return q, s, h


@residual_rmsnorm_quant.register_fake
def _residual_rmsnorm_quant_fake(x, residual, gamma, eps):
    return (x.new_empty(x.shape, dtype=_E4M3), x.new_empty((1,), dtype=torch.float32),
            x.new_empty(x.shape, dtype=torch.bfloat16))


@custom_op("b200fp8::attention_fp8", mutates_args=(), device_types="cuda")
def attention_fp8(q: Tensor, k: Tensor, v: Tensor, batch: int, heads: int, kv_heads: int,
                  head_dim: int, causal: bool, q_scale: float, k_scale: float, v_scale: float,
                  ctx_scale: float, gate: Optional[Tensor], gate_scale: float) -> Tensor:
    return ops.attention_fp8(q, k, v, batch=batch, heads=heads, kv_heads=kv_heads,
                             head_dim=head_dim, causal=causal, q_scale=q_scale,
                             k_scale=k_scale, v_scale=v_scale, gate=gate,
                             gate_scale=gate_scale, ctx_scale=ctx_scale)


@attention_fp8.register_fake
def _attention_fp8_fake(q, k, v, batch, heads, kv_heads, head_dim, causal, q_scale, k_scale,
                        v_scale, ctx_scale, gate, gate_scale):
    return q.new_empty((q.shape[0], heads * head_dim), dtype=_E4M3)
