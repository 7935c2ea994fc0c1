"""Torch-facing wrappers of the C-ABI ops.

Tensors are passed to libb200fp8.so as raw device pointers plus shapes; the kernels run
on torch's current CUDA stream.  float8_e4m3fn tensors (or uint8 views of them) carry
FP8 data; a per-tensor scale ``s`` means ``value = stored * s``.
"""
from __future__ import annotations

import ctypes
import functools
from typing import Optional

import torch

from . import _lib
from ._lib import GemmArgs, check

_ACTS = {
    None: _lib.ACT_NONE, "none": _lib.ACT_NONE, "relu": _lib.ACT_RELU,
    "gelu_tanh": _lib.ACT_GELU_TANH, "leaky_relu": _lib.ACT_LEAKY_RELU,
    "silu": _lib.ACT_SILU,
}

_DT = {
    torch.float32: _lib.DTYPE_F32,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float8_e4m3fn: _lib.DTYPE_E4M3,
    torch.uint8: _lib.DTYPE_E4M3,
    torch.float16: _lib.DTYPE_F16,
}


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_cuda(*tensors: Optional[torch.Tensor]) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("b200fp8 ops take CUDA tensors only (no CPU fallback)")


_WORKSPACES = {}
_STATS = {}


def _stats_scratch(rows: int, device) -> torch.Tensor:
    """Per-device f32 scratch for the norm's (mean, rstd) hand-off between its passes (the
    two passes of one call run back to back on the caller's stream)."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _STATS.get(key)
    if buf is None or buf.numel() < 2 * rows:
        buf = torch.empty((max(2 * rows, 1 << 16),), dtype=torch.float32, device=dev)
        _STATS[key] = buf
    return buf


@functools.lru_cache(maxsize=None)
def _sm_count(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def _auto_split(m: int, n: int, k: int, device) -> bool:
    """Shapes for which the library splits K in two when ``splits`` is None (few 128 x 128
    tiles, long K: the rule of b2f_gemm_fp8's automatic choice); they get the cached
    workspace."""
    dev = torch.device(device)
    tiles = ((m + 127) // 128) * ((n + 127) // 128)
    return (k + 127) // 128 >= 32 and tiles * 2 <= _sm_count(dev.index or 0)


def gemm_workspace(m: int, n: int, device) -> torch.Tensor:
    """Split-K workspace for an m x n GEMM output on ``device``: zero-filled once, cached per
    device and grown on demand.  Its tile counters carry a per-call tag, so a call that
    timed out and left them mid-protocol does not mislead the next call.  One workspace per
    device means split-K GEMMs on one device must not
    overlap in time (the library issues them on the caller's single stream)."""
    need = int(_lib.lib().b2f_gemm_workspace_bytes(m, n))
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros((max(need, 1 << 20),), dtype=torch.uint8, device=dev)
        _WORKSPACES[key] = ws
    return ws


def _fp8_rows(t: torch.Tensor, name: str) -> None:
    if t.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise TypeError(f"{name} must be float8_e4m3fn (or its uint8 storage)")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a row-major 2-D tensor")


def gemm_fp8(a: torch.Tensor, b_nk: torch.Tensor, *, scale_a: float = 1.0,
             scale_b: float = 1.0, alpha_tensor: Optional[torch.Tensor] = None,
             col_scale: Optional[torch.Tensor] = None,
             bias: Optional[torch.Tensor] = None, pre_mul: float = 1.0,
             pre_add: float = 0.0, act: Optional[str] = None, act_param: float = 0.0,
             post_mul: float = 1.0, residual: Optional[torch.Tensor] = None,
             residual_scale: float = 1.0, out: Optional[torch.Tensor] = None,
             out_dtype: torch.dtype = torch.bfloat16, out_scale: float = 1.0,
             amax: Optional[torch.Tensor] = None, rowsum: bool = False,
             tile_n: int = 0, splits: Optional[int] = None,
             workspace: Optional[torch.Tensor] = None,
             gate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = epilogue(scale_a*scale_b * A . B_nk^T)  (see b2f_gemm_fp8).

    ``gate`` (f32 or bf16 [M, N]) multiplies the value after ``post_mul``, before the
    residual is added: the gated-residual epilogue.

    ``out_scale`` is the quantisation scale of an e4m3 output (stored = v / out_scale).
    With ``rowsum=True`` the output is f32 [M] holding sum over columns of v / out_scale.
    ``splits`` > 1 selects split-K with that many K slices (using ``workspace`` or the cached
    one of :func:`gemm_workspace`); None / 1 = off.
    """
    _check_cuda(a, b_nk, bias, residual, out, amax, alpha_tensor, col_scale, gate)
    _fp8_rows(a, "a")
    _fp8_rows(b_nk, "b_nk")
    m, k = a.shape
    n, k2 = b_nk.shape
    if k != k2:
        raise ValueError(f"K mismatch: {k} vs {k2}")
    if rowsum:
        if out is None:
            out = torch.zeros((m,), device=a.device, dtype=torch.float32)
        out_dtype = torch.float32
    elif out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    args = GemmArgs()
    _lib.lib().b2f_gemm_args_init(ctypes.byref(args))
    args.m, args.n, args.k = m, n, k
    args.a, args.lda = a.data_ptr(), a.stride(0)
    args.b, args.ldb = b_nk.data_ptr(), b_nk.stride(0)
    args.alpha = float(scale_a) * float(scale_b)
    args.alpha_ptr = _ptr(alpha_tensor)
    if col_scale is not None:
        if col_scale.dtype != torch.float32 or not col_scale.is_contiguous() or col_scale.numel() != n:
            raise TypeError("col_scale must be contiguous float32 [n]")
    args.col_scale = _ptr(col_scale)
    if bias is not None:
        if bias.dtype != torch.float32 or not bias.is_contiguous():
            raise TypeError("bias must be contiguous float32")
    args.bias = _ptr(bias)
    args.pre_mul, args.pre_add = pre_mul, pre_add
    args.act = _ACTS[act]
    args.act_param = act_param
    args.post_mul = post_mul
    if residual is not None:
        if residual.dim() != 2 or residual.stride(1) != 1:
            raise ValueError("residual must be row-major 2-D")
        args.residual = residual.data_ptr()
        args.residual_dtype = _DT[residual.dtype]
        args.residual_ld = residual.stride(0)
        args.residual_scale = residual_scale
    if gate is not None:
        if gate.dim() != 2 or gate.stride(1) != 1 or gate.dtype not in (torch.float32,
                                                                        torch.bfloat16):
            raise ValueError("gate must be a row-major 2-D f32 or bf16 tensor")
        args.gate, args.gate_dtype, args.gate_ld = gate.data_ptr(), _DT[gate.dtype], gate.stride(0)
    args.out = out.data_ptr()
    args.out_dtype = _DT[out.dtype]
    args.out_ld = out.stride(0) if out.dim() == 2 else 1
    args.out_scale = out_scale
    args.amax = _ptr(amax)
    args.mode = _lib.GEMM_ROWSUM if rowsum else _lib.GEMM_STORE
    args.tile_n = tile_n
    args.splits = 0 if splits is None else int(splits)
    if (splits is not None and splits > 1) or (splits is None and _auto_split(m, n, k, a.device)):
        ws = workspace if workspace is not None else gemm_workspace(m, n, a.device)
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel() * ws.element_size()
    check(_lib.lib().b2f_gemm_fp8(ctypes.byref(args), _stream()))
    return out


def gemm_fp8_head_prep(a: torch.Tensor, b_nk: torch.Tensor, *, out: torch.Tensor,
                       out_scale: float, q_out: Optional[torch.Tensor],
                       k_out: Optional[torch.Tensor], v_out: Optional[torch.Tensor],
                       q_off: int, q_heads: int, k_off: int, k_heads: int, v_off: int,
                       v_heads: int, q_head_stride: int = 128, scale_a: float = 1.0,
                       scale_b: float = 1.0, col_scale: Optional[torch.Tensor] = None,
                       bias: Optional[torch.Tensor] = None,
                       q_norm_w: Optional[torch.Tensor] = None,
                       k_norm_w: Optional[torch.Tensor] = None, weight_offset: float = 0.0,
                       eps: float = 1e-6, cos: Optional[torch.Tensor] = None,
                       sin: Optional[torch.Tensor] = None, seq: int = 0,
                       qk_out_scale: Optional[float] = None) -> bool:
    """q / gate / k / v projection with the attention-operand preparation in its epilogue
    (b2f_gemm_fp8_head_prep): the result of :func:`gemm_fp8` (e4m3 ``out`` at ``out_scale``)
    followed by :func:`attn_prep`, except that only the non-head columns (the gate) are
    written to ``out``.  Head dim 128, full-head RoPE; with ``q_heads = k_heads = 0`` only
    the V copy is fused (any head size: v "heads" are 128-column blocks).  Returns False,
    having done nothing, for shapes the fused kernel does not cover."""
    _check_cuda(a, b_nk, out, q_out, k_out, v_out, col_scale, bias, q_norm_w, k_norm_w, cos,
                sin)
    _fp8_rows(a, "a")
    _fp8_rows(b_nk, "b_nk")
    m, k = a.shape
    n, k2 = b_nk.shape
    if k != k2:
        raise ValueError(f"K mismatch: {k} vs {k2}")
    if out.dtype != torch.float8_e4m3fn:
        raise TypeError("out must be e4m3")
    if col_scale is not None and (col_scale.dtype != torch.float32 or not col_scale.is_contiguous()
                                  or col_scale.numel() != n):
        raise TypeError("col_scale must be contiguous float32 [n]")
    args = GemmArgs()
    L = _lib.lib()
    L.b2f_gemm_args_init(ctypes.byref(args))
    args.m, args.n, args.k = m, n, k
    args.a, args.lda = a.data_ptr(), a.stride(0)
    args.b, args.ldb = b_nk.data_ptr(), b_nk.stride(0)
    args.alpha = float(scale_a) * float(scale_b)
    args.col_scale = _ptr(col_scale)
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise TypeError("bias must be contiguous float32")
    args.bias = _ptr(bias)
    args.out, args.out_dtype, args.out_ld = out.data_ptr(), _DT[out.dtype], out.stride(0)
    args.out_scale = out_scale
    hp = _lib.HeadPrepArgs()
    hp.q_off, hp.q_head_stride, hp.q_heads = q_off, q_head_stride, q_heads
    hp.k_off, hp.k_heads, hp.v_off, hp.v_heads = k_off, k_heads, v_off, v_heads
    hp.q_out, hp.q_ld = _ptr(q_out), (q_out.stride(0) if q_out is not None else 0)
    hp.k_out, hp.k_ld = _ptr(k_out), (k_out.stride(0) if k_out is not None else 0)
    hp.v_out, hp.v_ld = _ptr(v_out), (v_out.stride(0) if v_out is not None else 0)
    hp.v_dtype = _DT[v_out.dtype] if v_out is not None else _lib.DTYPE_F16
    hp.q_norm_w, hp.k_norm_w = _ptr(q_norm_w), _ptr(k_norm_w)
    hp.weight_offset, hp.eps = weight_offset, eps
    hp.rope_cos, hp.rope_sin, hp.seq = _ptr(cos), _ptr(sin), seq
    hp.out_scale = out_scale if qk_out_scale is None else qk_out_scale
    rc = L.b2f_gemm_fp8_head_prep(ctypes.byref(args), ctypes.byref(hp), _stream())
    if rc == _lib.B2F_ERR_UNSUPPORTED:
        return False
    check(rc)
    return True


def norm_quant(x: torch.Tensor, weight: torch.Tensor, *, kind: str = "rms",
               bias: Optional[torch.Tensor] = None, weight_offset: float = 0.0,
               eps: float = 1e-6, x_scale: float = 1.0,
               residual: Optional[torch.Tensor] = None,
               h_out: Optional[torch.Tensor] = None, y_out: Optional[torch.Tensor] = None,
               q_out: Optional[torch.Tensor] = None, q_scale: Optional[float] = None,
               amax: Optional[torch.Tensor] = None,
               scale_out: Optional[torch.Tensor] = None, phase: Optional[str] = None,
               schedule: str = "auto", query_schedule: bool = False,
               row_stats: Optional[torch.Tensor] = None):
    """Residual-add + RMSNorm/LayerNorm + e4m3 quantisation (see b2f_norm_quant).

    ``q_scale=None`` selects the dynamic per-tensor scale amax(|y|)/448, returned in
    ``scale_out`` (f32 [1]).  With a dynamic scale, ``phase="stats"`` runs pass 1 only
    (h_out written, amax of these rows left in ``amax``) and ``phase="apply"`` runs pass 2
    only from the given ``amax`` (so row shards can share one scale after a MAX
    all-reduce).  ``schedule="rowgroup"`` forces the unstaged kernels.  ``row_stats``
    (f32 [rows, 2]) carries each row's (mean, rstd) from pass 1 to pass 2; a full dynamic
    call without it uses a per-device scratch buffer.
    Returns ``(q_out, scale_out)``; with ``query_schedule`` launches nothing and returns
    the schedule the call would use ("stream", "rowgroup" or "warp").
    """
    _check_cuda(x, weight, bias, residual, h_out, y_out, q_out, amax, scale_out)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be row-major 2-D")
    rows, cols = x.shape
    if q_out is None:
        q_out = torch.empty((rows, cols), device=x.device, dtype=torch.float8_e4m3fn)
    dynamic = q_scale is None
    if dynamic:
        if amax is None:
            amax = torch.zeros(1, device=x.device, dtype=torch.float32)
        if scale_out is None:
            scale_out = torch.empty(1, device=x.device, dtype=torch.float32)
    args = _lib.NormArgs()
    _lib.lib().b2f_norm_args_init(ctypes.byref(args))
    args.rows, args.cols = rows, cols
    args.x, args.x_dtype, args.x_scale, args.x_ld = x.data_ptr(), _DT[x.dtype], x_scale, x.stride(0)
    if residual is not None:
        args.residual, args.residual_dtype = residual.data_ptr(), _DT[residual.dtype]
        args.residual_ld = residual.stride(0)
    if weight.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("weight must be f32 or bf16")
    if bias is not None and bias.dtype != weight.dtype:
        raise TypeError("bias dtype must match weight dtype")
    args.weight, args.bias = weight.data_ptr(), _ptr(bias)
    args.weight_dtype, args.weight_offset = _DT[weight.dtype], weight_offset
    args.kind = {"rms": _lib.NORM_RMS, "layer": _lib.NORM_LAYER}[kind]
    args.eps = eps
    if h_out is not None:
        args.h_out, args.h_dtype, args.h_ld = h_out.data_ptr(), _DT[h_out.dtype], h_out.stride(0)
    if y_out is not None:
        if y_out.dtype != torch.bfloat16:
            raise TypeError("y_out must be bf16")
        args.y_out, args.y_ld = y_out.data_ptr(), y_out.stride(0)
    args.q_out, args.q_ld = q_out.data_ptr(), q_out.stride(0)
    args.q_scale = 1.0 if dynamic else float(q_scale)
    if not dynamic:
        if phase is not None:
            raise ValueError("phase applies to the dynamic scale only")
        args.dynamic_scale = _lib.SCALE_STATIC
    else:
        args.dynamic_scale = {None: _lib.SCALE_DYNAMIC, "stats": _lib.SCALE_DYNAMIC_STATS,
                              "apply": _lib.SCALE_DYNAMIC_APPLY}[phase]
    args.amax, args.scale_out = _ptr(amax), _ptr(scale_out)
    if row_stats is None and dynamic and phase is None:
        row_stats = _stats_scratch(rows, x.device)
    if row_stats is not None:
        _check_cuda(row_stats)
        if row_stats.dtype != torch.float32 or row_stats.numel() < 2 * rows:
            raise ValueError("row_stats must be f32 with room for [rows, 2]")
        args.row_stats = row_stats.data_ptr()
    args.schedule = {"auto": _lib.NORM_SCHEDULE_AUTO,
                     "rowgroup": _lib.NORM_SCHEDULE_ROWGROUP}[schedule]
    if query_schedule:
        rc = _lib.lib().b2f_norm_plan(ctypes.byref(args))
        if rc < 0:
            check(-rc)
        return {0: "stream", 1: "rowgroup", 2: "warp"}[rc]
    check(_lib.lib().b2f_norm_quant(ctypes.byref(args), _stream()))
    return q_out, scale_out


_LN_WS = {}


def layer_norm_rows(x: torch.Tensor, *, out: Optional[torch.Tensor] = None,
                    x_scale: float = 1.0, eps: float = 1e-5,
                    weight: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                    out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """LayerNorm over each row of a 2-D tensor with very long rows (b2f_layer_norm_rows):
    every row is split over many CTAs.  ``x`` e4m3 (value = stored * x_scale), bf16 or f32;
    ``out`` f32 or bf16; optional f32 ``weight`` / ``bias`` [cols]."""
    _check_cuda(x, out, weight, bias)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be a row-major 2-D tensor")
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), device=x.device, dtype=out_dtype)
    if out.shape != x.shape or out.stride(1) != 1:
        raise ValueError("out must match x's shape, row-major")
    for t, nm in ((weight, "weight"), (bias, "bias")):
        if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != cols):
            raise TypeError(f"{nm} must be contiguous float32 [cols]")
    L = _lib.lib()
    need = int(L.b2f_layer_norm_rows_workspace_bytes(rows, cols))
    key = x.device.index if x.device.index is not None else torch.cuda.current_device()
    ws = _LN_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty((max(need, 4096),), dtype=torch.uint8, device=x.device)
        _LN_WS[key] = ws
    a = _lib.LnRowsArgs()
    L.b2f_lnrows_args_init(ctypes.byref(a))
    a.rows, a.cols = rows, cols
    a.x, a.x_dtype, a.x_ld, a.x_scale = x.data_ptr(), _DT[x.dtype], x.stride(0), float(x_scale)
    a.weight, a.bias, a.eps = _ptr(weight), _ptr(bias), float(eps)
    a.out, a.out_dtype, a.out_ld = out.data_ptr(), _DT[out.dtype], out.stride(0)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    check(L.b2f_layer_norm_rows(ctypes.byref(a), _stream()))
    return out


def attention_fp8(q: torch.Tensor, k: torch.Tensor, v_bf16: torch.Tensor, *, batch: int,
                  heads: int, kv_heads: int, head_dim: int, causal: bool = True,
                  q_scale: float = 1.0, k_scale: float = 1.0, v_scale: float = 1.0,
                  sm_scale: float = 0.0, gate: Optional[torch.Tensor] = None,
                  gate_scale: float = 1.0, gate_head_stride: Optional[int] = None,
                  ctx: Optional[torch.Tensor] = None, ctx_scale: float = 1.0) -> torch.Tensor:
    """Fused attention (see b2f_attention_fp8).  q/k are e4m3 2-D [T, cols] views with head h
    at column h*head_dim (row pitch = stride(0)); v is bf16 or f16 [T, cols] (f16 selects
    the f16-probability path, head_dim 64 / 128); returns the e4m3 context
    [T, heads*head_dim]."""
    _check_cuda(q, k, v_bf16, gate, ctx)
    _fp8_rows(q, "q")
    _fp8_rows(k, "k")
    if (v_bf16.dtype not in (torch.bfloat16, torch.float16) or v_bf16.dim() != 2
            or v_bf16.stride(1) != 1):
        raise TypeError("v must be a row-major bf16 or f16 2-D tensor")
    t = q.shape[0]
    if t % batch:
        raise ValueError("token count must be batch * seq")
    if ctx is None:
        ctx = torch.empty((t, heads * head_dim), device=q.device, dtype=torch.float8_e4m3fn)
    a = _lib.AttnArgs()
    _lib.lib().b2f_attn_args_init(ctypes.byref(a))
    a.batch, a.seq, a.hq, a.hkv, a.head_dim = batch, t // batch, heads, kv_heads, head_dim
    a.causal = 1 if causal else 0
    a.q, a.q_ld, a.q_scale = q.data_ptr(), q.stride(0), q_scale
    a.k, a.k_ld, a.k_scale = k.data_ptr(), k.stride(0), k_scale
    a.v, a.v_ld, a.v_scale = v_bf16.data_ptr(), v_bf16.stride(0), v_scale
    a.v_dtype = _DT[v_bf16.dtype]
    a.sm_scale = sm_scale
    if gate is not None:
        if gate.dim() != 2 or gate.stride(1) != 1:
            raise ValueError("gate must be row-major 2-D")
        a.gate, a.gate_dtype, a.gate_ld = gate.data_ptr(), _DT[gate.dtype], gate.stride(0)
        a.gate_head_stride = head_dim if gate_head_stride is None else gate_head_stride
        a.gate_scale = gate_scale
    a.ctx, a.ctx_ld, a.ctx_scale = ctx.data_ptr(), ctx.stride(0), ctx_scale
    check(_lib.lib().b2f_attention_fp8(ctypes.byref(a), _stream()))
    return ctx


def _rope_args(x, heads, head_dim, in_scale, out_scale, head_stride, weight, weight_offset,
               eps, cos, sin, rotary_dim, seq, out):
    _check_cuda(x, weight, cos, sin, out)
    _fp8_rows(x, "x")
    rows = x.shape[0]
    if out is None:
        out = torch.empty((rows, heads * head_dim), device=x.device, dtype=torch.float8_e4m3fn)
    a = _lib.RopeArgs()
    a.rows, a.heads, a.head_dim = rows, heads, head_dim
    setattr(a, "in", x.data_ptr())
    a.in_ld = x.stride(0)
    a.in_head_stride = head_dim if head_stride is None else head_stride
    a.in_scale = in_scale
    if weight is not None and weight.dtype != torch.float32:
        raise TypeError("weight must be f32")
    a.weight, a.weight_offset, a.eps = _ptr(weight), weight_offset, eps
    a.cos, a.sin, a.rotary_dim, a.seq = _ptr(cos), _ptr(sin), rotary_dim, seq
    a.out, a.out_ld, a.out_scale = out.data_ptr(), out.stride(0), out_scale
    return a, out


def head_norm_rope(x: torch.Tensor, *, heads: int, head_dim: int, in_scale: float,
                   out_scale: float, head_stride: Optional[int] = None,
                   weight: Optional[torch.Tensor] = None, weight_offset: float = 1.0,
                   eps: float = 1e-6, cos: Optional[torch.Tensor] = None,
                   sin: Optional[torch.Tensor] = None, rotary_dim: int = 0, seq: int = 0,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-head RMSNorm (w + weight_offset) + rotate-half RoPE + e4m3 requantisation."""
    a, out = _rope_args(x, heads, head_dim, in_scale, out_scale, head_stride, weight,
                        weight_offset, eps, cos, sin, rotary_dim, seq, out)
    check(_lib.lib().b2f_head_norm_rope(ctypes.byref(a), _stream()))
    return out


def attn_prep(q_src: torch.Tensor, k_src: torch.Tensor, v_src: Optional[torch.Tensor], *,
              q_heads: int,
              k_heads: int, head_dim: int, in_scale: float, out_scale: float,
              q_head_stride: Optional[int] = None, q_weight=None, k_weight=None,
              weight_offset: float = 1.0, eps: float = 1e-6, cos=None, sin=None,
              rotary_dim: int = 0, seq: int = 0, q_out=None, k_out=None,
              v_out: torch.Tensor = None) -> bool:
    """q / k head norm + RoPE (as :func:`head_norm_rope`) and the e4m3 -> 16-bit V copy
    (as :func:`fp8_to_f16` / :func:`fp8_to_bf16`, by ``v_out``'s dtype) in one launch
    (b2f_attn_prep).  Returns False, having done nothing, for shapes that launch does not
    cover (the caller then runs the three operations)."""
    _check_cuda(v_src, v_out)
    if (v_src is None) != (v_out is None):
        raise ValueError("v_src and v_out go together (both None: no V copy)")
    qa, q_out = _rope_args(q_src, q_heads, head_dim, in_scale, out_scale, q_head_stride,
                           q_weight, weight_offset, eps, cos, sin, rotary_dim, seq, q_out)
    ka, k_out = _rope_args(k_src, k_heads, head_dim, in_scale, out_scale, None, k_weight,
                           weight_offset, eps, cos, sin, rotary_dim, seq, k_out)
    if v_src is None:
        vargs = (None, 0, None, 0, 0, _lib.DTYPE_F16)
    else:
        vargs = (v_src.data_ptr(), v_src.stride(0), v_out.data_ptr(), v_out.stride(0),
                 v_src.shape[1], _DT[v_out.dtype])
    rc = _lib.lib().b2f_attn_prep(ctypes.byref(qa), ctypes.byref(ka), *vargs, _stream())
    if rc == _lib.B2F_ERR_UNSUPPORTED:
        return False
    check(rc)
    return True


def quantize_fp8(x: torch.Tensor, *, scale: Optional[float] = None,
                 out: Optional[torch.Tensor] = None, amax: Optional[torch.Tensor] = None,
                 scale_out: Optional[torch.Tensor] = None,
                 scale_mul: Optional[torch.Tensor] = None,
                 scale_prod_out: Optional[torch.Tensor] = None):
    """Per-tensor e4m3 quantisation of an f32 / bf16 [rows, cols] tensor (see
    b2f_quantize_fp8).  ``scale=None`` selects s = amax(|x|) / 448, returned as an f32 [1]
    device tensor.  Returns ``(q, s)``."""
    _check_cuda(x, out, amax, scale_out, scale_mul, scale_prod_out)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be row-major 2-D")
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), device=x.device, dtype=torch.float8_e4m3fn)
    a = _lib.QuantArgs()
    _lib.lib().b2f_quant_args_init(ctypes.byref(a))
    a.rows, a.cols = rows, cols
    a.x, a.x_dtype, a.x_ld = x.data_ptr(), _DT[x.dtype], x.stride(0)
    a.q, a.q_ld = out.data_ptr(), out.stride(0)
    if scale is None:
        amax = torch.empty(1, device=x.device) if amax is None else amax
        scale_out = torch.empty(1, device=x.device) if scale_out is None else scale_out
        a.dynamic = 1
    else:
        a.scale = float(scale)
    a.amax, a.scale_out = _ptr(amax), _ptr(scale_out)
    a.scale_mul, a.scale_prod_out = _ptr(scale_mul), _ptr(scale_prod_out)
    check(_lib.lib().b2f_quantize_fp8(ctypes.byref(a), _stream()))
    return out, (scale_out if scale is None else scale)


def fp8_to_bf16(x: torch.Tensor, scale: float = 1.0,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 copy of an e4m3 [rows, cols] view (exact), times ``scale``."""
    _check_cuda(x, out)
    _fp8_rows(x, "x")
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), device=x.device, dtype=torch.bfloat16)
    check(_lib.lib().b2f_fp8_to_bf16(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0),
                                     rows, cols, scale, _stream()))
    return out


def fp8_to_f16(x: torch.Tensor, scale: float = 1.0,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """f16 copy of an e4m3 [rows, cols] view (exact), times ``scale``."""
    _check_cuda(x, out)
    _fp8_rows(x, "x")
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), device=x.device, dtype=torch.float16)
    check(_lib.lib().b2f_fp8_to_f16(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0),
                                    rows, cols, scale, _stream()))
    return out


def swiglu_fp8(gate: torch.Tensor, up: torch.Tensor, *, in_scale: float, out_scale: float,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """e4m3(silu(gate * s_in) * (up * s_in) / s_out) for e4m3 [rows, cols] views."""
    _check_cuda(gate, up, out)
    _fp8_rows(gate, "gate")
    _fp8_rows(up, "up")
    rows, cols = gate.shape
    if out is None:
        out = torch.empty((rows, cols), device=gate.device, dtype=torch.float8_e4m3fn)
    check(_lib.lib().b2f_swiglu_fp8(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0),
                                    out.data_ptr(), out.stride(0), rows, cols, in_scale,
                                    out_scale, _stream()))
    return out
