"""GPT-2-style and Qwen-style FP8 decoder blocks composed from the b200fp8 kernels.

Every stage is one of this library's sm_100a kernels; the block keeps its intermediate
tensors in preallocated device buffers so that a whole forward can be captured once into
a CUDA graph (``capture``) and replayed without per-launch host cost (``replay``).

GPT-2 block (tasks/model_gpt2_small_transformer_block_fp8/starter.py:114-140, reference
math :393-488), 8 launches:
  norm_quant(LN1) -> gemm(QKV + bias, e4m3) -> fp8_to_bf16(V) -> attention(causal)
  -> gemm(out-proj + bias + residual x) -> norm_quant(LN2) -> gemm(FC + bias, GELU-tanh,
  e4m3) -> gemm(proj + bias + residual r1)
Qwen full-attention block (tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:66-98,
reference math :333-416):
  norm_quant(RMSNorm 1+w) -> one fused gemm over [Wq | Wgate | Wk | Wv] with per-column
  scales -> head_norm_rope(q), head_norm_rope(k) -> fp8_to_bf16(V) -> attention(causal,
  GQA, sigmoid gate) -> gemm(o-proj + residual) [-> norm_quant -> gemm([Wgate|Wup])
  -> swiglu -> gemm(down + residual)]
Weights are passed as any object with the fields of the reference-style containers
(e4m3 weight tensors, float per-tensor scales, f32 vectors); they are copied to the
device once.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib, ops

_E4M3 = torch.float8_e4m3fn


def _dev(t: Optional[torch.Tensor], device, dtype=None) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = t.to(device=device)
    if dtype is not None:
        t = t.to(dtype)
    return t.contiguous()


def _gemm(*args, **kwargs):
    """The blocks' GEMMs run with one K slice: the native block entry points carry no
    split-K workspace, and the two forms of a block stay bit-identical."""
    return ops.gemm_fp8(*args, splits=1, **kwargs)


def _v_dtype(head_dim: int) -> torch.dtype:
    """V operand type of the blocks: f16 for head_dim 64 / 128, so the attention rounds P
    to f16 (2^-11 relative; measured as fast as bf16 P on B200, 179 us at the Qwen shape,
    with six times fewer requantised codes off by one), bf16 for head_dim 256.  Both hold
    the e4m3 values exactly."""
    return torch.float16 if head_dim <= 128 else torch.bfloat16


def _v_convert(src: torch.Tensor, dst: torch.Tensor) -> None:
    if dst.dtype == torch.float16:
        ops.fp8_to_f16(src, out=dst)
    else:
        ops.fp8_to_bf16(src, out=dst)


_DTC = {torch.float32: 0, torch.bfloat16: 1, torch.float8_e4m3fn: 2, torch.float16: 3}


def _mark(marks: Optional[list], name: str) -> None:
    """Stage boundary of an eager forward: records a CUDA event on the current stream when
    the caller collects per-stage timings (``marks`` is a list of (stage, event))."""
    if marks is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _block_workspace(owner, nbytes: int, device) -> torch.Tensor:
    ws = getattr(owner, "_abi_ws", None)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=device)
        owner._abi_ws = ws
    return ws


class _Graphable:
    """Capture/replay helper shared by the blocks."""

    def _init_graph(self):
        self._graph = None
        self._g_in = None
        self._g_out = None

    def capture(self, hidden: torch.Tensor, hidden_scale: float = 1.0) -> torch.Tensor:
        """Capture one forward on a side stream; later ``replay`` reruns it on the data
        currently in ``self.graph_input``.  Returns the graph's output buffer."""
        self._g_in = hidden.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self.forward(self._g_in, hidden_scale)  # warm caches outside the capture
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._g_out = self.forward(self._g_in, hidden_scale)
        torch.cuda.current_stream().wait_stream(s)
        self._graph = g
        return self._g_out

    @property
    def graph_input(self) -> torch.Tensor:
        return self._g_in

    def replay(self) -> torch.Tensor:
        self._graph.replay()
        return self._g_out

    def stage_times(self, hidden: torch.Tensor, hidden_scale: float = 1.0,
                    reps: int = 5) -> dict:
        """Mean device time (ms) of each stage of the forward, from CUDA events between the
        stages of eager forwards.  A device-side sleep is queued first so that the host has
        issued every launch before the GPU reaches them: the intervals are device time, not
        host launch gaps."""
        acc = {}
        for _ in range(reps):
            marks = []
            torch.cuda._sleep(4_000_000)
            self.forward(hidden, hidden_scale, marks=marks)
            torch.cuda.synchronize()
            for (_, e0), (name, e1) in zip(marks, marks[1:]):
                acc.setdefault(name, []).append(e0.elapsed_time(e1))
        return {k: sum(v) / len(v) for k, v in acc.items()}


class GPT2Block(_Graphable):

    def __init__(self, w, *, batch: int, seq: int, residual_dtype=torch.float32,
                 out_dtype=torch.float32, device="cuda", causal: bool = True,
                 rope_cos: Optional[torch.Tensor] = None,
                 rope_sin: Optional[torch.Tensor] = None):
        """``rope_cos/rope_sin`` [seq, head_dim] and ``causal=False`` give the Qwen vision
        block (tasks/model_qwen35_4b_vision_block_fp8): RoPE on q, k, non-causal."""
        self.batch, self.seq = batch, seq
        self.t = batch * seq
        self.causal = causal
        self.heads = w.heads
        self.d = w.qkv_w.shape[1]
        self.hd = self.d // self.heads
        self.mlp = w.fc_w.shape[0]
        self.eps = w.eps
        self.ns, self.qs, self.cs, self.ms = w.norm_scale, w.qkv_scale, w.ctx_scale, w.mlp_scale
        self.qkv_w, self.out_w = _dev(w.qkv_w, device), _dev(w.out_w, device)
        self.fc_w, self.proj_w = _dev(w.fc_w, device), _dev(w.proj_w, device)
        self.qkv_s, self.out_s, self.fc_s, self.proj_s = w.qkv_s, w.out_s, w.fc_s, w.proj_s
        f32 = torch.float32
        self.qkv_b, self.out_b = _dev(w.qkv_b, device, f32), _dev(w.out_b, device, f32)
        self.fc_b, self.proj_b = _dev(w.fc_b, device, f32), _dev(w.proj_b, device, f32)
        self.ln1_w, self.ln1_b = _dev(w.ln1_w, device, f32), _dev(w.ln1_b, device, f32)
        self.ln2_w, self.ln2_b = _dev(w.ln2_w, device, f32), _dev(w.ln2_b, device, f32)
        t, d = self.t, self.d
        self.n1 = torch.empty((t, d), device=device, dtype=_E4M3)
        self.qkv = torch.empty((t, 3 * d), device=device, dtype=_E4M3)
        self.v16 = torch.empty((t, d), device=device, dtype=_v_dtype(self.hd))
        self.ctx = torch.empty((t, d), device=device, dtype=_E4M3)
        self.r1 = torch.empty((t, d), device=device, dtype=residual_dtype)
        self.n2 = torch.empty((t, d), device=device, dtype=_E4M3)
        self.h = torch.empty((t, self.mlp), device=device, dtype=_E4M3)
        self.out = torch.empty((t, d), device=device, dtype=out_dtype)
        self.rope = rope_cos is not None
        if self.rope:
            self.cos = _dev(rope_cos[:seq], device, f32)
            self.sin = _dev(rope_sin[:seq], device, f32)
            self.q_rot = torch.empty((t, d), device=device, dtype=_E4M3)
            self.k_rot = torch.empty((t, d), device=device, dtype=_E4M3)
        # LN1, QKV GEMM (+ the V copy when d is a multiple of 128, else a separate launch),
        # [q / k RoPE], attention, out GEMM, LN2, FC GEMM, proj GEMM
        self.launches_per_forward = (7 if d % 128 == 0 and t >= 128 else 8) + \
            (2 if self.rope else 0)
        self._init_graph()

    def flops(self) -> float:
        t, d, m, s = self.t, self.d, self.mlp, self.seq
        gemm = 2 * t * (3 * d * d + d * d + 2 * d * m)
        attn = (2 if self.causal else 4) * self.batch * self.heads * s * s * self.hd
        return float(gemm + attn)

    def forward(self, hidden: torch.Tensor, hidden_scale: float = 1.0,
                marks: Optional[list] = None) -> torch.Tensor:
        """One forward; with ``marks`` (a list) every stage ends with a recorded CUDA event
        (eager per-stage timing; not for graph capture)."""
        d = self.d
        _mark(marks, "start")
        ops.norm_quant(hidden, self.ln1_w, kind="layer", bias=self.ln1_b, eps=self.eps,
                       x_scale=hidden_scale, q_out=self.n1, q_scale=self.ns)
        _mark(marks, "ln1")
        if d % 128 == 0 and self.t >= 128 and ops.gemm_fp8_head_prep(
                self.n1, self.qkv_w, scale_a=self.ns, scale_b=self.qkv_s, bias=self.qkv_b,
                out=self.qkv, out_scale=self.qs, q_out=None, k_out=None, v_out=self.v16,
                q_off=0, q_heads=0, k_off=0, k_heads=0, v_off=2 * d, v_heads=d // 128):
            # the 16-bit V image leaves the QKV GEMM's epilogue directly
            _mark(marks, "qkv_gemm_v")
        else:
            _gemm(self.n1, self.qkv_w, scale_a=self.ns, scale_b=self.qkv_s, bias=self.qkv_b,
                  out=self.qkv, out_scale=self.qs)
            _mark(marks, "qkv_gemm")
            _v_convert(self.qkv[:, 2 * d:], self.v16)
            _mark(marks, "v_convert")
        q, k = self.qkv[:, :d], self.qkv[:, d:2 * d]
        if self.rope:
            for src, dst in ((q, self.q_rot), (k, self.k_rot)):
                ops.head_norm_rope(src, heads=self.heads, head_dim=self.hd, in_scale=self.qs,
                                   out_scale=self.qs, cos=self.cos, sin=self.sin,
                                   rotary_dim=self.hd, seq=self.seq, out=dst)
            q, k = self.q_rot, self.k_rot
            _mark(marks, "rope")
        ops.attention_fp8(q, k, self.v16, batch=self.batch,
                          heads=self.heads, kv_heads=self.heads, head_dim=self.hd,
                          causal=self.causal,
                          q_scale=self.qs, k_scale=self.qs, v_scale=self.qs, ctx=self.ctx,
                          ctx_scale=self.cs)
        _mark(marks, "attention")
        _gemm(self.ctx, self.out_w, scale_a=self.cs, scale_b=self.out_s, bias=self.out_b,
              residual=hidden, residual_scale=hidden_scale, out=self.r1)
        _mark(marks, "out_gemm")
        ops.norm_quant(self.r1, self.ln2_w, kind="layer", bias=self.ln2_b, eps=self.eps,
                       q_out=self.n2, q_scale=self.ns)
        _mark(marks, "ln2")
        _gemm(self.n2, self.fc_w, scale_a=self.ns, scale_b=self.fc_s, bias=self.fc_b,
              act="gelu_tanh", out=self.h, out_scale=self.ms)
        _mark(marks, "fc_gemm")
        _gemm(self.h, self.proj_w, scale_a=self.ms, scale_b=self.proj_s, bias=self.proj_b,
              residual=self.r1, out=self.out)
        _mark(marks, "proj_gemm")
        return self.out

    def forward_abi(self, hidden: torch.Tensor, hidden_scale: float = 1.0) -> torch.Tensor:
        """The same forward through the native entry point b2f_gpt2_block (one C call;
        intermediates in a block-owned workspace); writes and returns ``self.out``."""
        a = _lib.Gpt2BlockArgs()
        L = _lib.lib()
        L.b2f_gpt2_block_args_init(ctypes.byref(a))
        a.batch, a.seq, a.d_model, a.heads, a.mlp = self.batch, self.seq, self.d, self.heads, self.mlp
        a.hidden, a.hidden_dtype, a.hidden_ld = hidden.data_ptr(), _DTC[hidden.dtype], hidden.stride(0)
        a.hidden_scale = hidden_scale
        a.qkv_w, a.qkv_s, a.qkv_b = _p(self.qkv_w), self.qkv_s, _p(self.qkv_b)
        a.out_w, a.out_s, a.out_b = _p(self.out_w), self.out_s, _p(self.out_b)
        a.fc_w, a.fc_s, a.fc_b = _p(self.fc_w), self.fc_s, _p(self.fc_b)
        a.proj_w, a.proj_s, a.proj_b = _p(self.proj_w), self.proj_s, _p(self.proj_b)
        a.ln1_w, a.ln1_b, a.ln2_w, a.ln2_b = _p(self.ln1_w), _p(self.ln1_b), _p(self.ln2_w), _p(self.ln2_b)
        a.eps = self.eps
        a.norm_scale, a.qkv_scale, a.ctx_scale, a.mlp_scale = self.ns, self.qs, self.cs, self.ms
        a.causal = 1 if self.causal else 0
        if self.rope:
            a.rope_cos, a.rope_sin = _p(self.cos), _p(self.sin)
        a.residual_dtype = _DTC[self.r1.dtype]
        a.out, a.out_dtype, a.out_ld = self.out.data_ptr(), _DTC[self.out.dtype], self.out.stride(0)
        ws = _block_workspace(self, int(L.b2f_gpt2_block_workspace_bytes(ctypes.byref(a))),
                              self.out.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        ops.check(L.b2f_gpt2_block(ctypes.byref(a), ops._stream()))
        return self.out


class QwenBlock(_Graphable):
    """``add_residual=False`` leaves the residual add out of the o-projection: the block then
    returns only this rank's partial of a heads-parallel o-projection (the other ranks'
    partials and the residual are summed by the caller's all-reduce)."""

    def __init__(self, w, *, batch: int, seq: int, residual_dtype=torch.float32,
                 out_dtype=torch.float32, device="cuda", add_residual: bool = True):
        self.batch, self.seq = batch, seq
        self.add_residual = add_residual
        self.t = t = batch * seq
        self.h, self.hk, self.dh = w.heads, w.kv_heads, w.head_dim
        self.hidden = w.q_w.shape[1]
        self.rot = w.rotary_dim
        self.eps = w.eps
        self.interleaved = w.interleaved
        self.ns, self.qs, self.cs = w.norm_scale, w.qkv_scale, w.ctx_scale
        self.mps, self.mas = w.mlp_proj_scale, w.mlp_act_scale
        h, hk, dh = self.h, self.hk, self.dh
        parts = [w.q_w] + ([] if w.interleaved else [w.gate_w]) + [w.k_w, w.v_w]
        scales = [w.q_s] + ([] if w.interleaved else [w.gate_s]) + [w.k_s, w.v_s]
        self.w_cat = torch.cat([p.to(device) for p in parts], dim=0).contiguous()
        self.cs_cat = torch.cat([torch.full((p.shape[0],), s * self.ns, dtype=torch.float32)
                                 for p, s in zip(parts, scales)]).to(device)
        qg = 2 * h * dh if w.interleaved else h * dh
        self.q_off, self.q_hstride = 0, (2 * dh if w.interleaved else dh)
        self.g_off = dh if w.interleaved else h * dh
        self.k_off = qg if w.interleaved else 2 * h * dh
        self.v_off = self.k_off + hk * dh
        self.n_cat = self.w_cat.shape[0]
        self.o_w, self.o_s = _dev(w.o_w, device), w.o_s
        f32 = torch.float32
        self.in_norm = _dev(w.in_norm_w, device, f32)
        self.q_norm, self.k_norm = _dev(w.q_norm_w, device, f32), _dev(w.k_norm_w, device, f32)
        self.cos = _dev(w.cos[:seq], device, f32)
        self.sin = _dev(w.sin[:seq], device, f32)
        self.has_mlp = w.mlp_down_w is not None
        if self.has_mlp and not add_residual:
            raise ValueError("add_residual=False needs a block without the MLP (the MLP "
                             "reads the full residual stream r1)")
        self.n1 = torch.empty((t, self.hidden), device=device, dtype=_E4M3)
        self.proj = torch.empty((t, self.n_cat), device=device, dtype=_E4M3)
        self.q = torch.empty((t, h * dh), device=device, dtype=_E4M3)
        self.k = torch.empty((t, hk * dh), device=device, dtype=_E4M3)
        self.v16 = torch.empty((t, hk * dh), device=device, dtype=_v_dtype(dh))
        self.ctx = torch.empty((t, h * dh), device=device, dtype=_E4M3)
        if self.has_mlp:
            self.r1 = torch.empty((t, self.hidden), device=device, dtype=residual_dtype)
            self.post_norm = _dev(w.post_norm_w, device, f32)
            self.inter = w.mlp_gate_w.shape[0]
            self.gu_w = torch.cat([w.mlp_gate_w.to(device), w.mlp_up_w.to(device)], 0).contiguous()
            self.gu_cs = torch.cat([
                torch.full((self.inter,), w.mlp_gate_s * self.ns, dtype=f32),
                torch.full((self.inter,), w.mlp_up_s * self.ns, dtype=f32)]).to(device)
            self.down_w, self.down_s = _dev(w.mlp_down_w, device), w.mlp_down_s
            self.n2 = torch.empty((t, self.hidden), device=device, dtype=_E4M3)
            self.gu = torch.empty((t, 2 * self.inter), device=device, dtype=_E4M3)
            self.act = torch.empty((t, self.inter), device=device, dtype=_E4M3)
        self.out = torch.empty((t, self.hidden), device=device, dtype=out_dtype)
        self._init_graph()

    @property
    def v_copy_in_gemm(self) -> bool:
        """The 16-bit V image leaves the projection GEMM's epilogue (b2f_gemm_fp8_head_prep
        with V blocks only: >= 256 tokens, V columns in whole 128-column blocks).  (The q / k
        norm + RoPE can run in that epilogue too, but measured slower than a separate
        launch: each epilogue thread owns one row, so its rotary-table loads do not
        coalesce.)"""
        return self.t >= 256 and (self.hk * self.dh) % 128 == 0 and self.v_off % 128 == 0

    @property
    def _qk_one_launch(self) -> bool:
        return (self.dh == 128 and self.h % 4 == 0 and self.hk % 4 == 0 and self.h <= 32
                and self.rot in (0, 128))

    @property
    def launches_per_forward(self) -> int:
        """Kernel launches of one forward: in-norm, projection GEMM, q / k (/ V)
        preparation (one b2f_attn_prep launch where it covers the shape, else one per
        operand), attention, o-projection, and the MLP's four."""
        if self._qk_one_launch:
            n = 5
        else:
            n = 6 if self.v_copy_in_gemm else 7
        return n + (4 if self.has_mlp else 0)

    def flops(self) -> float:
        t, hd = self.t, self.hidden
        gemm = 2 * t * hd * self.n_cat + 2 * t * self.h * self.dh * hd
        if self.has_mlp:
            gemm += 2 * t * hd * 2 * self.inter + 2 * t * self.inter * hd
        attn = 2 * self.batch * self.h * self.seq * self.seq * self.dh
        return float(gemm + attn)

    def _qk_prep(self, vsrc):
        """q / k head norm + RoPE, plus the V copy from ``vsrc`` unless it is None (V already
        written): one b2f_attn_prep launch where it covers the shape, else one per operand."""
        h, hk, dh = self.h, self.hk, self.dh
        fused = ops.attn_prep(
            self.proj[:, self.q_off:], self.proj[:, self.k_off:], vsrc, q_heads=h,
            k_heads=hk, head_dim=dh, in_scale=self.qs, out_scale=self.qs,
            q_head_stride=self.q_hstride, q_weight=self.q_norm, k_weight=self.k_norm,
            weight_offset=1.0, eps=self.eps, cos=self.cos, sin=self.sin,
            rotary_dim=self.rot, seq=self.seq, q_out=self.q, k_out=self.k,
            v_out=None if vsrc is None else self.v16)
        if not fused:
            ops.head_norm_rope(self.proj[:, self.q_off:], heads=h, head_dim=dh,
                               in_scale=self.qs, out_scale=self.qs, head_stride=self.q_hstride,
                               weight=self.q_norm, weight_offset=1.0, eps=self.eps,
                               cos=self.cos, sin=self.sin, rotary_dim=self.rot, seq=self.seq,
                               out=self.q)
            ops.head_norm_rope(self.proj[:, self.k_off:], heads=hk, head_dim=dh,
                               in_scale=self.qs, out_scale=self.qs, weight=self.k_norm,
                               weight_offset=1.0, eps=self.eps, cos=self.cos, sin=self.sin,
                               rotary_dim=self.rot, seq=self.seq, out=self.k)
            if vsrc is not None:
                _v_convert(vsrc, self.v16)

    def _qgkv_unfused(self, marks):
        """Projection GEMM, then the q / k / V preparations (one b2f_attn_prep launch where
        it covers the shape, else three)."""
        h, hk, dh = self.h, self.hk, self.dh
        _gemm(self.n1, self.w_cat, col_scale=self.cs_cat, out=self.proj,
              out_scale=self.qs)
        _mark(marks, "qgkv_gemm")
        self._qk_prep(self.proj[:, self.v_off:self.v_off + hk * dh])
        _mark(marks, "qkv_prep")

    def forward(self, hidden: torch.Tensor, hidden_scale: float = 1.0,
                marks: Optional[list] = None) -> torch.Tensor:
        """One forward; with ``marks`` (a list) every stage ends with a recorded CUDA event
        (eager per-stage timing; not for graph capture)."""
        h, hk, dh = self.h, self.hk, self.dh
        _mark(marks, "start")
        ops.norm_quant(hidden, self.in_norm, kind="rms", weight_offset=1.0, eps=self.eps,
                       x_scale=hidden_scale, q_out=self.n1, q_scale=self.ns)
        _mark(marks, "in_norm")
        if self.v_copy_in_gemm and ops.gemm_fp8_head_prep(
                self.n1, self.w_cat, col_scale=self.cs_cat, out=self.proj, out_scale=self.qs,
                q_out=None, k_out=None, v_out=self.v16, q_off=0, q_heads=0, k_off=0,
                k_heads=0, v_off=self.v_off, v_heads=hk * dh // 128):
            _mark(marks, "qgkv_gemm_v")
            self._qk_prep(None)
            _mark(marks, "qk_prep")
        else:
            self._qgkv_unfused(marks)
        ops.attention_fp8(self.q, self.k, self.v16, batch=self.batch, heads=h, kv_heads=hk,
                          head_dim=dh, causal=True, q_scale=self.qs, k_scale=self.qs,
                          v_scale=self.qs, gate=self.proj[:, self.g_off:], gate_scale=self.qs,
                          gate_head_stride=self.q_hstride, ctx=self.ctx, ctx_scale=self.cs)
        _mark(marks, "attention")
        r1 = self.r1 if self.has_mlp else self.out
        _gemm(self.ctx, self.o_w, scale_a=self.cs, scale_b=self.o_s,
              residual=hidden if self.add_residual else None,
              residual_scale=hidden_scale, out=r1)
        _mark(marks, "o_gemm")
        if not self.has_mlp:
            return self.out
        ops.norm_quant(r1, self.post_norm, kind="rms", weight_offset=1.0, eps=self.eps,
                       q_out=self.n2, q_scale=self.ns)
        _gemm(self.n2, self.gu_w, col_scale=self.gu_cs, out=self.gu, out_scale=self.mps)
        ops.swiglu_fp8(self.gu[:, :self.inter], self.gu[:, self.inter:], in_scale=self.mps,
                       out_scale=self.mas, out=self.act)
        _gemm(self.act, self.down_w, scale_a=self.mas, scale_b=self.down_s, residual=r1,
              out=self.out)
        _mark(marks, "mlp")
        return self.out

    def forward_abi(self, hidden: torch.Tensor, hidden_scale: float = 1.0) -> torch.Tensor:
        """The same forward through the native entry point b2f_qwen_block; writes and
        returns ``self.out``."""
        a = _lib.QwenBlockArgs()
        L = _lib.lib()
        L.b2f_qwen_block_args_init(ctypes.byref(a))
        a.batch, a.seq, a.hidden = self.batch, self.seq, self.hidden
        a.heads, a.kv_heads, a.head_dim, a.rotary_dim = self.h, self.hk, self.dh, self.rot
        a.interleaved = 1 if self.interleaved else 0
        a.hidden_in, a.hidden_dtype, a.hidden_ld = hidden.data_ptr(), _DTC[hidden.dtype], hidden.stride(0)
        a.hidden_scale = hidden_scale
        a.qgkv_w, a.qgkv_col_scale = _p(self.w_cat), _p(self.cs_cat)
        a.o_w, a.o_s = _p(self.o_w), self.o_s
        a.in_norm_w, a.q_norm_w, a.k_norm_w = _p(self.in_norm), _p(self.q_norm), _p(self.k_norm)
        a.rope_cos, a.rope_sin = _p(self.cos), _p(self.sin)
        a.eps, a.norm_scale, a.qkv_scale, a.ctx_scale = self.eps, self.ns, self.qs, self.cs
        a.add_residual = 1 if self.add_residual else 0
        if self.has_mlp:
            a.post_norm_w, a.mlp_gu_w, a.mlp_gu_col_scale = _p(self.post_norm), _p(self.gu_w), _p(self.gu_cs)
            a.inter, a.mlp_down_w, a.mlp_down_s = self.inter, _p(self.down_w), self.down_s
            a.mlp_proj_scale, a.mlp_act_scale = self.mps, self.mas
            a.residual_dtype = _DTC[self.r1.dtype]
        a.out, a.out_dtype, a.out_ld = self.out.data_ptr(), _DTC[self.out.dtype], self.out.stride(0)
        ws = _block_workspace(self, int(L.b2f_qwen_block_workspace_bytes(ctypes.byref(a))),
                              self.out.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        ops.check(L.b2f_qwen_block(ctypes.byref(a), ops._stream()))
        return self.out
