"""KernelBench-style task modules for BASELINE's five configs (the KernelEvo contract).

KernelEvo evaluates a task as ``Model(*get_init_inputs())(*get_inputs())`` against
``ModelNew(*get_init_inputs())(*get_inputs())`` with ``torch.allclose(atol, rtol)``
(kernel_evo_archive/source/src/kernel_evo/core/eval/eval.py:190-245, 813-950).  Here:

- ``Model`` classes are the torch reference of each task (the reference evaluators'
  math: ``torch._scaled_mm`` for every FP8 linear, f32 LayerNorm / RMSNorm / softmax),
  run by torch on the GPU.  They are the side the candidate is checked against.
- ``ModelNew`` classes run only this library's sm_100a kernels (``b200fp8.ops`` /
  ``b200fp8.blocks``).  Both share the same seeded weights.
- ``TASKS[name]`` bundles ``Model``, ``ModelNew``, ``get_inputs``, ``get_init_inputs`` and
  the tolerance; ``task_source(name)`` renders the two source strings KernelEvo loads
  (the reference module it ``exec``s and the ``ModelNew`` module it imports).

Weights and inputs are seeded and drawn on the CPU generator (BASELINE: N(0,1)
activations, N(0, 0.02) weights, per-tensor amax e4m3 scales), then moved to the GPU.
"""
from __future__ import annotations

import math
from types import SimpleNamespace

import torch
import torch.nn.functional as F

from . import blocks, ops

E4M3 = torch.float8_e4m3fn


def _q_amax(x: torch.Tensor):
    s = float(x.abs().max()) / 448.0
    return (x / s).to(E4M3), s


def _q8(v: torch.Tensor, s: float) -> torch.Tensor:
    """e4m3 requantisation with saturation (the kernels' cvt.rn.satfinite)."""
    return (v / s).clamp(-448.0, 448.0).to(E4M3)


def _nq(shape, g, std=0.02):
    return _q_amax(torch.randn(shape, generator=g) * std)


def _scaled_linear(x_q, w_q, sx, sw, out_dtype=torch.float32):
    dev = x_q.device
    return torch._scaled_mm(x_q, w_q.t(), scale_a=torch.tensor(sx, device=dev),
                            scale_b=torch.tensor(sw, device=dev), out_dtype=out_dtype)


# ----------------------------------------------------------------------------- GEMMs
class SquareGemm(torch.nn.Module):
    """C = A . B^T, e4m3 A, B [n, n], bf16 out."""

    def forward(self, a, b, scale_a, scale_b):
        return _scaled_linear(a, b, float(scale_a), float(scale_b), torch.bfloat16)


class SquareGemmNew(SquareGemm):
    def forward(self, a, b, scale_a, scale_b):
        return ops.gemm_fp8(a, b, scale_a=float(scale_a), scale_b=float(scale_b))


def _square_inputs(n=4096, seed=20260726):
    g = torch.Generator().manual_seed(seed)
    a, sa = _q_amax(torch.randn((n, n), generator=g))
    b, sb = _q_amax(torch.randn((n, n), generator=g))
    return [a.cuda(), b.cuda(), torch.tensor(sa), torch.tensor(sb)]


class GemmBiasRelu(torch.nn.Module):
    """Y = relu(X . W^T + bias), X [128, 8192], W [8192, 8192]."""

    def __init__(self, in_features=8192, out_features=8192, seed=20260726):
        super().__init__()
        g = torch.Generator().manual_seed(seed + 1)
        w, self.sw = _q_amax(torch.randn((out_features, in_features), generator=g) * 0.1)
        self.register_buffer("w", w)
        self.register_buffer("bias", torch.randn((out_features,), generator=g) * 0.02)

    def forward(self, x, scale_x):
        y = _scaled_linear(x, self.w, float(scale_x), self.sw) + self.bias
        return torch.relu(y).to(torch.bfloat16)


class GemmBiasReluNew(GemmBiasRelu):
    def forward(self, x, scale_x):
        return ops.gemm_fp8(x, self.w, scale_a=float(scale_x), scale_b=self.sw, bias=self.bias,
                            act="relu")


def _skinny_inputs(m=128, k=8192, seed=20260726):
    g = torch.Generator().manual_seed(seed)
    x, sx = _q_amax(torch.randn((m, k), generator=g) * 0.1)
    return [x.cuda(), torch.tensor(sx)]


# ----------------------------------------------------------------------------- norm
class ResidualRMSNormQuant(torch.nn.Module):
    """h = x + r (bf16), y = RMSNorm(h) * gamma (eps 1e-6),
    q = e4m3(y / s) with s = amax(|y|) / 448.  Returns (dequantised q, h)."""

    def __init__(self, hidden=4096, seed=20260731):
        super().__init__()
        g = torch.Generator().manual_seed(seed + 1)
        self.register_buffer("gamma", (1 + 0.02 * torch.randn((hidden,), generator=g)).to(torch.bfloat16))
        self.eps = 1e-6

    def forward(self, x, residual):
        h = (x.float() + residual.float()).to(torch.bfloat16)
        hf = h.float()
        y = (hf * torch.rsqrt(hf.square().mean(-1, keepdim=True) + self.eps) *
             self.gamma.float()).to(torch.bfloat16).float()
        s = y.abs().max() / 448.0
        q = (y / s).to(E4M3)
        return q.float() * s, h


class ResidualRMSNormQuantNew(ResidualRMSNormQuant):
    def forward(self, x, residual):
        h = torch.empty_like(x)
        q, s = ops.norm_quant(x, self.gamma, residual=residual, h_out=h, eps=self.eps)
        return q.float() * s, h


def _norm_inputs(rows=16384, cols=4096, seed=20260731):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((rows, cols), generator=g).to(torch.bfloat16)
    r = torch.randn((rows, cols), generator=g).to(torch.bfloat16)
    return [x.cuda(), r.cuda()]


# ----------------------------------------------------------------------------- blocks
def _gpt2_weights(seed, d=768, mlp=3072):
    g = torch.Generator().manual_seed(seed)
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


def _attention_ref(q, k, v, batch, causal, gate=None):
    """f32 softmax attention per sequence: q [T, H, D], k/v [T, Hkv, D]."""
    t, h, d = q.shape
    s = t // batch
    rep = h // k.shape[1]
    out = []
    for b in range(batch):
        sl = slice(b * s, (b + 1) * s)
        qb = q[sl].transpose(0, 1)
        kb = k[sl].repeat_interleave(rep, dim=1).transpose(0, 1)
        vb = v[sl].repeat_interleave(rep, dim=1).transpose(0, 1)
        o = F.scaled_dot_product_attention(qb, kb, vb, is_causal=causal,
                                           scale=1.0 / math.sqrt(d))
        out.append(o.transpose(0, 1))
    o = torch.cat(out, 0)
    return o if gate is None else o * torch.sigmoid(gate)


class GPT2BlockModel(torch.nn.Module):
    """GPT-2-small block, B x S tokens, bf16 residual stream; the
    reference evaluator's quantisation points
    (tasks/model_gpt2_small_transformer_block_fp8/starter.py:393-488)."""

    def __init__(self, batch=8, seq=1024, seed=20260801):
        super().__init__()
        self.batch, self.seq = batch, seq
        self.w = _gpt2_weights(seed)
        for k, v in vars(self.w).items():
            if torch.is_tensor(v):
                setattr(self.w, k, v.cuda())

    def forward(self, hidden):
        w = self.w
        t, d = hidden.shape
        x = hidden.float()
        q = _q8
        n1 = q(F.layer_norm(x, (d,), w.ln1_w, w.ln1_b, w.eps), w.norm_scale)
        qkv = q(_scaled_linear(n1, w.qkv_w, w.norm_scale, w.qkv_s) + w.qkv_b, w.qkv_scale)
        qkv = (qkv.float() * w.qkv_scale).view(t, 3, w.heads, d // w.heads)
        ctx = _attention_ref(qkv[:, 0], qkv[:, 1], qkv[:, 2], self.batch, True)
        ctx = q(ctx.reshape(t, d), w.ctx_scale)
        r1 = (x + _scaled_linear(ctx, w.out_w, w.ctx_scale, w.out_s) + w.out_b).to(torch.bfloat16)
        n2 = q(F.layer_norm(r1.float(), (d,), w.ln2_w, w.ln2_b, w.eps), w.norm_scale)
        fc = _scaled_linear(n2, w.fc_w, w.norm_scale, w.fc_s) + w.fc_b
        m = q(F.gelu(fc, approximate="tanh"), w.mlp_scale)
        out = r1.float() + _scaled_linear(m, w.proj_w, w.mlp_scale, w.proj_s) + w.proj_b
        return out.to(torch.bfloat16)


class GPT2BlockNew(GPT2BlockModel):
    def __init__(self, batch=8, seq=1024, seed=20260801):
        super().__init__(batch, seq, seed)
        self.blk = blocks.GPT2Block(self.w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                                    out_dtype=torch.bfloat16)

    def forward(self, hidden):
        return self.blk.forward(hidden)


def _qwen_weights(seed, seq, hidden=2560, heads=32, kv_heads=8, hd=128, theta=1e6):
    g = torch.Generator().manual_seed(seed)
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


class QwenBlockModel(torch.nn.Module):
    """Qwen gated full-attention block, B x S tokens, 32q / 8kv x 128,
    RMSNorm(1+w) on the input and on q, k; RoPE theta 1e6; sigmoid gate from a separate
    projection; bf16 residual (quantisation points of
    tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-392)."""

    def __init__(self, batch=4, seq=2048, seed=20260801):
        super().__init__()
        self.batch, self.seq = batch, seq
        self.w = _qwen_weights(seed, seq)
        for k, v in vars(self.w).items():
            if torch.is_tensor(v):
                setattr(self.w, k, v.cuda())

    def forward(self, hidden):
        w = self.w
        t, hid = hidden.shape
        h, hk, d = w.heads, w.kv_heads, w.head_dim
        x = hidden.float()
        q8 = _q8
        dq = lambda v, s: v.float() * s  # noqa: E731

        def rms(v, wt):
            return v * torch.rsqrt(v.square().mean(-1, keepdim=True) + w.eps) * (1.0 + wt)

        def rope(v):
            cos = w.cos.repeat(self.batch, 1)[:, None, :]
            sin = w.sin.repeat(self.batch, 1)[:, None, :]
            half = d // 2
            rot = torch.cat((-v[..., half:], v[..., :half]), dim=-1)
            return v * cos + rot * sin

        n1 = q8(rms(x, w.in_norm_w), w.norm_scale)
        qs = w.qkv_scale
        lin = lambda wt, s: dq(q8(_scaled_linear(n1, wt, w.norm_scale, s), qs), qs)  # noqa: E731
        qq = lin(w.q_w, w.q_s).view(t, h, d)
        gate = lin(w.gate_w, w.gate_s).view(t, h, d)
        kk = lin(w.k_w, w.k_s).view(t, hk, d)
        vv = lin(w.v_w, w.v_s).view(t, hk, d)
        qq = dq(q8(rope(rms(qq, w.q_norm_w)), qs), qs)
        kk = dq(q8(rope(rms(kk, w.k_norm_w)), qs), qs)
        ctx = _attention_ref(qq, kk, vv, self.batch, True, gate)
        ctx = q8(ctx.reshape(t, h * d), w.ctx_scale)
        return (x + _scaled_linear(ctx, w.o_w, w.ctx_scale, w.o_s)).to(torch.bfloat16)


class QwenBlockNew(QwenBlockModel):
    def __init__(self, batch=4, seq=2048, seed=20260801):
        super().__init__(batch, seq, seed)
        self.blk = blocks.QwenBlock(self.w, batch=batch, seq=seq, residual_dtype=torch.bfloat16,
                                    out_dtype=torch.bfloat16)

    def forward(self, hidden):
        return self.blk.forward(hidden)


def _hidden_inputs(tokens, hidden, seed=20260801):
    g = torch.Generator().manual_seed(seed + 7)
    return [torch.randn((tokens, hidden), generator=g).to(torch.bfloat16).cuda()]


# ----------------------------------------------------------------------------- registry
TASKS = {
    "gemm_bias_relu_fp8": dict(Model=GemmBiasRelu, ModelNew=GemmBiasReluNew,
                               get_init_inputs=lambda: [8192, 8192],
                               get_inputs=lambda: _skinny_inputs(), atol=0.05, rtol=2 ** -7),
    "square_gemm_fp8": dict(Model=SquareGemm, ModelNew=SquareGemmNew,
                            get_init_inputs=lambda: [], get_inputs=lambda: _square_inputs(),
                            atol=0.5, rtol=2 ** -7),
    "residual_rmsnorm_quant_fp8": dict(Model=ResidualRMSNormQuant,
                                       ModelNew=ResidualRMSNormQuantNew,
                                       get_init_inputs=lambda: [4096],
                                       get_inputs=lambda: _norm_inputs(), atol=0.3, rtol=0.07),
    "gpt2_block_fp8": dict(Model=GPT2BlockModel, ModelNew=GPT2BlockNew,
                           get_init_inputs=lambda: [8, 1024],
                           get_inputs=lambda: _hidden_inputs(8 * 1024, 768),
                           atol=0.06, rtol=2 ** -7),
    "qwen_attention_block_fp8": dict(Model=QwenBlockModel, ModelNew=QwenBlockNew,
                                     get_init_inputs=lambda: [4, 2048],
                                     get_inputs=lambda: _hidden_inputs(4 * 2048, 2560),
                                     atol=0.08, rtol=2 ** -7),
}

_CLASS = {"gemm_bias_relu_fp8": ("GemmBiasRelu", "GemmBiasReluNew"),
          "square_gemm_fp8": ("SquareGemm", "SquareGemmNew"),
          "residual_rmsnorm_quant_fp8": ("ResidualRMSNormQuant", "ResidualRMSNormQuantNew"),
          "gpt2_block_fp8": ("GPT2BlockModel", "GPT2BlockNew"),
          "qwen_attention_block_fp8": ("QwenBlockModel", "QwenBlockNew")}


def task_source(name: str):
    """(reference source, ModelNew source) in the form KernelEvo loads: the first defines
    Model / get_inputs / get_init_inputs and the per-task ``output_atol`` / ``output_rtol``
    globals that its evaluator reads (eval.py:525-536), the second defines ModelNew."""
    ref_cls, new_cls = _CLASS[name]
    ref = ("from b200fp8 import kernelbench as _kb\n"
           f"Model = _kb.{ref_cls}\n"
           f"get_inputs = _kb.TASKS[{name!r}]['get_inputs']\n"
           f"get_init_inputs = _kb.TASKS[{name!r}]['get_init_inputs']\n"
           f"output_atol = {TASKS[name]['atol']!r}\n"
           f"output_rtol = {TASKS[name]['rtol']!r}\n")
    new = "from b200fp8 import kernelbench as _kb\n" f"ModelNew = _kb.{new_cls}\n"
    return ref, new
