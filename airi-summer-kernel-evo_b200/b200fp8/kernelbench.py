"""KernelBench-style task modules for BASELINE's five configs (the KernelEvo contract).

KernelEvo evaluates a task source defining ``Model``, ``get_inputs`` and
``get_init_inputs`` (plus optional ``output_atol`` / ``output_rtol`` globals) against a
candidate defining ``ModelNew`` (kernel_evo_archive/source/src/kernel_evo/core/eval/eval.py:
418-439, 525-536, 590-606, 840-900):

- it seeds the global RNG, builds ``Model(*init)`` and ``ModelNew(*init)`` (so both draw the
  same weights), moves both with ``.to(device=..., dtype=precision)``;
- per trial it seeds again, calls ``get_inputs()``, casts every tensor input to
  ``precision`` and moves it to the device;
- it compares the single output tensor with ``torch.allclose(expected, actual, atol, rtol)``
  and requires it to be finite.

Everything here survives that contract: inputs are float tensors drawn from the global RNG,
and weights are registered buffers holding e4m3-exact values (every e4m3 value is exact in
fp32, bf16 and fp16, so a dtype cast of the module leaves them intact) with per-tensor
scales kept as Python floats.

- ``Model`` classes are the torch reference of each task: the GEMM tasks dequantise both
  e4m3 operands to f32 and multiply in f32 (BASELINE's GEMM reference), the blocks follow
  the reference evaluators' math (``torch._scaled_mm`` for every FP8 linear, f32 RMSNorm /
  LayerNorm / softmax).
- ``ModelNew`` classes run this library's sm_100a kernels only (``b200fp8.ops`` /
  ``b200fp8.blocks``); activations are quantised on the device by ``quantize_fp8``.
- ``TASKS[name]`` bundles the pieces and tolerances; ``task_source(name)`` renders the two
  source strings KernelEvo loads.

Tolerances: GEMM outputs are bf16 (rtol 2^-7 = one bf16 ulp); requantised e4m3 outputs
compare within one e4m3 step (rtol 2^-3); the block outputs use the reference evaluators'
absolute thresholds (GPT-2 0.05, Qwen 0.08) plus one bf16 ulp.
"""
from __future__ import annotations

import math
from types import SimpleNamespace

import torch
import torch.nn.functional as F

from . import blocks, ops

E4M3 = torch.float8_e4m3fn


def _codes_amax(w: torch.Tensor):
    """e4m3 quantisation with a per-tensor amax scale; returns (f32 values of the stored
    e4m3 codes, scale)."""
    s = float(w.abs().max()) / 448.0
    return (w / s).to(E4M3).float(), s


def _q8(v: torch.Tensor, s) -> torch.Tensor:
    """e4m3 requantisation with saturation (the kernels' cvt.rn.satfinite)."""
    return (v / s).clamp(-448.0, 448.0).to(E4M3)


def _fdiv(a: torch.Tensor, b: float) -> torch.Tensor:
    """a / b with IEEE division on any device (torch multiplies by the reciprocal when a CUDA
    tensor is divided by a Python number, which can differ in the last bit)."""
    return a / torch.full_like(a, b)


def _q_dynamic(x: torch.Tensor):
    """Reference of the per-tensor amax quantisation of an activation."""
    xf = x.float()
    s = _fdiv(xf.abs().max(), 448.0)
    s = torch.where(s > 0, s, torch.ones_like(s))
    return (xf / s).to(E4M3), s


def _dequant_linear(x_q, w_q, sx, sw):
    """f32 reference of an FP8 linear: dequantise both operands to f32, f32 matmul (the
    BASELINE GEMM configs' "Torch reference dequantises to fp32")."""
    sx = sx.reshape(()).float() if torch.is_tensor(sx) else float(sx)
    sw = sw.reshape(()).float() if torch.is_tensor(sw) else float(sw)
    with _no_tf32():
        return (x_q.float() * sx) @ (w_q.float() * sw).t()


class _no_tf32:
    def __enter__(self):
        self.prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self.prev


def _scaled_linear(x_q, w_q, sx, sw, out_dtype=torch.float32):
    dev = x_q.device
    sx = sx.reshape(()).float() if torch.is_tensor(sx) else torch.tensor(float(sx), device=dev)
    sw = sw.reshape(()).float() if torch.is_tensor(sw) else torch.tensor(float(sw), device=dev)
    return torch._scaled_mm(x_q, w_q.t(), scale_a=sx, scale_b=sw, out_dtype=out_dtype)


class _Fp8Module(torch.nn.Module):
    """Holds e4m3 weights as buffers of their exact values; ``_e4m3(name)`` returns the e4m3
    tensor on the buffer's current device (cached until the buffer changes)."""

    def _add_weight(self, name, w: torch.Tensor):
        codes, s = _codes_amax(w)
        self.register_buffer(name, codes)
        setattr(self, name + "_s", s)

    def _e4m3(self, name):
        buf = getattr(self, name)
        cache = self.__dict__.setdefault("_e4m3_cache", {})
        key = (buf.data_ptr(), buf.device, buf.dtype, buf._version)
        hit = cache.get(name)
        if hit is None or hit[0] != key:
            hit = (key, buf.to(E4M3).contiguous())
            cache[name] = hit
        return hit[1]


# ----------------------------------------------------------------------------- GEMMs
class SquareGemm(torch.nn.Module):
    """C = A . B^T (B stored [N, K], the reference's matrix_b_nk
    layout), A and B quantised to e4m3 with per-tensor amax scales, f32 accumulation,
    bf16 output."""

    def forward(self, a, b):
        qa, sa = _q_dynamic(a)
        qb, sb = _q_dynamic(b)
        return _dequant_linear(qa, qb, sa, sb).to(torch.bfloat16)


class SquareGemmNew(SquareGemm):
    def forward(self, a, b):
        qa, sa = ops.quantize_fp8(a)
        prod = torch.empty(1, device=a.device)
        qb, _ = ops.quantize_fp8(b, scale_mul=sa, scale_prod_out=prod)
        return ops.gemm_fp8(qa, qb, alpha_tensor=prod)


def _square_inputs(n=4096):
    return [torch.randn(n, n), torch.randn(n, n)]


class GemmBiasRelu(_Fp8Module):
    """Y = relu(X . W^T + bias), X [128, 8192] and W [8192, 8192]
    quantised from N(0,1) x 0.1 with per-tensor scales, bias N(0, 0.02), bf16 output."""

    def __init__(self, in_features=8192, out_features=8192):
        super().__init__()
        self._add_weight("w", torch.randn(out_features, in_features) * 0.1)
        self.register_buffer("bias", torch.randn(out_features) * 0.02)

    def forward(self, x):
        qx, sx = _q_dynamic(x)
        y = _dequant_linear(qx, self._e4m3("w"), sx, self.w_s) + self.bias.float()
        return torch.relu(y).to(torch.bfloat16)


class GemmBiasReluNew(GemmBiasRelu):
    def forward(self, x):
        qx, sx = ops.quantize_fp8(x)
        return ops.gemm_fp8(qx, self._e4m3("w"), scale_b=self.w_s, alpha_tensor=sx,
                            bias=self.bias.float(), act="relu")


def _skinny_inputs(m=128, k=8192):
    return [torch.randn(m, k) * 0.1]


# ----------------------------------------------------------------------------- norm
class ResidualRMSNormQuant(torch.nn.Module):
    """h = bf16(x + residual), y = bf16(RMSNorm(h) * gamma) (eps 1e-6),
    q = e4m3(y / s) with s = amax(|y|) / 448.  Returns [2, rows, cols] f32: the dequantised
    q (q * s) and the updated residual stream h."""

    def __init__(self, hidden=4096):
        super().__init__()
        self.register_buffer("gamma", (1 + 0.02 * torch.randn(hidden)).to(torch.bfloat16).float())
        self.eps = 1e-6

    def forward(self, x, residual):
        h = (x.float() + residual.float()).to(torch.bfloat16)
        hf = h.float()
        y = (hf * torch.rsqrt(hf.square().mean(-1, keepdim=True) + self.eps) *
             self.gamma.float()).to(torch.bfloat16).float()
        s = _fdiv(y.abs().max(), 448.0)
        q = (y / s).to(E4M3)
        return torch.stack((q.float() * s, hf))


class ResidualRMSNormQuantNew(ResidualRMSNormQuant):
    def forward(self, x, residual):
        h = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
        q, s = ops.norm_quant(x, self.gamma.float(), residual=residual, h_out=h, eps=self.eps)
        return torch.stack((q.float() * s, h.float()))


def _norm_inputs(rows=16384, cols=4096):
    return [torch.randn(rows, cols), torch.randn(rows, cols)]


# ----------------------------------------------------------------------------- blocks
def _attention_ref(q, k, v, batch, causal, gate=None):
    """f32 softmax attention per sequence: q [T, H, D], k/v [T, Hkv, D] (GQA)."""
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


_SCALES = dict(norm_scale=1 / 64.0, qkv_scale=1 / 64.0, ctx_scale=1 / 64.0, mlp_scale=1 / 64.0)


class GPT2BlockModel(_Fp8Module):
    """GPT-2-small block (d 768, 12 x 64 heads, MLP 3072, tanh-GELU,
    pre-LayerNorm, causal attention, biases on every linear), B x S tokens, f32 input,
    bf16 residual stream and output; the reference evaluator's quantisation points
    (tasks/model_gpt2_small_transformer_block_fp8/starter.py:393-488)."""

    def __init__(self, batch=8, seq=1024, d=768, mlp=3072, heads=12):
        super().__init__()
        self.batch, self.seq, self.heads, self.eps = batch, seq, heads, 1e-5
        for name, shape in (("qkv_w", (3 * d, d)), ("out_w", (d, d)), ("fc_w", (mlp, d)),
                            ("proj_w", (d, mlp))):
            self._add_weight(name, torch.randn(shape) * 0.02)
        b = lambda n: torch.randn(n) * 0.02  # noqa: E731
        for name, n in (("qkv_b", 3 * d), ("out_b", d), ("fc_b", mlp), ("proj_b", d)):
            self.register_buffer(name, b(n))
        self.register_buffer("ln1_w", 1 + b(d))
        self.register_buffer("ln1_b", b(d))
        self.register_buffer("ln2_w", 1 + b(d))
        self.register_buffer("ln2_b", b(d))

    def _weights(self):
        w = SimpleNamespace(heads=self.heads, eps=self.eps, **_SCALES)
        for name in ("qkv_w", "out_w", "fc_w", "proj_w"):
            setattr(w, name, self._e4m3(name))
            setattr(w, name[:-2] + "_s", getattr(self, name + "_s"))
        for name in ("qkv_b", "out_b", "fc_b", "proj_b", "ln1_w", "ln1_b", "ln2_w", "ln2_b"):
            setattr(w, name, getattr(self, name).float())
        return w

    def forward(self, hidden):
        w = self._weights()
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
    def forward(self, hidden):
        key = (hidden.device, tuple(hidden.shape), hidden.dtype)
        blk = self.__dict__.get("_blk")
        if blk is None or blk[0] != key:
            blk = (key, blocks.GPT2Block(self._weights(), batch=self.batch, seq=self.seq,
                                         residual_dtype=torch.bfloat16,
                                         out_dtype=torch.bfloat16, device=hidden.device))
            self.__dict__["_blk"] = blk
        return blk[1].forward(hidden.contiguous())


class QwenBlockModel(_Fp8Module):
    """Qwen gated full-attention block, B x S tokens, hidden 2560,
    32 query / 8 KV heads x 128 (GQA), RMSNorm (1 + w) on the input and on q, k, RoPE theta
    1e6, causal softmax, sigmoid gate from a separate 2560 -> 4096 projection, f32 input,
    bf16 residual stream and output (quantisation points of
    tasks/model_qwen35_4b_full_attention_block_fp8/starter.py:333-392)."""

    def __init__(self, batch=4, seq=2048, hidden=2560, heads=32, kv_heads=8, hd=128,
                 theta=1e6):
        super().__init__()
        self.batch, self.seq = batch, seq
        self.heads, self.kv_heads, self.hd, self.eps = heads, kv_heads, hd, 1e-6
        for name, shape in (("q_w", (heads * hd, hidden)), ("gate_w", (heads * hd, hidden)),
                            ("k_w", (kv_heads * hd, hidden)), ("v_w", (kv_heads * hd, hidden)),
                            ("o_w", (hidden, heads * hd))):
            self._add_weight(name, torch.randn(shape) * 0.02)
        self.register_buffer("in_norm_w", torch.randn(hidden) * 0.02)
        self.register_buffer("q_norm_w", torch.randn(hd) * 0.02)
        self.register_buffer("k_norm_w", torch.randn(hd) * 0.02)
        pos = torch.arange(seq, dtype=torch.float32)
        inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
        f = pos[:, None] * inv[None, :]
        emb = torch.cat((f, f), dim=-1)
        self._cos, self._sin = emb.cos(), emb.sin()  # f32 tables, not cast with the module

    def _weights(self, device):
        w = SimpleNamespace(heads=self.heads, kv_heads=self.kv_heads, head_dim=self.hd,
                            rotary_dim=self.hd, interleaved=False, eps=self.eps,
                            norm_scale=1 / 64.0, qkv_scale=1 / 64.0, ctx_scale=1 / 64.0,
                            mlp_proj_scale=1 / 64.0, mlp_act_scale=1 / 32.0, post_norm_w=None,
                            mlp_gate_w=None, mlp_up_w=None, mlp_down_w=None, mlp_gate_s=1.0,
                            mlp_up_s=1.0, mlp_down_s=1.0)
        for name in ("q_w", "gate_w", "k_w", "v_w", "o_w"):
            setattr(w, name, self._e4m3(name))
            setattr(w, name[:-2] + "_s", getattr(self, name + "_s"))
        for name in ("in_norm_w", "q_norm_w", "k_norm_w"):
            setattr(w, name, getattr(self, name).float())
        w.cos, w.sin = self._cos.to(device), self._sin.to(device)
        return w

    def forward(self, hidden):
        w = self._weights(hidden.device)
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
    def forward(self, hidden):
        key = (hidden.device, tuple(hidden.shape), hidden.dtype)
        blk = self.__dict__.get("_blk")
        if blk is None or blk[0] != key:
            blk = (key, blocks.QwenBlock(self._weights(hidden.device), batch=self.batch,
                                         seq=self.seq, residual_dtype=torch.bfloat16,
                                         out_dtype=torch.bfloat16, device=hidden.device))
            self.__dict__["_blk"] = blk
        return blk[1].forward(hidden.contiguous())


# ----------------------------------------------------------------------------- registry
TASKS = {
    "gemm_bias_relu_fp8": dict(Model=GemmBiasRelu, ModelNew=GemmBiasReluNew,
                               get_init_inputs=lambda: [8192, 8192],
                               get_inputs=lambda: _skinny_inputs(), atol=1e-3, rtol=2 ** -7),
    "square_gemm_fp8": dict(Model=SquareGemm, ModelNew=SquareGemmNew,
                            get_init_inputs=lambda: [], get_inputs=lambda: _square_inputs(),
                            atol=1e-3, rtol=2 ** -7),
    "residual_rmsnorm_quant_fp8": dict(Model=ResidualRMSNormQuant,
                                       ModelNew=ResidualRMSNormQuantNew,
                                       get_init_inputs=lambda: [4096],
                                       get_inputs=lambda: _norm_inputs(), atol=1e-4,
                                       rtol=2 ** -3),
    "gpt2_block_fp8": dict(Model=GPT2BlockModel, ModelNew=GPT2BlockNew,
                           get_init_inputs=lambda: [8, 1024],
                           get_inputs=lambda: [torch.randn(8 * 1024, 768)],
                           atol=0.05, rtol=2 ** -7),
    "qwen_attention_block_fp8": dict(Model=QwenBlockModel, ModelNew=QwenBlockNew,
                                     get_init_inputs=lambda: [4, 2048],
                                     get_inputs=lambda: [torch.randn(4 * 2048, 2560)],
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
    globals its evaluator reads, the second defines ModelNew."""
    ref_cls, new_cls = _CLASS[name]
    task = TASKS[name]
    ref = ("from b200fp8 import kernelbench as _kb\n"
           f"Model = _kb.{ref_cls}\n"
           f"get_inputs = _kb.TASKS[{name!r}]['get_inputs']\n"
           f"get_init_inputs = _kb.TASKS[{name!r}]['get_init_inputs']\n"
           f"output_atol = {task['atol']!r}\n"
           f"output_rtol = {task['rtol']!r}\n")
    new = "from b200fp8 import kernelbench as _kb\n" f"ModelNew = _kb.{new_cls}\n"
    return ref, new
