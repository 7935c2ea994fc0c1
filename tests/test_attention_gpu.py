"""Parity of the fused tcgen05 attention (b2f_attention_fp8) and its operand prep
(b2f_head_norm_rope, b2f_fp8_to_bf16, b2f_fp8_to_f16) with the CPU oracle.

Bars for the e4m3 context against the oracle's unquantised f32 context (reference math
keeps P in f32; the kernel rounds P to f16 with f16 V, to bf16 with bf16 V, before P.V):
  - every element: |ctx - ref| <= half an e4m3 step at |ref| (the requantisation itself)
    + 2^-7 * max|v| (P rounding and f32 sum order), in value space;
  - every element with |ref| >= 2^-8 * max|v| (in stored units; 2^-7 * max|v| with bf16 P,
    whose rounding is 8x coarser): at most one e4m3 code from the oracle's requantised code
    (the requirement for requantised outputs).  Below
    that floor a context is a near-cancellation of +-v terms whose absolute error is far
    below the e4m3 resolution of the larger values, and its code distance is not
    meaningful (sign flips around zero);
  - f16 V: >= 99 % of the codes equal the oracle's; bf16 V (2^-8 relative P rounding):
    >= 94 %.
The code-distance histogram is printed (pytest -s) for every case.
"""
from __future__ import annotations

import pytest
import torch

from helpers import e4m3_ulp_diff, gen
from oracle import attention as oatt

pytestmark = pytest.mark.gpu


def _ops():
    from b200fp8 import ops
    return ops


def e4m3_half_step(x: torch.Tensor) -> torch.Tensor:
    """Half the spacing of e4m3 values around |x| (x in stored units)."""
    a = x.abs().clamp_min(2.0 ** -6)
    return torch.exp2(torch.floor(torch.log2(a)) - 3.0) * 0.5


def assert_ctx_close(ctx_q, ref_f32, scale, vmax, min_same=0.99):
    """min_same 0.99 is the f16-P bar; the bf16-P callers pass 0.94 (and get the 2^-7
    code floor)."""
    got = ctx_q.cpu().float()
    ref_units = ref_f32 / scale
    bound = e4m3_half_step(ref_units) + 2.0 ** -7 * vmax / scale
    err = (got - ref_units).abs()
    bad = err > bound
    assert not bad.any(), f"{int(bad.sum())} elements out of bound, max err {float(err.max())}"
    codes = e4m3_ulp_diff(ctx_q.cpu(), ref_units.clamp(-448.0, 448.0).to(torch.float8_e4m3fn))
    hist = [int((codes == i).sum()) for i in range(3)] + [int((codes >= 3).sum())]
    floor = (2.0 ** -8 if min_same >= 0.99 else 2.0 ** -7) * vmax / scale
    above = ref_units.abs() >= floor
    print(f"e4m3 code distance histogram [0, 1, 2, >=3]: {hist}; "
          f"max above floor {floor:.3g}: {int(codes[above].max()) if above.any() else 0}")
    assert int(codes[above].max()) <= 1
    assert float((codes == 0).float().mean()) >= min_same, hist


def _e4m3(x: torch.Tensor) -> torch.Tensor:
    # torch's cast to float8_e4m3fn turns values beyond +-448 into NaN: clamp first
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def _qkv(t, hq, hkv, d, g, scale=1 / 64.0):
    q = _e4m3(torch.randn((t, hq * d), generator=g) * 1.5 / scale)
    k = _e4m3(torch.randn((t, hkv * d), generator=g) * 1.5 / scale)
    v = _e4m3(torch.randn((t, hkv * d), generator=g) / scale)
    return q, k, v


_CASES = [
    (1, 128, 1, 1, 64, True), (2, 256, 2, 2, 64, True), (1, 128, 12, 12, 64, True),
    (1, 384, 4, 2, 128, True), (2, 128, 16, 4, 256, True), (1, 128, 16, 16, 64, False),
    (1, 200, 2, 1, 128, True), (1, 256, 4, 1, 128, False), (1, 1024, 2, 2, 64, True),
    (1, 512, 2, 1, 256, True), (2, 640, 8, 2, 128, True), (1, 384, 6, 3, 64, False),
    (2, 200, 4, 4, 64, True),  # head pairs with their own K / V, ragged last query tile
]


@pytest.mark.parametrize("vtype", ["bf16", "f16"])
@pytest.mark.parametrize("batch,seq,hq,hkv,d,causal", _CASES)
def test_attention_matches_oracle(batch, seq, hq, hkv, d, causal, vtype):
    if vtype == "f16" and d == 256:
        pytest.skip("f16 V is offered for head_dim 64 / 128")
    g = gen(1000 + seq + hq + d)
    s = 1 / 64.0
    t = batch * seq
    q, k, v = _qkv(t, hq, hkv, d, g, s)
    vf = v.float().view(t, hkv, d) * s
    ref = oatt.attention(q.float().view(t, hq, d) * s, k.float().view(t, hkv, d) * s, vf,
                         batch=batch, causal=causal).reshape(t, hq * d)
    ops = _ops()
    vd = ops.fp8_to_f16(v.cuda()) if vtype == "f16" else ops.fp8_to_bf16(v.cuda())
    ctx = ops.attention_fp8(q.cuda(), k.cuda(), vd, batch=batch,
                            heads=hq, kv_heads=hkv, head_dim=d, causal=causal, q_scale=s,
                            k_scale=s, v_scale=s, ctx_scale=s)
    torch.cuda.synchronize()
    assert_ctx_close(ctx, ref, s, float(vf.abs().max()), 0.99 if vtype == "f16" else 0.94)


@pytest.mark.parametrize("gdt", ["e4m3", "bf16"])
@pytest.mark.parametrize("batch,seq,hq,hkv,d,causal", [
    (1, 200, 4, 2, 64, True),     # paired GQA heads, ragged sequence, 64-byte gate rows
    (2, 256, 6, 6, 64, False),    # MHA, non-causal
    (1, 384, 8, 2, 128, True),    # Qwen-like GQA, 128-byte gate rows
    (1, 130, 3, 3, 128, True),    # odd head count, one partial query tile
])
def test_attention_gate_tiles_match_oracle(batch, seq, hq, hkv, d, causal, gdt):
    """Sigmoid output gate read from a column block of a wider projection (as the blocks
    lay it out): e4m3 gates arrive as TMA tiles in shared memory (128- or 64-byte swizzled
    rows), bf16 gates are read per row.  f16 V, as the blocks run it."""
    g = gen(3000 + seq + hq + d)
    s = 1 / 64.0
    t = batch * seq
    q, k, v = _qkv(t, hq, hkv, d, g, s)
    gate_vals = torch.randn((t, hq * d), generator=g) * 3.0
    if gdt == "e4m3":
        gate_st = _e4m3(gate_vals / s)
        gate_f = gate_st.float() * s
        gs = s
    else:
        gate_st = gate_vals.to(torch.bfloat16)
        gate_f = gate_st.float()
        gs = 1.0
    # the gate as columns [64, 64 + hq*d) of a wider row-major buffer
    wide = torch.zeros((t, hq * d + 128), dtype=gate_st.dtype)
    wide[:, 64:64 + hq * d] = gate_st
    vf = v.float().view(t, hkv, d) * s
    ref = oatt.attention(q.float().view(t, hq, d) * s, k.float().view(t, hkv, d) * s, vf,
                         batch=batch, causal=causal,
                         gate=gate_f.view(t, hq, d)).reshape(t, hq * d)
    ops = _ops()
    wide_d = wide.cuda()
    ctx = ops.attention_fp8(q.cuda(), k.cuda(), ops.fp8_to_f16(v.cuda()), batch=batch,
                            heads=hq, kv_heads=hkv, head_dim=d, causal=causal, q_scale=s,
                            k_scale=s, v_scale=s, gate=wide_d[:, 64:64 + hq * d],
                            gate_scale=gs, ctx_scale=s)
    torch.cuda.synchronize()
    assert_ctx_close(ctx, ref, s, float(vf.abs().max()))


def test_attention_gated_interleaved_qwen_reference_layout():
    # tasks/model_qwen35_4b_full_attention_block_fp8: q_gate [T, 16, 2, 256]; gate = half 1,
    # scores / 16 (sqrt(256)), causal, GQA 16/4, ctx * sigmoid(gate)
    t, hq, hkv, d = 128, 16, 4, 256
    g = gen(20260801)
    s = 1 / 64.0
    qg = (torch.randn((t, hq * 2 * d), generator=g) / s).to(torch.float8_e4m3fn)
    k = (torch.randn((t, hkv * d), generator=g) / s).to(torch.float8_e4m3fn)
    v = (torch.randn((t, hkv * d), generator=g) / s).to(torch.float8_e4m3fn)
    qh = qg.float().view(t, hq, 2, d) * s
    vf = v.float().view(t, hkv, d) * s
    ref = oatt.attention(qh[:, :, 0], k.float().view(t, hkv, d) * s, vf, batch=1, causal=True,
                         gate=qh[:, :, 1], sm_scale=1 / 16.0).reshape(t, hq * d)
    ops = _ops()
    qgc = qg.cuda()
    q_dense = qgc.view(t, hq, 2, d)[:, :, 0].contiguous().view(t, hq * d)
    ctx = ops.attention_fp8(q_dense, k.cuda(), ops.fp8_to_bf16(v.cuda()), batch=1, heads=hq,
                            kv_heads=hkv, head_dim=d, q_scale=s, k_scale=s, v_scale=s,
                            gate=qgc[:, d:], gate_scale=s, gate_head_stride=2 * d, ctx_scale=s)
    torch.cuda.synchronize()
    assert_ctx_close(ctx, ref, s, float(vf.abs().max()), 0.94)  # head_dim 256: bf16 V


@pytest.mark.parametrize("d,rot,h,wide", [
    (256, 64, 4, False), (128, 128, 4, False), (64, 64, 4, False),
    (128, 128, 32, True),   # Qwen q: 32 heads inside the fused projection (4-head groups)
    (128, 128, 6, True),    # head count not a multiple of 4: per-head kernel
    (128, 0, 16, True),     # norm only, 4-head groups
])
def test_head_norm_rope(d, rot, h, wide):
    t, seq = 256, 128
    g = gen(7 + d + h)
    s = 1 / 64.0
    x = _e4m3(torch.randn((t, h * d), generator=g) / s)
    w = torch.randn((d,), generator=g) * 0.02
    cos, sin = oatt.rope_tables(seq, rot, 1e6, batch=t // seq) if rot else (None, None)
    ref = oatt.head_rmsnorm_rope(x.float().view(t, h, d) * s, w, cos, sin, rot)
    ref_q = (ref.reshape(t, h * d) / s).to(torch.float8_e4m3fn)
    xd = x.cuda()
    if wide:  # columns [256, 256 + h*d) of a wider row-major projection
        buf = torch.zeros((t, h * d + 512), dtype=torch.uint8, device="cuda")
        buf[:, 256:256 + h * d] = xd.view(torch.uint8)
        xd = buf[:, 256:256 + h * d].view(torch.float8_e4m3fn)
    tab = (lambda z: None if z is None else z[:seq].contiguous().cuda())  # noqa: E731
    out = _ops().head_norm_rope(xd, heads=h, head_dim=d, in_scale=s, out_scale=s,
                                weight=w.cuda(), cos=tab(cos), sin=tab(sin), rotary_dim=rot,
                                seq=seq)
    torch.cuda.synchronize()
    diff = e4m3_ulp_diff(out.cpu(), ref_q)
    assert int(diff.max()) <= 1
    assert float((diff > 0).float().mean()) < 0.01


def test_fp8_to_f16_exact():
    g = gen(4)
    x = (torch.randn((64, 256), generator=g) * 50).to(torch.float8_e4m3fn)
    out = _ops().fp8_to_f16(x.cuda(), scale=1 / 64.0)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), (x.float() / 64.0).to(torch.float16))


def test_fp8_to_bf16_exact():
    g = gen(3)
    x = (torch.randn((64, 256), generator=g) * 50).to(torch.float8_e4m3fn)
    out = _ops().fp8_to_bf16(x.cuda(), scale=1 / 64.0)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), (x.float() / 64.0).to(torch.bfloat16))


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 4)])
def test_attn_prep_one_launch_matches_separate_ops(hq, hkv):
    """b2f_attn_prep (q / k head norm + RoPE and the V copy in one launch) against the
    oracle (q, k within one e4m3 code, as test_head_norm_rope) and the exact V image."""
    t, seq, d = 512, 256, 128
    g = gen(11 + hq)
    s = 1 / 64.0
    ncat = (2 * hq + 2 * hkv) * d
    proj = _e4m3(torch.randn((t, ncat), generator=g) / s)
    wq = torch.randn((d,), generator=g) * 0.02
    wk = torch.randn((d,), generator=g) * 0.02
    cos, sin = oatt.rope_tables(seq, d, 1e6, batch=t // seq)
    q_src = proj[:, :hq * d].float().view(t, hq, d) * s
    k_src = proj[:, 2 * hq * d:(2 * hq + hkv) * d].float().view(t, hkv, d) * s
    q_ref = (oatt.head_rmsnorm_rope(q_src, wq, cos, sin, d).reshape(t, hq * d) / s).to(torch.float8_e4m3fn)
    k_ref = (oatt.head_rmsnorm_rope(k_src, wk, cos, sin, d).reshape(t, hkv * d) / s).to(torch.float8_e4m3fn)
    ops = _ops()
    pd = proj.cuda()
    qo = torch.empty((t, hq * d), dtype=torch.float8_e4m3fn, device="cuda")
    ko = torch.empty((t, hkv * d), dtype=torch.float8_e4m3fn, device="cuda")
    vo = torch.empty((t, hkv * d), dtype=torch.float16, device="cuda")
    tab = lambda z: z[:seq].contiguous().cuda()  # noqa: E731
    ok = ops.attn_prep(pd[:, :], pd[:, 2 * hq * d:], pd[:, (2 * hq + hkv) * d:],
                       q_heads=hq, k_heads=hkv, head_dim=d, in_scale=s, out_scale=s,
                       q_weight=wq.cuda(), k_weight=wk.cuda(), cos=tab(cos), sin=tab(sin),
                       rotary_dim=d, seq=seq, q_out=qo, k_out=ko, v_out=vo)
    torch.cuda.synchronize()
    assert ok
    for got, ref in ((qo, q_ref), (ko, k_ref)):
        diff = e4m3_ulp_diff(got.cpu(), ref)
        assert int(diff.max()) <= 1 and float((diff > 0).float().mean()) < 0.01
    v_ref = proj[:, (2 * hq + hkv) * d:].float().to(torch.float16)
    assert torch.equal(vo.cpu(), v_ref)


@pytest.mark.parametrize("hq,hkv,interleaved,rope", [
    (32, 8, False, True),    # the bench block's layout: q heads, gate heads, k, v
    (16, 4, True, True),     # q / gate interleaved per head (head stride 256)
    (8, 4, False, False),    # no RoPE
])
def test_gemm_head_prep_matches_gemm_then_prep(hq, hkv, interleaved, rope):
    """b2f_gemm_fp8_head_prep (q / k norm + RoPE and the V copy in the projection GEMM's
    epilogue) against the same GEMM's e4m3 output run through b2f_attn_prep: the gate
    columns and the V image are bit-identical, q / k within one e4m3 code (the f32 norm is
    summed in the same order; contraction choices may differ) and almost all equal."""
    ops = _ops()
    t, seq, d, hid = 512, 256, 128, 512
    g = gen(31 + hq + int(interleaved))
    s = 1 / 64.0
    ncat = (2 * hq + 2 * hkv) * d
    a = _e4m3(torch.randn((t, hid), generator=g) * 4)
    w = _e4m3(torch.randn((ncat, hid), generator=g) * 4)
    cs = (torch.rand((ncat,), generator=g) * 0.5 + 0.75) * (2.0 ** -9)
    wq = torch.randn((d,), generator=g) * 0.02
    wk = torch.randn((d,), generator=g) * 0.02
    cos, sin = oatt.rope_tables(seq, d, 1e6, batch=1)
    tab = lambda z: z[:seq].contiguous().cuda()  # noqa: E731
    qh = 2 * d if interleaved else d
    q_off, g_off = 0, (d if interleaved else hq * d)
    k_off = 2 * hq * d
    v_off = k_off + hkv * d
    ad, wd, csd = a.cuda(), w.cuda(), cs.cuda()
    rope_kw = dict(cos=tab(cos), sin=tab(sin)) if rope else {}

    proj = ops.gemm_fp8(ad, wd, col_scale=csd, out_dtype=torch.float8_e4m3fn, out_scale=s)
    q1 = torch.empty((t, hq * d), dtype=torch.float8_e4m3fn, device="cuda")
    k1 = torch.empty((t, hkv * d), dtype=torch.float8_e4m3fn, device="cuda")
    v1 = torch.empty((t, hkv * d), dtype=torch.float16, device="cuda")
    assert ops.attn_prep(proj[:, q_off:], proj[:, k_off:], proj[:, v_off:v_off + hkv * d],
                         q_heads=hq, k_heads=hkv, head_dim=d, in_scale=s, out_scale=s,
                         q_head_stride=qh, q_weight=wq.cuda(), k_weight=wk.cuda(),
                         rotary_dim=d if rope else 0, seq=seq, q_out=q1, k_out=k1, v_out=v1,
                         **rope_kw)

    proj2 = torch.zeros((t, ncat), dtype=torch.float8_e4m3fn, device="cuda")
    q2 = torch.empty_like(q1)
    k2 = torch.empty_like(k1)
    v2 = torch.empty_like(v1)
    assert ops.gemm_fp8_head_prep(ad, wd, col_scale=csd, out=proj2, out_scale=s, q_out=q2,
                                  k_out=k2, v_out=v2, q_off=q_off, q_heads=hq,
                                  q_head_stride=qh, k_off=k_off, k_heads=hkv, v_off=v_off,
                                  v_heads=hkv, q_norm_w=wq.cuda(), k_norm_w=wk.cuda(),
                                  weight_offset=1.0, eps=1e-6, seq=seq, **rope_kw)
    torch.cuda.synchronize()
    gate_cols = torch.cat([torch.arange(g_off + h * qh, g_off + h * qh + d) for h in range(hq)])
    assert torch.equal(proj2.view(torch.uint8)[:, gate_cols].cpu(),
                       proj.view(torch.uint8)[:, gate_cols].cpu())
    assert torch.equal(v2.cpu(), v1.cpu())
    for got, ref in ((q2, q1), (k2, k1)):
        diff = e4m3_ulp_diff(got.cpu(), ref.cpu())
        assert int(diff.max()) <= 1 and float((diff > 0).float().mean()) < 0.001


@pytest.mark.parametrize("t,d", [(512, 768), (300, 1024)])
def test_gemm_v_copy_in_epilogue_matches_gemm_then_convert(t, d):
    """The GPT-2 / vision QKV GEMM (bias, single-CTA 256-column tiles) writing the 16-bit V
    image from its epilogue (b2f_gemm_fp8_head_prep with V blocks only): q / k columns and
    the V image bit-identical to the plain GEMM followed by the e4m3 -> f16 conversion."""
    ops = _ops()
    g = gen(7 + d)
    s = 1 / 64.0
    a = _e4m3(torch.randn((t, d), generator=g) * 4).cuda()
    w = _e4m3(torch.randn((3 * d, d), generator=g) * 4).cuda()
    bias = (torch.randn((3 * d,), generator=g) * 0.1).cuda()
    kw = dict(scale_a=2.0 ** -5, scale_b=2.0 ** -6, bias=bias)
    qkv = ops.gemm_fp8(a, w, out_dtype=torch.float8_e4m3fn, out_scale=s, **kw)
    v1 = ops.fp8_to_f16(qkv[:, 2 * d:], out=torch.empty((t, d), dtype=torch.float16,
                                                           device="cuda"))
    qkv2 = torch.zeros_like(qkv)
    v2 = torch.empty((t, d), dtype=torch.float16, device="cuda")
    assert ops.gemm_fp8_head_prep(a, w, out=qkv2, out_scale=s, q_out=None, k_out=None,
                                  v_out=v2, q_off=0, q_heads=0, k_off=0, k_heads=0,
                                  v_off=2 * d, v_heads=d // 128, **kw)
    torch.cuda.synchronize()
    assert torch.equal(qkv2.view(torch.uint8)[:, :2 * d].cpu(), qkv.view(torch.uint8)[:, :2 * d].cpu())
    assert torch.equal(v2.cpu(), v1.cpu())


def test_attn_prep_without_v_copy():
    """b2f_attn_prep with no V operand (the V image already written by the projection
    GEMM's epilogue): q / k outputs identical to the call with the V copy."""
    ops = _ops()
    t, seq, d, hq, hkv = 512, 256, 128, 16, 4
    g = gen(5)
    s = 1 / 64.0
    proj = _e4m3(torch.randn((t, (2 * hq + 2 * hkv) * d), generator=g) / s).cuda()
    wq = (torch.randn((d,), generator=g) * 0.02).cuda()
    wk = (torch.randn((d,), generator=g) * 0.02).cuda()
    cos, sin = oatt.rope_tables(seq, d, 1e6, batch=1)
    kw = dict(q_heads=hq, k_heads=hkv, head_dim=d, in_scale=s, out_scale=s, q_weight=wq,
              k_weight=wk, cos=cos[:seq].contiguous().cuda(), sin=sin[:seq].contiguous().cuda(),
              rotary_dim=d, seq=seq)
    outs = []
    for with_v in (True, False):
        qo = torch.empty((t, hq * d), dtype=torch.float8_e4m3fn, device="cuda")
        ko = torch.empty((t, hkv * d), dtype=torch.float8_e4m3fn, device="cuda")
        vo = torch.empty((t, hkv * d), dtype=torch.float16, device="cuda") if with_v else None
        vsrc = proj[:, (2 * hq + hkv) * d:] if with_v else None
        assert ops.attn_prep(proj, proj[:, 2 * hq * d:], vsrc, q_out=qo, k_out=ko, v_out=vo, **kw)
        outs.append((qo, ko))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0].view(torch.uint8).cpu(), outs[1][0].view(torch.uint8).cpu())
    assert torch.equal(outs[0][1].view(torch.uint8).cpu(), outs[1][1].view(torch.uint8).cpu())
