"""Parity of b2f_norm_quant (residual + RMSNorm/LayerNorm + e4m3) with the CPU oracle.

Bars: e4m3 outputs within 1 e4m3 ulp of the oracle (different f32 summation order may
flip a rounding), with at most 0.5% of elements off by one; bf16 residual stream exact
(x + r rounded once); dynamic scale within 1e-6 relative.
"""
from __future__ import annotations

import pytest
import torch

from helpers import e4m3_ulp_diff, gen, randn
from oracle import norm as onorm

pytestmark = pytest.mark.gpu


def _ops():
    from b200fp8 import ops
    return ops


def _assert_q(q_gpu, q_ref, frac=0.005):
    d = e4m3_ulp_diff(q_gpu.cpu(), q_ref)
    assert int(d.max()) <= 1, int(d.max())
    assert float((d > 0).float().mean()) <= frac


@pytest.mark.parametrize("rows,cols", [(1, 8), (7, 768), (64, 2560), (300, 4096), (1024, 4096)])
def test_residual_rmsnorm_amax_quant_config3(rows, cols):
    g = gen(20260731 + rows)
    x = randn((rows, cols), g).to(torch.bfloat16)
    r = randn((rows, cols), g).to(torch.bfloat16)
    gamma = (1 + randn((cols,), g, 0.02)).to(torch.bfloat16)
    q_ref, s_ref, h_ref = onorm.residual_rmsnorm_amax_quant(x, r, gamma, eps=1e-6)
    h = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    q, s = _ops().norm_quant(x.cuda(), gamma.cuda(), kind="rms", eps=1e-6, residual=r.cuda(),
                             h_out=h)
    torch.cuda.synchronize()
    assert torch.equal(h.cpu(), h_ref)
    assert abs(float(s.cpu()) - s_ref) <= 1e-6 * s_ref
    _assert_q(q, q_ref)


def test_qwen_rmsnorm_one_plus_w_from_fp8_input():
    # Qwen block: norm1 = rms_norm(dequant(hidden_fp8)) * (1 + w), quantised at 1/64.
    rows, cols = 128, 2560
    g = gen(20260801)
    src = torch.empty((rows, cols)).uniform_(-1, 1, generator=g)
    xq = (src * 448.0).to(torch.float8_e4m3fn)
    w = randn((cols,), g, 0.02)
    _, y = onorm.residual_norm(xq, w, kind="rms", weight_offset=1.0, eps=1e-6, x_scale=1 / 448.0)
    q_ref = (y / (1 / 64.0)).to(torch.float8_e4m3fn)
    q, _ = _ops().norm_quant(xq.cuda(), w.cuda(), kind="rms", weight_offset=1.0, eps=1e-6,
                             x_scale=1 / 448.0, q_scale=1 / 64.0)
    torch.cuda.synchronize()
    _assert_q(q, q_ref)


@pytest.mark.parametrize("rows,cols", [(128, 768), (513, 768), (64, 4096)])
def test_gpt2_layernorm_quant(rows, cols):
    g = gen(20260801 + rows)
    x = randn((rows, cols), g).to(torch.bfloat16)
    w = 1 + randn((cols,), g, 0.02)
    b = randn((cols,), g, 0.02)
    _, y = onorm.residual_norm(x, w, kind="layer", bias=b, eps=1e-5)
    q_ref = (y / (1 / 64.0)).to(torch.float8_e4m3fn)
    yb = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    q, _ = _ops().norm_quant(x.cuda(), w.cuda(), kind="layer", bias=b.cuda(), eps=1e-5,
                             q_scale=1 / 64.0, y_out=yb)
    torch.cuda.synchronize()
    _assert_q(q, q_ref)
    assert torch.allclose(yb.cpu().float(), y, rtol=2 ** -7, atol=1e-5)


def test_f32_residual_stream():
    rows, cols = 96, 1024
    g = gen(5)
    x = randn((rows, cols), g)
    r = randn((rows, cols), g)
    w = randn((cols,), g, 0.02)
    h_ref, y = onorm.residual_norm(x, w, kind="rms", weight_offset=1.0, eps=1e-6, residual=r)
    h = torch.empty((rows, cols), device="cuda")
    q, _ = _ops().norm_quant(x.cuda(), w.cuda(), kind="rms", weight_offset=1.0, eps=1e-6,
                             residual=r.cuda(), h_out=h, q_scale=1 / 64.0)
    torch.cuda.synchronize()
    assert torch.allclose(h.cpu(), h_ref, rtol=0, atol=0)
    _assert_q(q, (y / (1 / 64.0)).to(torch.float8_e4m3fn))


def _norm_case(rows, cols, x_dtype, res_dtype, kind, static, seed):
    g = gen(seed)
    x = randn((rows, cols), g)
    if x_dtype == torch.float8_e4m3fn:
        # rows padded to a 16-byte pitch (the ABI's e4m3 row rule); a view keeps `cols`
        pitch = (cols + 15) // 16 * 16
        xp = torch.zeros((rows, pitch))
        xp[:, :cols] = x * 448 / float(x.abs().max())
        x = xp.to(x_dtype)  # callers slice [:, :cols] on the device
    else:
        x = x.to(x_dtype)
    r = None if res_dtype is None else randn((rows, cols), g).to(res_dtype)
    w = (1 + randn((cols,), g, 0.02))
    b = randn((cols,), g, 0.02) if kind == "layer" else None
    return x, r, w, b


@pytest.mark.parametrize("rows,cols,x_dtype,res_dtype,kind,static", [
    (1000, 4096, torch.bfloat16, torch.bfloat16, "rms", False),
    (333, 768, torch.bfloat16, torch.bfloat16, "layer", True),
    (257, 2560, torch.float8_e4m3fn, None, "rms", True),
    (130, 8192, torch.float32, torch.float32, "layer", False),
    (77, 1024, torch.bfloat16, torch.float32, "rms", True),
    (5, 8, torch.float8_e4m3fn, None, "rms", False),       # 8-byte rows: row-group fallback
    (64, 16, torch.float8_e4m3fn, torch.bfloat16, "layer", True),
    (2049, 512, torch.bfloat16, None, "layer", False),
])
def test_stream_and_rowgroup_schedules_agree(rows, cols, x_dtype, res_dtype, kind, static):
    """The streaming schedule (warp-per-row, bulk copies into shared-memory rings) and the
    row-group kernels compute the same formulas with different f32 summation orders: h is
    identical, the scale equal to 1e-6, y within 1 bf16 ulp, q within 1 e4m3 step."""
    ops = _ops()
    x, r, w, b = _norm_case(rows, cols, x_dtype, res_dtype, kind, static, 7 + rows)
    dev = lambda t: None if t is None else t.cuda()  # noqa: E731
    xd = dev(x)[:, :cols]
    expect = "rowgroup" if (x_dtype == torch.float8_e4m3fn and cols % 16) else "stream"
    probe = ops.norm_quant(xd, w.cuda(), kind=kind, bias=dev(b), residual=dev(r),
                           q_scale=(1 / 64.0) if static else None, query_schedule=True)
    assert probe == expect
    outs = []
    for schedule in ("auto", "rowgroup"):
        h = torch.empty((rows, cols), dtype=res_dtype or torch.bfloat16, device="cuda") \
            if r is not None else None
        y = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
        q, s = ops.norm_quant(xd, w.cuda(), kind=kind, bias=dev(b), eps=1e-5,
                              x_scale=0.5 if x_dtype == torch.float8_e4m3fn else 1.0,
                              residual=dev(r), h_out=h, y_out=y,
                              q_scale=(1 / 64.0) if static else None, schedule=schedule)
        torch.cuda.synchronize()
        outs.append((q.view(torch.uint8).cpu(), None if s is None else s.cpu(),
                     None if h is None else h.cpu(), y.cpu()))
    (qa, sa, ha, ya), (qb, sb, hb, yb) = outs
    if ha is not None:
        assert torch.equal(ha, hb)
    if sa is not None:
        assert abs(float(sa) - float(sb)) <= 1e-6 * abs(float(sb))
    yd = (ya.float() - yb.float()).abs()
    assert bool((yd <= yb.float().abs() * 2.0 ** -7 + 1e-30).all())
    _assert_q(qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn).cpu())


@pytest.mark.parametrize("wdt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols,kind,bias,x_scale", [
    (8192, 768, "layer", True, 1.0),    # GPT-2 LayerNorm: same lane order as row groups
    (333, 768, "layer", False, 0.5),
    (257, 2560, "rms", False, 1.0),     # Qwen input RMSNorm (1 + w)
    (1000, 1152, "layer", True, 1.0),   # vision LayerNorm
    (7, 3072, "rms", False, 2.0),       # widest row of the warp schedule
    (40, 3072, "layer", True, 1.0),     # widest LayerNorm row with gamma + bias
    (3, 8, "layer", True, 1.0),
])
def test_warp_schedule_matches_rowgroup(rows, cols, kind, bias, x_scale, wdt):
    """Short bf16 rows with a static scale and no residual run one warp per row.  Same
    formulas as the row-group kernels; with 32 threads per row (cols <= 1024) the f32
    summation order is the same too, so the bytes are identical; wider rows are within one
    e4m3 step."""
    ops = _ops()
    g = torch.Generator().manual_seed(rows + cols)
    x = randn((rows, cols), g).to(torch.bfloat16).cuda()
    w = (1 + randn((cols,), g, 0.02)).to(wdt).cuda()
    b = randn((cols,), g, 0.02).to(wdt).cuda() if bias else None
    off = 1.0 if kind == "rms" else 0.0
    kw = dict(kind=kind, bias=b, weight_offset=off, eps=1e-5, x_scale=x_scale, q_scale=1 / 64.0)
    assert ops.norm_quant(x, w, query_schedule=True, **kw) == "warp"
    qa, _ = ops.norm_quant(x, w, **kw)
    qb, _ = ops.norm_quant(x, w, schedule="rowgroup", **kw)
    torch.cuda.synchronize()
    if cols <= 1024:
        assert torch.equal(qa.view(torch.uint8).cpu(), qb.view(torch.uint8).cpu())
    else:
        _assert_q(qa.cpu(), qb.cpu())


@pytest.mark.parametrize("shards", [2, 3])
def test_stats_apply_phases_share_one_scale_across_row_shards(shards):
    """Row shards run pass 1 (``phase="stats"``), their amax values are max-reduced (the
    all-reduce of a row-sharded job), then each runs pass 2 (``phase="apply"``): the result
    equals the single-device dynamic-scale run."""
    ops = _ops()
    rows, cols = 1500, 4096
    x, r, w, _ = _norm_case(rows, cols, torch.bfloat16, torch.bfloat16, "rms", False, 99)
    x, r, w = x.cuda(), r.cuda(), w.to(torch.bfloat16).cuda()
    h_full = torch.empty_like(x)
    q_full, s_full = ops.norm_quant(x, w, residual=r, h_out=h_full)
    bounds = [rows * i // shards for i in range(shards + 1)]
    amaxes, hs = [], []
    for i in range(shards):
        sl = slice(bounds[i], bounds[i + 1])
        a = torch.zeros(1, device="cuda")
        h = torch.empty_like(x[sl])
        ops.norm_quant(x[sl], w, residual=r[sl], h_out=h, amax=a, phase="stats")
        amaxes.append(a)
        hs.append(h)
    amax = torch.stack(amaxes).max().reshape(1)
    qs, ss = [], []
    for i in range(shards):
        sl = slice(bounds[i], bounds[i + 1])
        s = torch.empty(1, device="cuda")
        q, _ = ops.norm_quant(x[sl], w, residual=r[sl], h_out=hs[i], amax=amax.clone(),
                              scale_out=s, phase="apply")
        qs.append(q)
        ss.append(s)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(hs), h_full)
    for s in ss:
        assert torch.equal(s, s_full)
    assert torch.equal(torch.cat(qs).view(torch.uint8), q_full.view(torch.uint8))


@pytest.mark.parametrize("kind,static", [("rms", False), ("rms", True), ("layer", True)])
def test_stream_schedule_against_oracle_large(kind, static):
    """BASELINE config 3 size through the streaming schedule against the CPU oracle."""
    ops = _ops()
    rows, cols = 16384, 4096
    g = gen(4242)
    x = randn((rows, cols), g).to(torch.bfloat16)
    r = randn((rows, cols), g).to(torch.bfloat16)
    w = (1 + randn((cols,), g, 0.02)).to(torch.bfloat16)
    b = randn((cols,), g, 0.02).to(torch.bfloat16) if kind == "layer" else None
    h_ref, y_ref = onorm.residual_norm(x, w, kind=kind, bias=b, eps=1e-6, residual=r,
                                       h_dtype=torch.bfloat16)
    if static:
        q_ref = (y_ref / (1 / 64.0)).to(torch.float8_e4m3fn)
    else:
        yb = y_ref.to(torch.bfloat16).float()
        s_ref = float(yb.abs().max()) / 448.0
        q_ref = (yb / s_ref).to(torch.float8_e4m3fn)
    h = torch.empty((rows, cols), dtype=torch.bfloat16, device="cuda")
    q, s = ops.norm_quant(x.cuda(), w.cuda(), kind=kind, bias=None if b is None else b.cuda(),
                          eps=1e-6, residual=r.cuda(), h_out=h,
                          q_scale=(1 / 64.0) if static else None)
    torch.cuda.synchronize()
    assert torch.equal(h.cpu(), h_ref.to(torch.bfloat16))
    if not static:
        assert abs(float(s.cpu()) - s_ref) <= 1e-6 * s_ref
    _assert_q(q, q_ref)


@pytest.mark.parametrize("rows,cols,xdt,odt,affine", [
    (3, 100000, torch.float8_e4m3fn, torch.float32, False),
    (2, 65536 * 3 + 17, torch.bfloat16, torch.float32, True),
    (5, 1000, torch.float32, torch.bfloat16, True),
    (1, 131072, torch.float8_e4m3fn, torch.bfloat16, False),
])
def test_layer_norm_rows_against_oracle(rows, cols, xdt, odt, affine):
    """Long-row LayerNorm (b2f_layer_norm_rows): each row split over many CTAs, ragged
    chunk tails, f32 statistics per chunk combined in f64."""
    ops = _ops()
    g = gen(rows * 7 + cols)
    src = torch.rand((rows, cols), generator=g)
    if xdt == torch.float8_e4m3fn:
        x, xs = (src * 448).to(xdt), 1 / 448.0
    else:
        x, xs = src.to(xdt), 1.0
    w = (1 + 0.1 * randn((cols,), g)) if affine else None
    b = 0.1 * randn((cols,), g) if affine else None
    ref = onorm.layer_norm_rows(x.float() * xs, 1e-5, w, b)
    out = ops.layer_norm_rows(x.cuda(), x_scale=xs, eps=1e-5, out_dtype=odt,
                              weight=None if w is None else w.cuda(),
                              bias=None if b is None else b.cuda())
    torch.cuda.synchronize()
    tol = 1e-4 if odt == torch.float32 else 2.0 ** -8 * float(ref.abs().max())
    assert float((out.float().cpu() - ref).abs().max()) <= tol


def test_layer_norm_rows_level1_40_golden():
    """tasks/level1_40_layer_norm_fp8 at its shape [16 x 4,194,304], e4m3 at 1/448, f32
    out: every element against the f64 oracle and the golden samples (task bar 0.01)."""
    import os
    import sys
    from conftest import ROOT
    gdir = os.path.join(ROOT, "tests", "golden")
    if gdir not in sys.path:
        sys.path.insert(0, gdir)
    import task_inputs as ti
    inp = ti.layer_norm_task()
    fix = torch.load(os.path.join(gdir, "level1_40_layer_norm_fp8.pt"))
    out = _ops().layer_norm_rows(inp["x"].cuda(), x_scale=inp["x_scale"], eps=inp["eps"])
    torch.cuda.synchronize()
    got = out.cpu()
    assert float((got.reshape(-1)[fix["index"]] - fix["value"]).abs().max()) <= 1e-4
    ref = onorm.layer_norm_rows(inp["x"].float() * inp["x_scale"], inp["eps"])
    assert float((got - ref).abs().max()) <= 1e-4  # task bar: 0.01
