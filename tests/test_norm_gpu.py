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
