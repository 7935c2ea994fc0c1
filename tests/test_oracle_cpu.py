"""CPU checks of the oracle itself: small cases against independent formulations."""
from __future__ import annotations

import math

import torch

from helpers import gen
from oracle import attention as oatt
from oracle import fp8 as ofp8
from oracle import gemm as og


def test_scaled_mm_matches_torch_scaled_mm_cpu():
    # the reference evaluators' own call, torch._scaled_mm, executed on CPU
    g = gen(1)
    a, sa = ofp8.quantize_amax(torch.randn((16, 64), generator=g))
    b, sb = ofp8.quantize_amax(torch.randn((32, 64), generator=g))
    ref = og.reference_scaled_mm_cpu(a, b, sa, sb)
    ours = og.scaled_mm(a, b, sa, sb)
    assert torch.allclose(ours, ref, rtol=1e-5, atol=1e-5)


def test_attention_against_naive_loop():
    g = gen(2)
    t, h, d = 8, 2, 4
    q, k, v = (torch.randn((t, h, d), generator=g) for _ in range(3))
    out = oatt.attention(q, k, v, batch=1, causal=True)
    for hh in range(h):
        for i in range(t):
            s = [float((q[i, hh] * k[j, hh]).sum()) / math.sqrt(d) for j in range(i + 1)]
            m = max(s)
            p = [math.exp(x - m) for x in s]
            z = sum(p)
            ctx = sum(p[j] / z * v[j, hh] for j in range(i + 1))
            assert torch.allclose(out[i, hh], ctx, atol=1e-5)


def test_rope_rotate_half_matches_complex_rotation():
    g = gen(3)
    x = torch.randn((4, 1, 8), generator=g)
    cos, sin = oatt.rope_tables(4, 8, 10000.0)
    y = oatt.head_rmsnorm_rope(x, None, cos, sin, 8)
    xc = torch.complex(x[..., :4], x[..., 4:])
    ang = torch.complex(cos[:, :4], sin[:, :4])[:, None, :]
    yc = xc * ang
    assert torch.allclose(y, torch.cat((yc.real, yc.imag), -1), atol=1e-5)
