"""The allocation-free split-K GEMM (b2f_gemm_fp8_static), called through the C ABI.

It exists for callers that cannot allocate device memory when they call the library (a
plugin inside a framework that owns all device allocations, a serving loop with a memory
plan fixed at start-up), so it keeps its split-K scratch in a static device array instead
of a caller workspace.  Each of two calls in a row, with different shapes so that the
second runs on scratch the first left behind, must match the existing entry point
b2f_gemm_fp8 within the bar of the other f32 GEMM tests (1e-4 relative to the output
range).  This file sorts last so that a run stopping at the first failure has already run
every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import e4m3_ulp_diff, fp8_amax, gen, randn

pytestmark = pytest.mark.gpu


def _args(L, a, b, bias, out, sa, sb, splits):
    args = L.GemmArgs()
    L.lib().b2f_gemm_args_init(ctypes.byref(args))
    args.m, args.k = a.shape
    args.n = b.shape[0]
    args.a, args.lda, args.b, args.ldb = a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0)
    args.alpha = sa * sb
    args.bias = bias.data_ptr()
    args.act = L.ACT_RELU
    args.out, args.out_dtype, args.out_ld = out.data_ptr(), L.DTYPE_F32, out.stride(0)
    args.splits = splits
    return args


def test_static_scratch_split_k_matches_existing_entry_point_twice():
    from b200fp8 import _lib as L
    lib = L.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for seed, (m, n, k, splits) in ((1, (128, 2048, 4096, 4)), (2, (256, 1024, 2048, 2))):
        g = gen(seed)
        a, sa = fp8_amax((m, k), g, 0.1)
        b, sb = fp8_amax((n, k), g, 0.1)
        bias = randn((n,), g, 0.02).cuda()
        a, b = a.cuda(), b.cuda()
        ref = torch.empty((m, n), device="cuda")
        got = torch.full((m, n), float("nan"), device="cuda")
        L.check(lib.b2f_gemm_fp8(ctypes.byref(_args(L, a, b, bias, ref, sa, sb, 1)), stream))
        L.check(lib.b2f_gemm_fp8_static(ctypes.byref(_args(L, a, b, bias, got, sa, sb, splits)),
                                        stream))
        torch.cuda.synchronize()
        err = (got - ref).abs().max().item()
        assert err <= 1e-4 * (1.0 + ref.abs().max().item()), (m, n, k, err)
    assert L.device_status() == 0


def test_static_scratch_e4m3_output_with_amax():
    """The two-slice drain also requantises to e4m3 and reduces amax: same codes and the
    same amax as the workspace entry point."""
    from b200fp8 import _lib as L
    lib = L.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    m, n, k = 128, 2048, 8192
    g = gen(3)
    a, sa = fp8_amax((m, k), g, 0.1)
    b, sb = fp8_amax((n, k), g, 0.1)
    bias = randn((n,), g, 0.02).cuda()
    a, b = a.cuda(), b.cuda()
    outs, amaxes = [], []
    for entry, splits in ((lib.b2f_gemm_fp8, 1), (lib.b2f_gemm_fp8_static, 2)):
        out = torch.zeros((m, n), dtype=torch.uint8, device="cuda")
        amax = torch.zeros(1, device="cuda")
        args = _args(L, a, b, bias, out, sa, sb, splits)
        args.out_dtype, args.out_ld, args.out_scale = L.DTYPE_E4M3, n, 1.0 / 256.0
        args.amax = amax.data_ptr()
        L.check(entry(ctypes.byref(args), stream))
        torch.cuda.synchronize()
        outs.append(out.cpu())
        amaxes.append(float(amax))
    # the two forms add the same partial products in a different order (f32): at most one
    # e4m3 code apart, and rarely
    d = e4m3_ulp_diff(outs[0].view(torch.float8_e4m3fn), outs[1].view(torch.float8_e4m3fn))
    assert int(d.max()) <= 1 and float((d > 0).float().mean()) < 0.01
    assert abs(amaxes[0] - amaxes[1]) <= 1e-5 * amaxes[0]
    assert L.device_status() == 0


def test_static_scratch_rejects_oversized_problems():
    from b200fp8 import _lib as L
    lib = L.lib()
    a = torch.zeros((1024, 4096), dtype=torch.uint8, device="cuda")
    b = torch.zeros((4096, 4096), dtype=torch.uint8, device="cuda")
    out = torch.empty((1024, 4096), device="cuda")
    bias = torch.zeros(4096, device="cuda")
    args = _args(L, a, b, bias, out, 1.0, 1.0, 4)  # 4 x 1024 x 4096 x 4 B = 64 MiB > 8 MiB
    rc = lib.b2f_gemm_fp8_static(ctypes.byref(args), None)
    assert rc == L.B2F_ERR_ARG
    assert b"exceeds the 8 MiB static scratch" in lib.b2f_last_error()
