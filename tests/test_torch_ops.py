"""torch.library registrations: schemas and fake (shape) implementations on CPU, real
kernels against the direct ops on the GPU."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from b200fp8 import torch_ops  # noqa: F401  (registers torch.ops.b200fp8.*)


def test_ops_registered():
    for name in ("gemm_fp8", "quantize_fp8", "residual_rmsnorm_quant", "attention_fp8"):
        assert hasattr(torch.ops.b200fp8, name)


def test_fake_shapes():
    with FakeTensorMode(allow_non_fake_inputs=False):
        a = torch.empty((256, 512), dtype=torch.float8_e4m3fn, device="meta")
        b = torch.empty((384, 512), dtype=torch.float8_e4m3fn, device="meta")
        out = torch.ops.b200fp8.gemm_fp8(a, b, 1.0, 1.0, None, "relu", torch.bfloat16, 1.0,
                                         None, 1.0)
        assert out.shape == (256, 384) and out.dtype == torch.bfloat16
        x = torch.empty((64, 128), dtype=torch.float32, device="meta")
        q, s = torch.ops.b200fp8.quantize_fp8(x)
        assert q.dtype == torch.float8_e4m3fn and q.shape == x.shape and s.shape == (1,)
        xb = torch.empty((64, 128), dtype=torch.bfloat16, device="meta")
        g = torch.empty((128,), dtype=torch.bfloat16, device="meta")
        q, s, h = torch.ops.b200fp8.residual_rmsnorm_quant(xb, xb, g, 1e-6)
        assert h.dtype == torch.bfloat16 and q.shape == xb.shape
        qq = torch.empty((256, 4 * 64), dtype=torch.float8_e4m3fn, device="meta")
        kk = torch.empty((256, 2 * 64), dtype=torch.float8_e4m3fn, device="meta")
        vv = torch.empty((256, 2 * 64), dtype=torch.float16, device="meta")
        ctx = torch.ops.b200fp8.attention_fp8(qq, kk, vv, 2, 4, 2, 64, True, 1.0, 1.0, 1.0, 1.0,
                                              None, 1.0)
        assert ctx.shape == (256, 256) and ctx.dtype == torch.float8_e4m3fn


@pytest.mark.gpu
def test_custom_ops_match_direct_calls():
    from b200fp8 import ops
    g = torch.Generator().manual_seed(3)
    a = (torch.randn((256, 512), generator=g) * 40).to(torch.float8_e4m3fn).cuda()
    b = (torch.randn((384, 512), generator=g) * 40).to(torch.float8_e4m3fn).cuda()
    bias = torch.randn(384, generator=g).cuda()
    y1 = torch.ops.b200fp8.gemm_fp8(a, b, 0.01, 0.02, bias, "relu", torch.bfloat16, 1.0, None, 1.0)
    y2 = ops.gemm_fp8(a, b, scale_a=0.01, scale_b=0.02, bias=bias, act="relu")
    x = torch.randn((64, 128), generator=g).cuda()
    q1, s1 = torch.ops.b200fp8.quantize_fp8(x)
    q2, s2 = ops.quantize_fp8(x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)
