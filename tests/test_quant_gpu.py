"""b2f_quantize_fp8 (per-tensor e4m3 quantisation on the device) against the CPU oracle:
bit-exact bytes and scale (same f32 amax, f32 division, RNE)."""
import pytest
import torch

from helpers import gen, randn
from oracle.fp8 import quantize_amax_f32

pytestmark = pytest.mark.gpu


def _ops():
    from b200fp8 import ops
    return ops


@pytest.mark.parametrize("rows,cols,dtype", [
    (1, 8, torch.float32), (3, 24, torch.bfloat16), (128, 8192, torch.float32),
    (4096, 4096, torch.float32), (1000, 776, torch.bfloat16)])
def test_dynamic_quantisation_bit_exact(rows, cols, dtype):
    g = gen(rows * 7 + cols)
    x = (randn((rows, cols), g) * 3).to(dtype)
    q_ref, s_ref = quantize_amax_f32(x)
    q, s = _ops().quantize_fp8(x.cuda())
    torch.cuda.synchronize()
    assert float(s.cpu()) == s_ref
    assert torch.equal(q.view(torch.uint8).cpu(), q_ref.view(torch.uint8))


def test_static_scale_strided_rows_and_scale_product():
    ops = _ops()
    g = gen(5)
    base = randn((64, 48), g)
    x = base.cuda()[:, :32]  # row pitch 48 elements
    q, _ = ops.quantize_fp8(x, scale=0.01)
    ref = (base[:, :32] / torch.tensor(0.01, dtype=torch.float32)).clamp(-448, 448).to(
        torch.float8_e4m3fn)
    prod = torch.empty(1, device="cuda")
    other = torch.tensor([0.5], device="cuda")
    _, s = ops.quantize_fp8(x, scale_mul=other, scale_prod_out=prod)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.uint8).cpu(), ref.view(torch.uint8))
    assert float(prod.cpu()) == float(s.cpu()) * 0.5


def test_all_zero_input_uses_unit_scale():
    q, s = _ops().quantize_fp8(torch.zeros((16, 64), device="cuda"))
    torch.cuda.synchronize()
    assert float(s.cpu()) == 1.0
    assert int(q.view(torch.uint8).cpu().max()) == 0
