"""C-ABI behaviour on the GPU: bounded waits report through the status word."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_sets_status_and_context_survives():
    from b200fp8 import _lib
    lib = _lib.lib()
    assert _lib.device_status(reset=True) in (0, 1, 2, 3, 4, 5)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.b2f_debug_bounded_wait(ctypes.c_ulonglong(50_000_000), stream))  # 50 ms
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 3  # B2F_DEV_TIMEOUT_EPILOGUE
    # the context is still usable afterwards
    x = torch.ones(1024, device="cuda")
    assert float(x.sum()) == 1024.0
    assert _lib.device_status() == 0
