"""Failure detection on the GPU without a GPU fault: bounded in-kernel waits give up with an
error status the host reads, argument errors surface as RuntimeError with the library's message,
and the CUDA context stays usable after both."""

from __future__ import annotations

import pytest
import torch

from diffucore_b200 import _int8, _lib, kernels

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    status, err = kernels.selftest_wait_timeout("cuda", limit_cycles=2_000_000)   # ~1 ms
    assert status == 1          # the wait gave up instead of hanging
    assert err == 2             # device error word: self-test expiry
    assert _lib.device_error() == 0
    # the context is still healthy afterwards
    q = torch.randint(-127, 128, (64, 128), dtype=torch.int8, device="cuda")
    acc = _int8.int_mm(q, q)
    assert torch.equal(acc.cpu(), torch._int_mm(q, q.t()).cpu())


def test_argument_errors_raise_with_reason():
    q = torch.zeros(8, 24, dtype=torch.int8, device="cuda")
    w = torch.zeros(16, 24, dtype=torch.int8, device="cuda")
    s = torch.ones(8, device="cuda")
    lib = _lib.load()
    import ctypes
    st = lib.dc_gemm_w8a8(ctypes.c_void_p(q.data_ptr()), 24, ctypes.c_void_p(w.data_ptr()), 24,
                          ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(s.data_ptr()), None, None, 16,
                          _lib.DTYPE_BF16, 8, 16, 24, 0, None)
    assert st != 0 and b"multiple of 16" in lib.dc_last_error()
    x = torch.randn(4, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="ConvRot group"):
        kernels.quant_rows(x, 256)
    v = torch.randn(1, 64, 2, 128, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match="strides"):
        bad = torch.randn(1, 64, 2, 130, device="cuda", dtype=torch.float16)[..., :128]
        kernels.attn_int8(bad, v, v, 0.1)
    assert _lib.device_error() == 0
    torch.cuda.synchronize()
