"""The attention entry point for callers that cannot allocate device memory.

Some applications own all of their GPU memory through their own pool (or run where cudaMalloc's
implicit synchronization is not allowed) and so cannot pass this library a workspace.
`dc_attn_int8_fwd_noalloc` keeps the attention's intermediate Q/K codes and scales in one fixed
device array inside the library instead. These tests call it through the C-ABI and check that it
gives what the workspace entry point `dc_attn_int8_fwd` gives, on two calls in a row with different
inputs (the second call reuses the array the first one left filled), and that shapes too large for
the fixed array are refused with a clear error. This file is collected last on purpose.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from diffucore_b200 import _lib

pytestmark = pytest.mark.gpu


def _strides(t: torch.Tensor):
    return _lib.i64_array((t.stride(0), t.stride(1), t.stride(2)))


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _inputs(seed, B=2, L=1000, H=3, D=128, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    # (B, H, L, D) storage read through (B, L, H, D) views, as attention_bhld passes them
    q, k, v = (torch.randn(B, H, L, D, generator=g).to(dtype).cuda().transpose(1, 2) for _ in range(3))
    return q, k, v


def _with_workspace(lib, q, k, v, mode):
    B, L, H, D = q.shape
    n = ctypes.c_size_t(0)
    assert lib.dc_attn_workspace_size(B, H, L, L, D, mode, ctypes.byref(n)) == 0
    ws = torch.empty(n.value, device="cuda", dtype=torch.uint8)
    o = torch.empty(B, L, H, D, device="cuda", dtype=q.dtype)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.dc_attn_int8_fwd(_p(q), _p(k), _p(v), _lib.DTYPE_BF16, B, H, L, L, D, _strides(q), _strides(k),
                              _strides(v), D ** -0.5, mode, _p(o), _strides(o), _p(ws), ws.numel(),
                              ctypes.c_void_p(st))
    assert rc == 0, lib.dc_last_error()
    return o


def _without_allocation(lib, q, k, v, mode):
    B, L, H, D = q.shape
    o = torch.empty(B, L, H, D, device="cuda", dtype=q.dtype)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.dc_attn_int8_fwd_noalloc(_p(q), _p(k), _p(v), _lib.DTYPE_BF16, B, H, L, L, D, _strides(q),
                                      _strides(k), _strides(v), D ** -0.5, mode, _p(o), _strides(o),
                                      ctypes.c_void_p(st))
    assert rc == 0, lib.dc_last_error()
    return o


@pytest.mark.parametrize("mode", [_lib.MODE_REF, _lib.MODE_BLOCK64])
def test_no_alloc_matches_workspace_entry_point_twice(mode):
    lib = _lib.load()
    for seed in (11, 12):                      # two calls in a row, different inputs
        q, k, v = _inputs(seed)
        got = _without_allocation(lib, q, k, v, mode).float()
        want = _with_workspace(lib, q, k, v, mode).float()
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() <= 2e-2
        cos = torch.nn.functional.cosine_similarity(got.flatten().double(), want.flatten().double(), dim=0)
        assert cos.item() >= 0.999


def test_no_alloc_refuses_shapes_beyond_its_scratch():
    lib = _lib.load()
    q = torch.zeros(1, 8, 1, 128, device="cuda", dtype=torch.bfloat16)      # pointers only; nothing runs
    huge = 200_000                                                            # codes alone: ~51 MB > 32 MiB
    o = torch.empty_like(q)
    rc = lib.dc_attn_int8_fwd_noalloc(_p(q), _p(q), _p(q), _lib.DTYPE_BF16, 1, 1, huge, huge, 128, _strides(q),
                                      _strides(q), _strides(q), 0.088, _lib.MODE_BLOCK64, _p(o), _strides(o),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc != 0
    assert b"scratch" in lib.dc_last_error()
