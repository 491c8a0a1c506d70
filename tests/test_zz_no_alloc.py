"""The attention entry point for callers that cannot allocate device memory.

Some applications own all of their GPU memory through their own pool (or run where cudaMalloc's
implicit synchronization is not allowed) and so cannot pass this library a workspace.
`dc_attn_int8_fwd_noalloc` keeps the attention's intermediate Q/K codes and scales in one fixed
device array inside the library instead. These tests call it through the C-ABI and check that it
gives exactly what the workspace entry point `dc_attn_int8_fwd` gives (both run the same kernels on
the same inputs; only where the codes live differs, so the outputs are bit-identical), on calls in
a row whose shapes shrink (the later calls reuse an array that the earlier, larger ones left
filled), and that shapes too large for the fixed array are refused with a clear error.

The file name sorts last so that pytest collects it after every other test file: a run that stops
at the first failure has then already run the rest of the suite. It passes alone in a fresh
process as well as after the other tests.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from diffucore_b200 import _lib

pytestmark = pytest.mark.gpu

_CODE = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


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
    rc = lib.dc_attn_int8_fwd(_p(q), _p(k), _p(v), _CODE[q.dtype], B, H, L, L, D, _strides(q), _strides(k),
                              _strides(v), D ** -0.5, mode, _p(o), _strides(o), _p(ws), ws.numel(),
                              ctypes.c_void_p(st))
    assert rc == 0, lib.dc_last_error()
    return o


def _without_allocation(lib, q, k, v, mode):
    B, L, H, D = q.shape
    o = torch.empty(B, L, H, D, device="cuda", dtype=q.dtype)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.dc_attn_int8_fwd_noalloc(_p(q), _p(k), _p(v), _CODE[q.dtype], B, H, L, L, D, _strides(q),
                                      _strides(k), _strides(v), D ** -0.5, mode, _p(o), _strides(o),
                                      ctypes.c_void_p(st))
    assert rc == 0, lib.dc_last_error()
    return o


# (seed, B, L, H, D, dtype): the largest first, then smaller ones with query / key tails
_SEQUENCE = [(11, 1, 4000, 4, 128, torch.bfloat16),
             (12, 2, 1000, 3, 128, torch.bfloat16),
             (13, 1, 300, 2, 128, torch.float16),
             (14, 2, 777, 5, 64, torch.bfloat16),
             (15, 1, 70, 3, 64, torch.float16)]


@pytest.mark.parametrize("mode", [_lib.MODE_REF, _lib.MODE_BLOCK64])
def test_no_alloc_matches_workspace_entry_point_in_a_row(mode):
    lib = _lib.load()
    for seed, B, L, H, D, dtype in _SEQUENCE:      # calls in a row; each reuses the array as left
        q, k, v = _inputs(seed, B, L, H, D, dtype)
        got = _without_allocation(lib, q, k, v, mode)
        want = _with_workspace(lib, q, k, v, mode)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert torch.equal(got, want), (seed, L, D, dtype)


def test_no_alloc_twice_same_shape_new_inputs():
    lib = _lib.load()
    for seed in (21, 22):                      # two calls in a row, same shape, different inputs
        q, k, v = _inputs(seed)
        got = _without_allocation(lib, q, k, v, _lib.MODE_REF)
        want = _with_workspace(lib, q, k, v, _lib.MODE_REF)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


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
