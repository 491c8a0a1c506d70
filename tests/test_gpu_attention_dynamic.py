"""The two-tile INT8 attention kernel with dynamic MMA issue (``DC_ATTN_ISSUE=dynamic``) against
the same kernel with its fixed issue order.

Only the order in which the MMA thread interleaves the two Q tiles' groups changes; within a tile
the Q.K^T and P.V groups, and so the TMEM accumulation order, stay the same, and the softmax warps
run the same code. The outputs must therefore be bit-identical, on BASELINE config 2, on ragged
sequence lengths (tail key tiles, a single key tile) and on scores whose running max moves every
tile (the O-rescale path).

Opt-in until the variant has run on a B200: set ``DC_TEST_ATTN_DYN=1``.
"""

from __future__ import annotations

import os

import pytest
import torch

from diffucore_b200 import _lib, kernels

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("DC_TEST_ATTN_DYN") != "1",
                       reason="dynamic-issue attention is opt-in until run on a B200 (DC_TEST_ATTN_DYN=1)"),
]
DEV = "cuda"


def _run(monkeypatch, q, k, v, mode, dynamic):
    monkeypatch.setenv("DC_ATTN_KERNEL", "two_tile")
    if dynamic:
        monkeypatch.setenv("DC_ATTN_ISSUE", "dynamic")
    else:
        monkeypatch.delenv("DC_ATTN_ISSUE", raising=False)
    out = kernels.attn_int8(q, k, v, q.shape[-1] ** -0.5, mode)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return out


@pytest.mark.parametrize("mode", [_lib.MODE_REF, _lib.MODE_BLOCK64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Lq,Lk,H,D", [(1, 4608, 4608, 24, 128), (2, 300, 77, 3, 128), (1, 513, 1000, 2, 64),
                                         (1, 256, 129, 1, 128)])
def test_dynamic_issue_bit_identical(monkeypatch, mode, dtype, B, Lq, Lk, H, D):
    g = torch.Generator().manual_seed(Lq + Lk)
    q = torch.randn(B, Lq, H, D, generator=g).to(dtype).to(DEV)
    k = (torch.randn(B, Lk, H, D, generator=g) + 0.5).to(dtype).to(DEV)
    v = torch.randn(B, Lk, H, D, generator=g).to(dtype).to(DEV)
    fixed = _run(monkeypatch, q, k, v, mode, False)
    dyn = _run(monkeypatch, q, k, v, mode, True)
    assert torch.equal(fixed, dyn)


def test_dynamic_issue_with_moving_max(monkeypatch):
    """Keys whose scores grow along the sequence, so every tile raises the running max."""
    g = torch.Generator().manual_seed(9)
    L, H, D = 2048, 2, 128
    q = torch.randn(1, L, H, D, generator=g)
    ramp = torch.linspace(0.2, 24.0, L)[None, :, None, None]
    k = torch.randn(1, L, H, D, generator=g) * ramp / D ** 0.5 + q.mean(dim=1, keepdim=True) * ramp
    v = torch.randn(1, L, H, D, generator=g)
    q, k, v = (t.to(torch.bfloat16).to(DEV) for t in (q, k, v))
    fixed = _run(monkeypatch, q, k, v, _lib.MODE_BLOCK64, False)
    dyn = _run(monkeypatch, q, k, v, _lib.MODE_BLOCK64, True)
    assert torch.equal(fixed, dyn)
