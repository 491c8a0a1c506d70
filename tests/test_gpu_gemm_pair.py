"""The two-CTA (``cta_group::2``, 256 x 256 tile) W8A8 GEMM against the one-CTA kernel.

Both compute the same integer dot products and apply the same epilogue per element, so every
output (int32 accumulators, rescaled bf16 / fp16 with bias and GELU, the gated residual, the
column-block layout) must be bit-identical; the int32 result is also checked against
``torch._int_mm``. Shapes cover BASELINE config 1, FLUX's widest reduction (K = 15360), and row /
column tails where the odd CTA of a pair holds no valid rows.

The pair kernel is the default for wide GEMMs of at least 512 rows without GELU; the tests force it
with ``DC_GEMM_PAIR=1`` and the one-CTA kernel with ``DC_GEMM_PAIR=0``.
"""

from __future__ import annotations

import pytest
import torch

from diffucore_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
DEV = "cuda"

SHAPES = [(4096, 3072, 3072), (4608, 3072, 15360), (300, 640, 512), (129, 257, 4096), (200, 1000, 256),
          (4160, 9216, 3072)]


def _operands(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(DEV)
    sx = (torch.rand(M, generator=g) * 0.02 + 1e-3).to(DEV)
    sw = (torch.rand(N, generator=g) * 0.002 + 1e-4).to(DEV)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    return q, w, sx, sw, bias


def _both(monkeypatch, fn):
    monkeypatch.setenv("DC_GEMM_PAIR", "0")
    one = fn()
    monkeypatch.setenv("DC_GEMM_PAIR", "1")
    pair = fn()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return one, pair


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_pair_int32_bit_exact(monkeypatch, M, N, K):
    q, w, *_ = _operands(M, N, K, 1)
    one, pair = _both(monkeypatch, lambda: kernels.gemm_w8a8(q, w, None, None, None, torch.int32))
    assert torch.equal(one, pair)
    if K % 8 == 0 and N % 8 == 0:
        assert torch.equal(pair, torch._int_mm(q, w.t()))


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("dtype,gelu", [(torch.bfloat16, _lib.GELU_NONE), (torch.float16, _lib.GELU_NONE),
                                        (torch.bfloat16, _lib.GELU_TANH)])
def test_pair_epilogue_bit_exact(monkeypatch, M, N, K, dtype, gelu):
    q, w, sx, sw, bias = _operands(M, N, K, 2)
    one, pair = _both(monkeypatch, lambda: kernels.gemm_w8a8(q, w, sx, sw, bias.to(dtype), dtype, gelu))
    assert torch.equal(one, pair)


@pytest.mark.parametrize("M,N,K", [(4608, 3072, 15360), (300, 640, 512)])
def test_pair_gated_residual_bit_exact(monkeypatch, M, N, K):
    q, w, sx, sw, bias = _operands(M, N, K, 3)
    g = torch.Generator().manual_seed(4)
    gate = (torch.randn(N, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV)

    def run():
        out = res.clone()
        kernels.gemm_w8a8_into(q, w, sx, sw, bias, out, gate=gate, residual=out)
        return out

    one, pair = _both(monkeypatch, run)
    assert torch.equal(one, pair)


@pytest.mark.parametrize("P", [2, 4])
def test_pair_column_blocks_bit_exact(monkeypatch, P):
    M, C = 1333, 1024
    q, w, sx, sw, bias = _operands(M, 3 * C, C, 5)
    Wd = 3 * C // P

    def run():
        out = torch.empty(P * M * Wd, device=DEV, dtype=torch.bfloat16)
        kernels.gemm_w8a8_into(q, w, sx, sw, bias, out, ldo=Wd, col_block=Wd, block_stride=M * Wd)
        return out

    one, pair = _both(monkeypatch, run)
    assert torch.equal(one, pair)
