"""The packed-pair rotated row quantizers (rowq_pair_kernel, rowq_cta_pair_kernel: the default
for group 256) against the one-group kernels they replaced (DC_ROWQ_PAIR=0), bit for bit: plain
rows with ConvRot (quant_rows, group 256), LayerNorm + modulation (ln_mod_quant), and the
segmented rows of an all-to-all receive buffer (quant_rows_seg), over widths with a partial last
iteration (groups past the row)."""

from __future__ import annotations

import pytest
import torch

from diffucore_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _both(monkeypatch, fn):
    monkeypatch.setenv("DC_ROWQ_PAIR", "0")                  # one-group kernels
    a = fn()
    monkeypatch.delenv("DC_ROWQ_PAIR", raising=False)        # default: packed pairs
    b = fn()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(4608, 3072), (333, 256), (100, 1280), (77, 4096), (5, 768), (4608, 15360),
                                 (300, 12288), (33, 4352), (7, 16384)])
def test_quant_rows_group256_bit_exact(monkeypatch, dtype, M, K):
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * 2).to(dtype).to(DEV)
    x[min(3, M - 1)] = 0                                     # a zero row
    (qa, sa), (qb, sb) = _both(monkeypatch, lambda: kernels.quant_rows(x, 256))
    assert torch.equal(qa, qb) and torch.equal(sa, sb)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(4608, 3072), (64, 256), (300, 1280)])
def test_ln_mod_quant_bit_exact(monkeypatch, dtype, M, K):
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(M, K, generator=g) * 3 + 0.5).to(dtype).to(DEV)
    shift = (torch.randn(K, generator=g) * 0.3).to(dtype).to(DEV)
    scale = (torch.randn(K, generator=g) * 0.3).to(dtype).to(DEV)
    (qa, sa), (qb, sb) = _both(monkeypatch, lambda: kernels.ln_mod_quant(x, shift, scale, 256))
    assert torch.equal(qa, qb) and torch.equal(sa, sb)


@pytest.mark.parametrize("P,W,K2", [(2, 1536, 0), (8, 384, 0), (8, 384, 12288), (1, 3072, 12288)])
def test_quant_rows_seg_bit_exact(monkeypatch, P, W, K2):
    g = torch.Generator().manual_seed(P + K2)
    M = 211
    recv = torch.randn(P, M, W, generator=g).to(torch.bfloat16).to(DEV)
    x2 = torch.randn(M, K2 + 64, generator=g).to(torch.bfloat16).to(DEV)[:, 64:] if K2 else None

    def run():
        q = torch.empty(M, P * W + K2, device=DEV, dtype=torch.int8)
        s = torch.empty(M, device=DEV, dtype=torch.float32)
        kernels.quant_rows_seg(recv, x2, 256, q, s)
        return q, s

    (qa, sa), (qb, sb) = _both(monkeypatch, run)
    assert torch.equal(qa, qb) and torch.equal(sa, sb)
