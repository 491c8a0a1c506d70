"""The rotated row quantizers against each other, bit for bit: the register-row kernel
(rowq_reg_kernel, the default), the packed-pair shared-memory kernels (rowq_pair_kernel,
rowq_cta_pair_kernel: DC_ROWQ_REG=0) and the one-group kernels (DC_ROWQ_REG=0 DC_ROWQ_PAIR=0),
on plain rows with ConvRot (quant_rows, group 256) and on the segmented rows of an all-to-all
receive buffer (quant_rows_seg), over widths with a partial last warp (groups past the row).
LayerNorm + modulation (ln_mod_quant): the shared-memory kernels agree bit for bit; the register
kernel sums the row's mean and variance in another order, so its codes are held to one step."""

from __future__ import annotations

import pytest
import torch

from diffucore_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
DEV = "cuda"

_VARIANTS = ({"DC_ROWQ_REG": "0", "DC_ROWQ_PAIR": "0"}, {"DC_ROWQ_REG": "0"}, {})


def _all(monkeypatch, fn):
    out = []
    for env in _VARIANTS:
        monkeypatch.delenv("DC_ROWQ_REG", raising=False)
        monkeypatch.delenv("DC_ROWQ_PAIR", raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        out.append(fn())
    monkeypatch.delenv("DC_ROWQ_REG", raising=False)
    monkeypatch.delenv("DC_ROWQ_PAIR", raising=False)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return out


def _assert_equal(results):
    (qa, sa) = results[0]
    for qb, sb in results[1:]:
        assert torch.equal(qa, qb) and torch.equal(sa, sb)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(4608, 3072), (333, 256), (100, 1280), (77, 4096), (5, 768), (4608, 15360),
                                 (300, 12288), (33, 4352), (7, 16384)])
def test_quant_rows_group256_bit_exact(monkeypatch, dtype, M, K):
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * 2).to(dtype).to(DEV)
    x[min(3, M - 1)] = 0                                     # a zero row
    _assert_equal(_all(monkeypatch, lambda: kernels.quant_rows(x, 256)))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K", [(4608, 3072), (64, 256), (300, 1280)])
def test_ln_mod_quant_bit_exact(monkeypatch, dtype, M, K):
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(M, K, generator=g) * 3 + 0.5).to(dtype).to(DEV)
    shift = (torch.randn(K, generator=g) * 0.3).to(dtype).to(DEV)
    scale = (torch.randn(K, generator=g) * 0.3).to(dtype).to(DEV)
    one, pair, reg = _all(monkeypatch, lambda: kernels.ln_mod_quant(x, shift, scale, 256))
    _assert_equal([one, pair])
    diff = (reg[0].int() - pair[0].int()).abs()
    assert diff.max().item() <= 1
    assert diff.ne(0).float().mean().item() < 5e-3
    assert ((reg[1] - pair[1]).abs() / pair[1]).max().item() < 8e-3


@pytest.mark.parametrize("P,W,K2", [(2, 1536, 0), (8, 384, 0), (8, 384, 12288), (1, 3072, 12288), (16, 192, 0)])
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

    _assert_equal(_all(monkeypatch, run))


@pytest.mark.parametrize("M,K", [(4096, 3072), (129, 256), (300, 1280), (64, 15360)])
def test_quant_rows_plain_register_kernel_bit_exact(monkeypatch, M, K):
    """Plain (unrotated) rows through the register-row kernel (DC_ROWQ_REG=2) against the
    default plain-row kernels."""
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(M, K, generator=g) * 2).to(torch.bfloat16).to(DEV)
    x[0] = 0
    want = kernels.quant_rows(x, 0)
    monkeypatch.setenv("DC_ROWQ_REG", "2")
    got = kernels.quant_rows(x, 0)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
