"""The CTA-pair INT8 attention kernel (``DC_ATTN_KERNEL=pair``, D = 128) against the one-CTA
two-tile kernel and the oracle.

The pair kernel runs the same per-row arithmetic (exact int32 Q.K^T, the same softmax code, P.V
on the tensor core with fp32 accumulation); only the split of the MMAs over two SMs differs, so
its output is expected to equal the one-CTA kernel's, and must in any case stay within the
attention tolerance of the oracle. Shapes cover BASELINE config 2, query lengths whose last pair
reaches past the padded rows, ragged key lengths, several batches and heads.

Opt-in until the kernel has run on a B200: set ``DC_TEST_ATTN_PAIR=1``.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
from diffucore_b200 import _lib, kernels
from tests.conftest import DTAG, torch_to_bits

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("DC_TEST_ATTN_PAIR") != "1",
                       reason="CTA-pair attention is opt-in until run on a B200 (DC_TEST_ATTN_PAIR=1)"),
]
DEV = "cuda"


def _run(monkeypatch, q, k, v, mode, kernel):
    monkeypatch.setenv("DC_ATTN_KERNEL", kernel)
    monkeypatch.delenv("DC_ATTN_ISSUE", raising=False)
    out = kernels.attn_int8(q, k, v, q.shape[-1] ** -0.5, mode)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    return out


@pytest.mark.parametrize("mode", [_lib.MODE_REF, _lib.MODE_BLOCK64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 4608, 4608, 24), (2, 300, 77, 3), (1, 513, 1000, 2), (1, 1024, 129, 1)])
def test_pair_matches_one_cta_kernel(monkeypatch, mode, dtype, B, Lq, Lk, H):
    g = torch.Generator().manual_seed(Lq + Lk + H)
    q = torch.randn(B, Lq, H, 128, generator=g).to(dtype).to(DEV)
    k = (torch.randn(B, Lk, H, 128, generator=g) + 0.5).to(dtype).to(DEV)
    v = torch.randn(B, Lk, H, 128, generator=g).to(dtype).to(DEV)
    one = _run(monkeypatch, q, k, v, mode, "two_tile").float()
    pair = _run(monkeypatch, q, k, v, mode, "pair").float()
    assert torch.isfinite(pair).all()
    if not torch.equal(one, pair):
        cos = torch.nn.functional.cosine_similarity(one.flatten().double(), pair.flatten().double(), dim=0).item()
        assert (one - pair).abs().max().item() <= 4e-3 and cos >= 0.99999


@pytest.mark.parametrize("mode", ["ref", "block64"])
def test_pair_against_oracle(monkeypatch, mode):
    g = torch.Generator().manual_seed(17)
    B, Lq, Lk, H = 1, 600, 700, 2
    q = torch.randn(B, Lq, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, generator=g).to(torch.bfloat16)
    code = _lib.MODE_REF if mode == "ref" else _lib.MODE_BLOCK64
    out = _run(monkeypatch, q.to(DEV), k.to(DEV), v.to(DEV), code, "pair").float().cpu().numpy()
    ref = oracle.attn_int8(torch_to_bits(q), torch_to_bits(k), torch_to_bits(v), DTAG[torch.bfloat16],
                           128 ** -0.5, mode)
    assert np.abs(out - ref).max() <= 2e-2
    cos = float((out.ravel() @ ref.ravel()) / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert cos >= 0.999
