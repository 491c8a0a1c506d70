"""Pins the attention oracle (and the product) to the REFERENCE's own CUDA kernels, built from the
reference's source into oracle/_ref/ by oracle/build_ref.py (skipped when that checker was not
built). The reference's prep kernels must give the oracle's K codes, K scales and K column sums bit
for bit; the reference's fp16 attention output must agree with the oracle's exact-softmax result
and with this package's output to the reference's own per-call error budget."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import build_ref
from diffucore_b200 import _attention
from tests.conftest import torch_to_bits

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not build_ref.available(), reason="reference checker not built")]


@pytest.fixture(scope="module")
def ref_mod():
    return build_ref.load()


@pytest.mark.parametrize("B,L,H", [(1, 77, 2), (2, 1000, 3), (1, 4608, 4), (1, 300, 1)])
def test_reference_k_prep_equals_oracle(ref_mod, B, L, H):
    g = torch.Generator().manual_seed(L)
    k = (torch.randn(B, L, H, 128, generator=g) + 0.5).half()
    ki, ks, ksum = torch.ops.dcref.k_prep(k.cuda())
    want = oracle.attn_prep(torch_to_bits(k), torch_to_bits(k), "f16", "ref")
    assert np.array_equal(ksum.cpu().numpy(), want["ksum"])
    assert np.array_equal(ks.cpu().numpy()[:, :, : want["k_scale"].shape[2]], want["k_scale"])
    assert np.array_equal(ki.cpu().numpy()[:, :, :L], want["k_codes"])


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 1024, 1024, 4), (1, 700, 77, 4), (1, 70, 3953, 2)])
def test_reference_output_agrees_with_oracle_and_product(ref_mod, B, Lq, Lk, H):
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, Lq, H, 128, generator=g).half()
    k = (torch.randn(B, Lk, H, 128, generator=g) + 0.5).half()
    v = torch.randn(B, Lk, H, 128, generator=g).half()
    ref = ref_mod.fwd(q.cuda(), k.cuda(), v.cuda(), 128 ** -0.5).float().cpu().reshape(B, Lq, H, 128)
    want = torch.from_numpy(oracle.attn_int8(torch_to_bits(q), torch_to_bits(k), torch_to_bits(v), "f16",
                                             128 ** -0.5, "ref"))
    ours = _attention.attention_blhd(q.cuda(), k.cuda(), v.cuda(), "int8_turing").float().cpu().reshape(want.shape)
    for got in (ref, ours):
        assert (got - want).abs().max() < 2e-2
        cos = torch.nn.functional.cosine_similarity(got.flatten().double(), want.flatten().double(), dim=0)
        assert cos >= 0.999
    assert (ours - ref).abs().max() < 2e-2
