"""The key-split INT8 attention (kernels.attn_int8_split -> dc_attn_int8_main_split:
attn_int8_kernel<..., SPLIT> over key ranges + attn_split_combine_kernel) on a B200: within the
attention tolerance of the CPU oracle (max-abs 2e-2, cosine >= 0.999) and within rounding of the
unsplit two-tile kernel it divides (cosine >= 0.99999), over ranges that end in a key tail, one
key tile per range, query tails, D = 64, fp16 and both quant modes; the default routing of
kernels.attn_int8 (DC_ATTN_SPLIT=0 turns it off)."""

from __future__ import annotations

import pytest
import torch

import oracle
from diffucore_b200 import _lib, kernels
from tests.conftest import DTAG, torch_to_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
MODES = {"ref": _lib.MODE_REF, "block64": _lib.MODE_BLOCK64}


def _inputs(B, Lq, Lk, H, D, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Lq, H, D, generator=g).to(dtype)
    k = (torch.randn(B, Lk, H, D, generator=g) + 0.5).to(dtype)
    v = torch.randn(B, Lk, H, D, generator=g).to(dtype)
    return q, k, v


def _cos(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return float((a @ b) / (a.norm() * b.norm()))


@pytest.mark.parametrize("mode", ["ref", "block64"])
@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 128), (torch.bfloat16, 64)])
@pytest.mark.parametrize("B,Lq,Lk,H,nsplit", [(1, 4608, 4608, 3, 2), (1, 700, 3953, 2, 4), (2, 300, 640, 2, 5),
                                              (1, 256, 1000, 1, 8), (1, 70, 129, 2, 2)])
def test_split_matches_oracle_and_unsplit(monkeypatch, mode, dtype, D, B, Lq, Lk, H, nsplit):
    monkeypatch.setenv("DC_ATTN_KERNEL", "two_tile")
    monkeypatch.setenv("DC_ATTN_SPLIT", "0")
    q, k, v = _inputs(B, Lq, Lk, H, D, dtype)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    sm = D ** -0.5
    got = kernels.attn_int8_split(qd, kd, vd, sm, nsplit, MODES[mode])
    whole = kernels.attn_int8(qd, kd, vd, sm, MODES[mode])
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert got.shape == whole.shape and got.dtype == dtype
    g, w = got.float().cpu(), whole.float().cpu()
    assert torch.isfinite(g).all()
    assert _cos(g, w) >= 0.99999 and (g - w).abs().max() < 1e-2
    bits = torch_to_bits
    ref = torch.from_numpy(oracle.attn_int8(bits(q), bits(k), bits(v), DTAG[dtype], sm, mode)).reshape(g.shape)
    assert (g - ref).abs().max() < 2e-2 and _cos(g, ref) >= 0.999


def test_split_is_deterministic():
    q, k, v = (t.to(DEV) for t in _inputs(1, 1024, 4608, 3, 128, torch.bfloat16, seed=4))
    a = kernels.attn_int8_split(q, k, v, 128 ** -0.5, 3)
    b = kernels.attn_int8_split(q, k, v, 128 ** -0.5, 3)
    assert torch.equal(a, b)


def test_auto_routing_splits_few_heads(monkeypatch):
    """The default dispatch sends a 3-head 16896-token call (FLUX 2048^2 on 8 GPUs) through the
    split path, whose result equals an explicit split call bit for bit; DC_ATTN_SPLIT=0 turns the
    routing off (the unsplit kernel's result)."""
    q, k, v = (t.to(DEV) for t in _inputs(1, 16896, 16896, 3, 128, torch.bfloat16, seed=6))
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    nsplit = kernels.choose_attn_split(1, 3, 16896, 16896, sms)
    assert nsplit > 1
    monkeypatch.delenv("DC_ATTN_SPLIT", raising=False)
    routed = kernels.attn_int8(q, k, v, 128 ** -0.5, _lib.MODE_REF)
    explicit = kernels.attn_int8_split(q, k, v, 128 ** -0.5, nsplit, _lib.MODE_REF)
    assert torch.equal(routed, explicit)
    monkeypatch.setenv("DC_ATTN_SPLIT", "0")
    plain = kernels.attn_int8(q, k, v, 128 ** -0.5, _lib.MODE_REF)
    assert not torch.equal(plain, routed)
    assert _cos(plain.float().cpu(), routed.float().cpu()) >= 0.99999


def test_running_max_moves_inside_a_range():
    """Scores growing along the keys: every range's running max moves tile by tile (the lazy O
    rescale inside each range) and the ranges' maxima differ widely (the combine weights)."""
    L, H, D = 2048, 2, 128
    g = torch.Generator().manual_seed(8)
    q = torch.ones(1, L, H, D)
    k = torch.linspace(0.0, 3.0, L).view(1, L, 1, 1).expand(1, L, H, D) + 0.01 * torch.randn(1, L, H, D, generator=g)
    v = torch.randn(1, L, H, D, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    got = kernels.attn_int8_split(q.to(DEV), k.to(DEV), v.to(DEV), D ** -0.5, 4, _lib.MODE_BLOCK64).float().cpu()
    ref = torch.from_numpy(oracle.attn_int8(torch_to_bits(q), torch_to_bits(k), torch_to_bits(v), "bf16",
                                            D ** -0.5, "block64")).reshape(got.shape)
    assert torch.isfinite(got).all()
    assert (got - ref).abs().max() < 2e-2 and _cos(got, ref) >= 0.999
