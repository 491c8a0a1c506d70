"""Attention dispatch semantics on CPU, mirroring the reference's tests/test_attention_dispatch.py:
the SDPA branch is bit-exact with plain scaled_dot_product_attention, a stamped "int8_turing" or
"fa2_turing" module still runs off the GPU (the per-call guard reroutes to SDPA, same numbers),
"auto" resolves silently to SDPA, an explicit backend that cannot run raises and names every
unmet requirement, the INT8 backend is stamped on self-attention only, and null keys equal
explicit zero padding. The INT8 kernel's numerics are covered by the GPU tests."""

from __future__ import annotations

from dataclasses import dataclass

import pytest
import torch
import torch.nn.functional as F

from diffucore_b200 import _attention, flux, unet
from diffucore_b200._attention import (attention_bhld, attention_blhd, fa2_turing_available,
                                       int8_turing_available, resolve_attention_backend,
                                       set_attention_backend)


@dataclass
class Policy:
    """The fields of the reference's DevicePolicy that backend resolution reads."""
    device: torch.device = torch.device("cpu")
    compute_dtype: torch.dtype = torch.float32
    attention: str = "sdpa"
    compile: bool = False


def _ref_blhd(q, k, v):
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return out.transpose(1, 2).reshape(q.shape[0], q.shape[1], -1)


def test_blhd_sdpa_matches_manual():
    torch.manual_seed(0)
    q, k, v = torch.randn(2, 64, 4, 32), torch.randn(2, 48, 4, 32), torch.randn(2, 48, 4, 32)
    assert torch.equal(attention_blhd(q, k, v, "sdpa"), _ref_blhd(q, k, v))


def test_bhld_sdpa_matches_manual():
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 4, 64, 32) for _ in range(3))
    ref = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(2, 64, -1)
    assert torch.equal(attention_bhld(q, k, v, "sdpa"), ref)


@pytest.mark.parametrize("backend", ["fa2_turing", "int8_turing"])
def test_stamped_backend_falls_back_off_gpu(backend):
    torch.manual_seed(0)
    q = torch.randn(1, 16, 2, 128)
    assert torch.equal(attention_blhd(q, q, q, backend), attention_blhd(q, q, q, "sdpa"))
    qh = q.transpose(1, 2)
    assert torch.equal(attention_bhld(qh, qh, qh, backend), attention_bhld(qh, qh, qh, "sdpa"))


def test_int8_falls_back_for_other_head_dims_and_dtypes():
    torch.manual_seed(0)
    for shape, dtype in (((1, 16, 2, 96), torch.float16), ((1, 16, 2, 128), torch.float32)):
        q = torch.randn(*shape).to(dtype)
        assert torch.equal(attention_blhd(q, q, q, "int8_turing"), attention_blhd(q, q, q, "sdpa"))


def test_resolve_sdpa_is_default_and_inert():
    assert resolve_attention_backend(Policy()) == "sdpa"


def test_resolve_auto_falls_back_silently_on_cpu():
    assert resolve_attention_backend(Policy(attention="auto")) == "sdpa"


@pytest.mark.parametrize("backend", ["fa2_turing", "int8_turing"])
def test_resolve_explicit_backend_raises_on_cpu(backend):
    with pytest.raises(ValueError, match=backend) as err:
        resolve_attention_backend(Policy(attention=backend))
    assert "device is not CUDA" in str(err.value)


@pytest.mark.parametrize("backend", ["fa2_turing", "int8_turing"])
def test_resolve_explicit_backend_raises_with_compile(backend):
    with pytest.raises(ValueError, match="compile"):
        resolve_attention_backend(Policy(compute_dtype=torch.float16, attention=backend, compile=True))


def test_resolve_rejects_unknown_attention_value():
    with pytest.raises(ValueError, match="attention"):
        resolve_attention_backend(Policy(attention="flash3"))


def test_availability_off_gpu():
    assert not fa2_turing_available()
    assert not int8_turing_available("cpu")


def test_int8_arch_is_sm100_only(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    for cap, want in (((7, 5), None), ((8, 6), None), ((9, 0), None), ((10, 0), "100a"), ((12, 0), None)):
        monkeypatch.setattr(torch.cuda, "get_device_capability", lambda d=None, c=cap: c)
        assert _attention._int8_arch() == want


def _tiny_flux_blocks():
    cfg = flux.FluxConfig(hidden_size=64, num_heads=2, mlp_ratio=2.0, depth=1, depth_single_blocks=1)
    return flux.DoubleStreamBlock(cfg), flux.SingleStreamBlock(cfg)


def test_int8_stamps_self_attention_only():
    """FLUX's joint attention and UNet self-attention get the INT8 kernel; UNet cross-attention
    keeps the exact backend."""
    double, single = _tiny_flux_blocks()
    self_attn = unet.CrossAttention(64, 64, 2, 32, is_selfattn=True)
    cross_attn = unet.CrossAttention(64, 48, 2, 32, is_selfattn=False)
    holder = torch.nn.ModuleList([double, single, self_attn, cross_attn])
    assert all(m.attn_backend == "sdpa" for m in (double, single, self_attn, cross_attn))
    assert set_attention_backend(holder, "int8_turing") == 4
    assert double.attn_backend == single.attn_backend == self_attn.attn_backend == "int8_turing"
    assert cross_attn.attn_backend == "sdpa"
    assert set_attention_backend(holder, "sdpa") == 4
    assert cross_attn.attn_backend == "sdpa" and double.attn_backend == "sdpa"


def test_stamped_attention_forward_unchanged_on_cpu():
    """End to end through an attention module: stamping the INT8 backend on a CPU module changes
    nothing (the guard reroutes), so offline forwards stay exact."""
    torch.manual_seed(0)
    attn = unet.CrossAttention(64, 64, 2, 32, is_selfattn=True).eval()
    x = torch.randn(1, 16, 64)
    with torch.no_grad():
        before = attn(x)
        set_attention_backend(attn, "int8_turing")
        after = attn(x)
    assert attn.attn_backend == "int8_turing"
    assert torch.equal(before, after)


def test_null_keys_sdpa_equals_padded():
    torch.manual_seed(0)
    n = 5
    q = torch.randn(1, 300, 4, 128)
    k = torch.randn(1, 77, 4, 128)
    v = torch.randn(1, 77, 4, 128)
    pad = (0, 0, 0, 0, 0, n)
    assert torch.equal(attention_blhd(q, k, v, null_keys=n), attention_blhd(q, F.pad(k, pad), F.pad(v, pad)))
