"""CPU parts of the Int8Linear module API (load-time helpers), mirroring the reference's own
tests/test_int8.py and the Int8Embedding tests of tests/test_moss_image.py: the ConvRot Hadamard
is symmetric and its own inverse, a weight survives quantize -> dequantize within 1 % relative
error with and without rotation, the scale survives a dtype cast, a sub-step LoRA delta
requantizes unbiased and reproducibly, quantize_linears / dequantize_linears round-trip, and the
int8 embedding table gathers and adopts like the reference's. The module's load-time helpers agree
with the reference's torch-op path (oracle/torch_ref.py). The W8A8 forward itself has no CPU path."""

from __future__ import annotations

import pytest
import torch

from diffucore_b200 import _int8
from oracle import torch_ref


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_hadamard_is_symmetric_and_self_inverse():
    h = _int8._hadamard(256, "cpu")
    torch.testing.assert_close(h, h.T)
    torch.testing.assert_close(h @ h, torch.eye(256), atol=1e-6, rtol=0)
    assert torch.equal(h, torch_ref.hadamard(256))


@pytest.mark.parametrize("group", [0, 256])
def test_weight_round_trip(group):
    torch.manual_seed(0)
    w = torch.randn(64, 512) * 0.02
    q, s = _int8.quantize_weight(w, group)
    assert _rel(_int8.dequantize_weight(q, s, group), w) < 0.01
    qr, sr = torch_ref.quantize_weight(w, group)
    assert torch.equal(q, qr) and torch.equal(s, sr)


def test_forward_refuses_cpu_tensors():
    """No CPU fallback in the product: the W8A8 forward needs the CUDA library."""
    lin = torch.nn.Linear(256, 64)
    m = _int8.Int8Linear.from_linear(lin, group=0)
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        m(torch.randn(4, 256))


def test_scale_survives_dtype_cast():
    """Casting the module (as pipelines do with `.to(dtype)`) keeps the int8 weight and the fp32
    scale bits (reference tests/test_int8.py:61-65)."""
    m = _int8.Int8Linear.from_linear(torch.nn.Linear(256, 32))
    s = m.scale.clone()
    m.to(torch.float16)
    assert m.weight.dtype == torch.int8 and torch.equal(m.scale, s)
    assert m.bias.dtype == torch.float16


@pytest.mark.parametrize("group", [0, 256])
def test_add_delta_requantizes_unbiased(group):
    """A LoRA delta of ~0.2 int8 steps still lands on average (seeded stochastic rounding keeps
    its mean) and the same seed gives the same bytes (reference tests/test_int8.py:107-140, the
    requantization half; LoRA file parsing is not part of this package)."""
    torch.manual_seed(3)
    lin = torch.nn.Linear(512, 96)
    m = _int8.Int8Linear.from_linear(lin, group)
    q0, s0 = m.weight.clone(), m.scale.clone()
    before = _int8.dequantize_weight(q0, s0, group)
    g = torch.Generator().manual_seed(3)
    down = torch.randn(4, 512, generator=g)
    up = torch.randn(96, 4, generator=g)
    k = 0.2 * s0.mean().item() / (up @ down).std().item()
    delta = (up @ down) * k
    seed = _int8.lora_seed("blocks.0.mlp.layer1", "lora.safetensors")
    m.add_delta_(delta, seed)
    change = _int8.dequantize_weight(m.weight, m.scale, group) - before
    gain = ((change * delta).sum() / (delta * delta).sum()).item()
    assert 0.9 < gain < 1.1
    again = _int8.Int8Linear.from_linear(lin, group)
    again.add_delta_(delta, seed)
    assert torch.equal(again.weight, m.weight) and torch.equal(again.scale, m.scale)


def test_quantize_then_dequantize_linears():
    """`quantize_linears` swaps the named layers for Int8Linear (ConvRot group 256 where the width
    allows it), `dequantize_linears` turns them back into plain layers close to the originals
    (reference tests/test_int8.py:74-91, the round-trip half)."""
    torch.manual_seed(1)
    ref = torch.nn.Sequential(torch.nn.Linear(512, 256, bias=False), torch.nn.GELU(), torch.nn.Linear(256, 128))
    model = torch.nn.Sequential(torch.nn.Linear(512, 256, bias=False), torch.nn.GELU(), torch.nn.Linear(256, 128))
    model.load_state_dict(ref.state_dict())
    assert _int8.quantize_linears(model, ["0", "2"], "cpu") == 2
    assert isinstance(model[0], _int8.Int8Linear) and model[0].group == 256
    assert isinstance(model[2], _int8.Int8Linear) and model[2].bias is not None
    assert _int8.dequantize_linears(model, torch.float32) == 2
    assert type(model[0]) is torch.nn.Linear and type(model[2]) is torch.nn.Linear
    x = torch.randn(8, 512)
    with torch.no_grad():
        assert _rel(model(x), ref(x)) < 0.02


def test_int8_embedding_rows_equal_the_dequantized_table():
    """Int8Embedding gathers, rescales and un-rotates only the requested rows (reference
    tests/test_moss_image.py:281-293)."""
    torch.manual_seed(0)
    table = torch.randn(50, 512) * 0.02
    q, scale = _int8.quantize_weight(table, 256)
    emb = _int8.Int8Embedding(50, 512, 256)
    emb.weight.copy_(q)
    emb.scale_bits.copy_(scale.view(torch.int32))
    ids = torch.tensor([[3, 7, 3], [0, 49, 10]])
    want = _int8.dequantize_weight(q, scale, 256)[ids]
    torch.testing.assert_close(emb(ids), want, rtol=1e-5, atol=1e-8)
    assert emb(ids).shape == (2, 3, 512)
    assert _rel(emb(ids), table[ids]) < 0.01
    emb.out_dtype = torch.float16
    assert emb(ids).dtype == torch.float16


def test_int8_embedding_adopts_a_comfy_table():
    """adopt_int8_embedding swaps a meta nn.Embedding for Int8Embedding and renames the scale
    entry so a strict load follows (reference tests/test_moss_image.py:296-309)."""
    import json
    torch.manual_seed(0)
    table = torch.randn(40, 256) * 0.02
    q, scale = _int8.quantize_weight(table, 256)
    tag = torch.tensor(list(json.dumps({"format": "int8_tensorwise", "convrot": True,
                                        "convrot_groupsize": 256}).encode()), dtype=torch.uint8)
    holder = torch.nn.Module()
    holder.embed_tokens = torch.nn.Embedding(40, 256, device="meta")
    sd = {"embed_tokens.weight": q, "embed_tokens.weight_scale": scale.unsqueeze(1), "embed_tokens.comfy_quant": tag}
    group = _int8.int8_layers(sd).pop("embed_tokens")
    assert group == 256
    sd = _int8.adopt_int8_embedding(holder, sd, "embed_tokens", group)
    holder.load_state_dict(sd, strict=True, assign=True)
    ids = torch.tensor([[5, 39, 0]])
    assert isinstance(holder.embed_tokens, _int8.Int8Embedding)
    torch.testing.assert_close(holder.embed_tokens(ids), _int8.dequantize_weight(q, scale, 256)[ids],
                               rtol=1e-5, atol=1e-8)


def test_scaled_mm_declines_off_the_gpu():
    """The reference's scaled_mm returns None when its fused GEMM can't take the call (here: CPU
    tensors, fp32 output); the int32 path it falls back to then refuses CPU tensors loudly."""
    q = torch.zeros(32, 64, dtype=torch.int8)
    w = torch.zeros(16, 64, dtype=torch.int8)
    sx, sw = torch.ones(32), torch.ones(16)
    assert _int8.scaled_mm(q, w, sx, sw, torch.float16) is None
    assert _int8.scaled_mm(q, w, sx, sw, torch.float32) is None
    with pytest.raises((RuntimeError, ValueError, TypeError)):
        _int8.int_mm(q, w)
