"""Pins the CPU oracle to the reference: every golden vector in tests/golden/ was produced by the
reference's own code (diffucore 0.2.4, torch-op path); the oracle must reproduce them bit for bit
where the reference's arithmetic is deterministic (group 0, int_mm, rescale), and within the
documented rounding differences where it is not (the ConvRot rotation order, erf ulps)."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

import oracle
from tests.conftest import GOLDEN, bits_to_torch


@pytest.mark.parametrize("name,dtype,group", [("qa_bf16_g0", "bf16", 0), ("qa_f16_g0", "f16", 0)])
def test_quant_rows_bit_exact_group0(golden, name, dtype, group):
    q, s = oracle.quant_rows(golden[f"{name}_x"], dtype, group)
    assert np.array_equal(q, golden[f"{name}_q"])
    assert np.array_equal(s.view(np.uint32), golden[f"{name}_s"].view(np.uint32))
    # the all-zero row clamps its scale to 1e-30 and codes to 0 (reference `_quantize_rows`)
    assert s[1] == np.float32(1e-30) and not q[1].any()


@pytest.mark.parametrize("name,dtype", [("qa_bf16_g256", "bf16"), ("qa_f16_g256", "f16")])
def test_quant_rows_group256_close_to_reference_matmul(golden, name, dtype):
    """The reference's CPU `_rotate` is an fp32 matmul; the kernel (and oracle) use the Triton
    butterfly. Both are x @ H up to fp32 rounding, so codes differ by at most 1 at rounding ties."""
    q, s = oracle.quant_rows(golden[f"{name}_x"], dtype, 256)
    ref_q, ref_s = golden[f"{name}_q"], golden[f"{name}_s"]
    diff = np.abs(q.astype(np.int32) - ref_q.astype(np.int32))
    assert diff.max() <= 1
    assert (diff > 0).mean() < 0.01
    np.testing.assert_allclose(s, ref_s, rtol=1e-5, atol=0)


def test_butterfly_is_the_reference_hadamard(golden):
    sign = golden["hadamard256_sign"].astype(np.float64) / 16.0       # reference _hadamard(256)
    rng = np.random.default_rng(0)
    x = rng.standard_normal(256).astype(np.float32)
    y = oracle.hadamard256(x)
    np.testing.assert_allclose(y, x.astype(np.float64) @ sign, rtol=0, atol=2e-6)
    # H is symmetric and its own inverse (reference test_int8.py:40-43)
    np.testing.assert_allclose(oracle.hadamard256(y), x, rtol=0, atol=5e-6)


@pytest.mark.parametrize("name", ["imm_small", "imm_mid"])
def test_int_mm_exact(golden, name):
    assert np.array_equal(oracle.int_mm(golden[f"{name}_q"], golden[f"{name}_w"]), golden[f"{name}_acc"])


@pytest.mark.parametrize("tag", ["bf16", "f16"])
def test_rescale_bit_exact(golden, tag):
    acc, sx, sw = golden[f"rs_{tag}_acc"], golden[f"rs_{tag}_sx"], golden[f"rs_{tag}_sw"]
    assert np.array_equal(oracle.rescale(acc, sx, sw, None, tag), golden[f"rs_{tag}_y"])
    assert np.array_equal(oracle.rescale(acc, sx, sw, golden[f"rs_{tag}_bias"], tag), golden[f"rs_{tag}_yb"])


@pytest.mark.parametrize("tag,dtype", [("lin_g0_bf16", "bf16"), ("lin_g0_f16", "f16")])
def test_linear_forward_bit_exact(golden, tag, dtype):
    w = golden[f"{tag}_w"]
    wq, ws = oracle.quant_rows(w if dtype != "f32" else w, dtype, 0)
    assert np.array_equal(wq, golden[f"{tag}_wq"]) and np.array_equal(ws, golden[f"{tag}_ws"])
    x = golden[f"{tag}_x"].reshape(-1, w.shape[1])
    y = oracle.linear(x, dtype, wq, ws, golden[f"{tag}_b"], 0)
    assert np.array_equal(y.reshape(golden[f"{tag}_y"].shape), golden[f"{tag}_y"])


def test_linear_group256_close(golden):
    tag = "lin_g256_bf16"
    x = golden[f"{tag}_x"].reshape(-1, 512)
    y = oracle.linear(x, "bf16", golden[f"{tag}_wq"], golden[f"{tag}_ws"], golden[f"{tag}_b"], 256)
    yf = oracle.to_float(y, "bf16")
    ref = oracle.to_float(golden[f"{tag}_y"], "bf16").reshape(yf.shape)
    assert np.abs(yf - ref).max() < 2e-2
    cos = float((yf * ref).sum() / np.linalg.norm(yf) / np.linalg.norm(ref))
    assert cos > 0.9999


def test_int8_mlp_close(golden):
    """l2(gelu(l1(x))): GELU uses libm erff here and torch's erf in the reference; after rounding
    to bf16 they agree on nearly every element, and the int8 pipeline stays within tolerance."""
    x = golden["mlp_x"].reshape(-1, 256)
    q, s = oracle.quant_rows(x, "bf16", 0)
    h = oracle.rescale(oracle.int_mm(q, golden["mlp_l1q"]), s, golden["mlp_l1s"], None, "bf16", gelu=1)
    assert (h != golden["mlp_h"].reshape(h.shape)).mean() < 0.01
    q2, s2 = oracle.quant_rows(h, "bf16", 0)
    y = oracle.rescale(oracle.int_mm(q2, golden["mlp_l2q"]), s2, golden["mlp_l2s"], None, "bf16")
    yf, ref = oracle.to_float(y, "bf16"), oracle.to_float(golden["mlp_y"], "bf16").reshape(-1, 256)
    assert np.abs(yf - ref).max() < 2e-2


def test_config1_codes_match_reference_hashes():
    """Full-size BASELINE config 1: the oracle's activation and weight codes/scales hash to the
    reference's (tests/golden/config1_sha256.json)."""
    meta = json.loads((GOLDEN / "config1_sha256.json").read_text())
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16)
    w = (torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    assert h(xb) == meta["x_sha256"]
    qx, sx = oracle.quant_rows(xb, "bf16", 0)
    assert h(qx) == meta["qx_sha256"] and h(sx) == meta["sx_sha256"]
    wq, ws = oracle.quant_rows(wb, "bf16", 0)
    assert h(wq) == meta["wq_sha256"] and h(ws) == meta["ws_sha256"]


def test_bits_roundtrip_matches_torch():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(4096) * np.exp(rng.uniform(-20, 12, 4096))).astype(np.float32)
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        ref = torch.from_numpy(x).to(dt).view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(oracle.to_bits(x, tag), ref)
        assert np.array_equal(oracle.to_float(ref, tag), bits_to_torch(ref, dt).float().numpy())


def test_torch_restatement_reproduces_config1_output_hashes():
    """The torch-op restatement of the reference's CPU path (oracle/torch_ref.py), the timed CPU
    baseline of config 1, gives the reference's own int32 accumulator and bf16 output bit for bit
    at full size (tests/golden/config1_sha256.json)."""
    from oracle import torch_ref
    meta = json.loads((GOLDEN / "config1_sha256.json").read_text())
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16)
    w = (torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(3072, generator=g) * 0.01).to(torch.bfloat16)
    h = lambda t: hashlib.sha256(np.ascontiguousarray(t.numpy()).tobytes()).hexdigest()  # noqa: E731
    wq, ws = torch_ref.quantize_weight(w, 0)
    assert h(wq) == meta["wq_sha256"] and h(ws) == meta["ws_sha256"]
    q, sx = torch_ref.quantize_rows(x)
    assert h(q) == meta["qx_sha256"] and h(sx) == meta["sx_sha256"]
    assert h(torch_ref.int_mm(q, wq)) == meta["acc_sha256"]
    y = torch_ref.int8_linear(x, wq, ws, b, 0)
    assert h(y.view(torch.int16)) == meta["y_sha256"]


def test_torch_restatement_rotation_matches_butterfly_within_ties(golden):
    """group 256: the fp32-matmul rotation of the restatement against the oracle's butterfly
    (same codes except at rounding ties, as for the reference's own _rotate)."""
    from oracle import torch_ref
    xb = golden["qa_bf16_g256_x"]
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    q, s = torch_ref.quantize_rows(torch_ref.rotate(x.float(), 256))
    qo, so = oracle.quant_rows(xb, "bf16", 256)
    assert (q.numpy() != qo).mean() < 2e-3
    np.testing.assert_allclose(s.numpy(), so, rtol=1e-5)
