"""CPU parts of the Int8Linear module API (load-time helpers), mirroring the reference's own
tests/test_int8.py:40-50: the ConvRot Hadamard is symmetric and its own inverse, and a weight
survives quantize -> dequantize within 1 % relative error with and without rotation. The
module's load-time helpers agree with the reference's torch-op path (oracle/torch_ref.py)."""

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
