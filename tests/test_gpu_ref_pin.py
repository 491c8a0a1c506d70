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


# ─── the reference's own Triton quantizer (its GPU path), staged from its source ─────────────

@pytest.fixture(scope="module")
def ref_int8():
    if not build_ref.int8_available():
        pytest.skip("reference _int8.py not staged in oracle/_ref")
    pytest.importorskip("triton")
    return build_ref.load_int8()


@pytest.fixture
def triton_division():
    from diffucore_b200 import _int8
    _int8.set_quant_division("triton")
    yield
    _int8.set_quant_division("ieee")


@pytest.mark.parametrize("M,K,group,dtype", [
    (4096, 3072, 0, torch.bfloat16), (4608, 3072, 256, torch.bfloat16), (4608, 15360, 256, torch.bfloat16),
    (4096, 12288, 256, torch.bfloat16), (512, 3072, 256, torch.float16), (300, 640, 0, torch.float16),
    (7, 256, 256, torch.bfloat16), (33, 1000, 0, torch.bfloat16),
    # one width of each block-size class of the Triton kernel (its butterfly order depends on it)
    (16384, 256, 256, torch.bfloat16), (16384, 512, 256, torch.bfloat16), (16384, 768, 256, torch.bfloat16),
    (8192, 1024, 256, torch.float16), (8192, 1280, 256, torch.bfloat16), (4096, 2048, 256, torch.bfloat16),
    (2048, 5120, 256, torch.bfloat16), (1024, 16384, 256, torch.bfloat16)])
def test_triton_division_equals_reference_triton_quantizer(ref_int8, triton_division, M, K, group, dtype):
    """With the "triton" division the native quantizer gives the reference's Triton
    `_rot_quant_kernel` (src/diffucore/models/_int8.py:399-406) codes and scales bit for bit, with and
    without the 256-wide ConvRot rotation, at the golden shapes, FLUX's row widths and one width of
    every block-size class of the Triton kernel."""
    from diffucore_b200 import _int8
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = (torch.randn(M, K, generator=g, device="cuda") * 2).to(dtype)
    rq, rs = ref_int8.quantize_activation(x, group)
    q, s = _int8.quantize_activation(x, group)
    assert torch.equal(q, rq)
    assert torch.equal(s, rs)


def test_default_division_equals_reference_torch_ops_on_cpu(ref_int8):
    """The default division is the reference's torch-op arithmetic (its CPU path, which the golden
    vectors pin): config 1's activation codes equal the reference's own CPU quantize_activation."""
    from diffucore_b200 import _int8
    assert _int8.quant_division() == "ieee"
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16)
    rq, rs = ref_int8.quantize_activation(x, 0)          # on the CPU: the torch ops
    q, s = _int8.quantize_activation(x.cuda(), 0)
    assert torch.equal(q.cpu(), rq) and torch.equal(s.cpu(), rs)


def test_reference_linear_on_gpu_equals_ours_with_triton_division(ref_int8, triton_division):
    """The reference's whole W8A8 linear on this GPU (Triton quantizer -> torch._int_mm -> Triton
    rescale, _int8.py:158-168, :299-323) and this package's Int8Linear holding the same int8 weights
    (the reference's own `from_linear` buffers, adopted as a checkpoint would be) give the same bf16
    output bit for bit once the quantizer divides as the reference's Triton kernel does (config 1's
    shapes, group 0 and 256)."""
    from diffucore_b200 import _int8
    for group in (0, 256):
        g = torch.Generator().manual_seed(group)
        lin = torch.nn.Linear(3072, 3072, bias=True).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_((torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16))
            lin.bias.copy_((torch.randn(3072, generator=g) * 0.01).to(torch.bfloat16))
        lin = lin.cuda()
        ref_layer = ref_int8.Int8Linear.from_linear(lin, group=group)
        ours = _int8.Int8Linear(3072, 3072, bias=True, group=group, device="cuda")
        ours.load_state_dict(ref_layer.state_dict())
        x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16).cuda()
        with torch.no_grad():
            assert torch.equal(ours(x), ref_layer(x))
