"""GPU parity of the W8A8 path through the C-ABI: the sm_100a quantizer, the tcgen05 GEMM (raw
int32 and the fused rescale/bias epilogue) and the Int8Linear module, against the CPU oracle and
the reference's golden vectors. Integer results and int8 codes are bit-exact; bf16/fp16 outputs
of the group-0 path are bit-exact too (the epilogue rounds exactly like the reference)."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch
import torch.nn as nn

import oracle
from diffucore_b200 import _int8, _lib, kernels
from tests.conftest import GOLDEN, bits_to_torch, torch_to_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sha(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


# ─── quantizer ──────────────────────────────────────────────────────────────────────────

@pytest.mark.parametrize("name,dtype", [("qa_bf16_g0", torch.bfloat16), ("qa_f16_g0", torch.float16)])
def test_quant_rows_matches_reference_golden(golden, name, dtype):
    x = bits_to_torch(golden[f"{name}_x"], dtype).to(DEV)
    q, s = _int8.quantize_activation(x, 0)
    assert np.array_equal(q.cpu().numpy(), golden[f"{name}_q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), golden[f"{name}_s"].view(np.uint32))


@pytest.mark.parametrize("name,dtype,tag", [("qa_bf16_g256", torch.bfloat16, "bf16"),
                                            ("qa_f16_g256", torch.float16, "f16")])
def test_quant_rows_group256_bit_exact_with_butterfly_oracle(golden, name, dtype, tag):
    x = bits_to_torch(golden[f"{name}_x"], dtype).to(DEV)
    q, s = _int8.quantize_activation(x, 256)
    oq, os_ = oracle.quant_rows(golden[f"{name}_x"], tag, 256)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy(), os_)


@pytest.mark.parametrize("M,K,group,dtype", [
    (1, 16, 0, torch.bfloat16), (3, 3072, 0, torch.bfloat16), (257, 15360, 0, torch.bfloat16),
    (100, 12288, 256, torch.bfloat16), (64, 4096, 256, torch.float16), (7, 77, 0, torch.float16),
    (33, 1000, 0, torch.bfloat16), (5, 16384, 256, torch.bfloat16)])
def test_quant_rows_shapes(M, K, group, dtype):
    g = torch.Generator().manual_seed(M * 7 + K)
    x = (torch.randn(M, K, generator=g) * 2).to(dtype)
    q, s = kernels.quant_rows(x.to(DEV), group)
    oq, os_ = oracle.quant_rows(torch_to_bits(x), "bf16" if dtype == torch.bfloat16 else "f16", group)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy(), os_)


def test_quant_rows_strided_and_fp32():
    g = torch.Generator().manual_seed(3)
    base = torch.randn(40, 1024, generator=g).to(torch.bfloat16).to(DEV)
    view = base[:, :512]                                    # row stride 1024, K 512
    q, s = kernels.quant_rows(view, 0)
    oq, os_ = oracle.quant_rows(torch_to_bits(view.contiguous()), "bf16", 0)
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)
    w = torch.randn(96, 768, generator=g) * 0.02            # fp32 weights (load-time path)
    q, s = kernels.quant_rows(w.to(DEV), 256)
    oq, os_ = oracle.quant_rows(w.numpy(), "f32", 256)
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)


@pytest.mark.parametrize("group", [0, 256])
@pytest.mark.parametrize("K", [256, 768, 4352, 12288, 15360, 16384])
def test_quant_rows_streaming_kernels_bit_exact(group, K):
    """Rows streamed through shared memory (warp per row up to K = 4096, CTA per row above), the
    ConvRot butterfly as register stages around a shared-memory transpose: codes and scales equal
    the oracle's, including an odd number of 256-groups (a half-warp idles) and rows spanning
    several CTA iterations."""
    g = torch.Generator().manual_seed(K + group)
    x = (torch.randn(37, K, generator=g) * torch.rand(37, 1, generator=g) * 4).to(torch.bfloat16)
    x[5] = 0                                                  # a zero row: scale 1e-30, codes 0
    q, s = kernels.quant_rows(x.to(DEV), group)
    oq, os_ = oracle.quant_rows(torch_to_bits(x), "bf16", group)
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(s.cpu().numpy(), os_)


def test_quant_rows_gelu_modes():
    g = torch.Generator().manual_seed(4)
    h = (torch.randn(64, 1024, generator=g) * 3).to(torch.bfloat16)
    for mode in (_lib.GELU_ERF, _lib.GELU_TANH):
        q, s = kernels.quant_rows(h.to(DEV), 0, mode)
        oq, os_ = oracle.quant_rows(torch_to_bits(h), "bf16", 0, mode)
        # erff/tanhf differ from libm by ulps; after bf16 rounding nearly all codes agree
        assert np.abs(q.cpu().numpy().astype(int) - oq.astype(int)).max() <= 1
        assert (q.cpu().numpy() != oq).mean() < 2e-3
        np.testing.assert_allclose(s.cpu().numpy(), os_, rtol=1e-2)


# ─── GEMM ───────────────────────────────────────────────────────────────────────────────

@pytest.mark.parametrize("m,n,k", [(33, 2048, 1024), (300, 512, 768), (4096, 2048, 2048), (1000, 8192, 2048),
                                   (1, 64, 16), (3, 96, 256), (17, 200, 48), (129, 257, 4096)])
def test_int_mm_bit_exact(m, n, k):
    """The reference test's bit-exact GEMM shapes (tests/test_int8.py:175) plus tails; checked
    against torch._int_mm (exact int32, independent of rounding) and, when small, the oracle."""
    g = torch.Generator().manual_seed(6)
    q = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    acc = _int8.int_mm(q.to(DEV), w.to(DEV)).cpu()
    if m * n * k <= 2 ** 27:
        assert np.array_equal(acc.numpy(), oracle.int_mm(q.numpy(), w.numpy()))
    if m > 16 and k % 8 == 0 and n % 8 == 0:
        assert torch.equal(acc, torch._int_mm(q.to(DEV), w.to(DEV).t()).cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(33, 2048, 1024), (300, 512, 768), (1000, 8192, 2048), (5, 136, 64)])
def test_fused_epilogue_bit_exact_with_rescale(dtype, m, n, k):
    """scaled_mm (fused) == rescale(int_mm) rounding for rounding (reference tests/test_int8.py:174-183),
    with and without bias."""
    g = torch.Generator().manual_seed(6)
    q = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).to(DEV)
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).to(DEV)
    sx, sw = (torch.rand(m, generator=g) * 1e-2).to(DEV), (torch.rand(n, generator=g) * 1e-3).to(DEV)
    bias = (torch.randn(n, generator=g) * 0.1).to(dtype).to(DEV)
    acc = _int8.int_mm(q, w)
    tag = "bf16" if dtype == torch.bfloat16 else "f16"
    for b in (None, bias):
        fused = kernels.gemm_w8a8(q, w, sx, sw, b, dtype)
        assert torch.equal(fused, _int8.rescale(acc, sx, sw, b, dtype))
        ref = oracle.rescale(acc.cpu().numpy(), sx.cpu().numpy(), sw.cpu().numpy(),
                             None if b is None else torch_to_bits(b), tag)
        assert np.array_equal(torch_to_bits(fused), ref)
    assert torch.equal(_int8.scaled_mm(q, w, sx, sw, dtype), kernels.gemm_w8a8(q, w, sx, sw, None, dtype))


@pytest.mark.parametrize("tag,dtype,group", [("lin_g0_bf16", torch.bfloat16, 0), ("lin_g0_f16", torch.float16, 0)])
def test_int8_linear_matches_reference_golden(golden, tag, dtype, group):
    lin = nn.Linear(512, 192, bias=True).to(dtype)
    with torch.no_grad():
        lin.weight.copy_(bits_to_torch(golden[f"{tag}_w"], dtype))
        lin.bias.copy_(bits_to_torch(golden[f"{tag}_b"], dtype))
    layer = _int8.Int8Linear.from_linear(lin.to(DEV), group)
    assert np.array_equal(layer.weight.cpu().numpy(), golden[f"{tag}_wq"])
    assert np.array_equal(layer.scale.cpu().numpy(), golden[f"{tag}_ws"])
    x = bits_to_torch(golden[f"{tag}_x"], dtype).to(DEV)
    y = layer(x)
    assert y.shape == (2, 40, 192) and y.dtype == dtype
    assert np.array_equal(torch_to_bits(y), golden[f"{tag}_y"])


def test_int8_linear_group256_matches_oracle_and_reference(golden):
    tag = "lin_g256_bf16"
    layer = _int8.Int8Linear(512, 192, bias=True, group=256, device=DEV)
    layer.weight.copy_(torch.from_numpy(golden[f"{tag}_wq"]))
    layer.scale_bits.copy_(torch.from_numpy(golden[f"{tag}_ws"].view(np.int32)))
    layer.bias = nn.Parameter(bits_to_torch(golden[f"{tag}_b"], torch.bfloat16).to(DEV), requires_grad=False)
    x = bits_to_torch(golden[f"{tag}_x"], torch.bfloat16).to(DEV)
    y = layer(x)
    ref_oracle = oracle.linear(golden[f"{tag}_x"].reshape(-1, 512), "bf16", golden[f"{tag}_wq"],
                               golden[f"{tag}_ws"], golden[f"{tag}_b"], 256)
    assert np.array_equal(torch_to_bits(y).reshape(ref_oracle.shape), ref_oracle)
    ref = bits_to_torch(golden[f"{tag}_y"], torch.bfloat16).float()
    assert (y.cpu().float() - ref).abs().max() < 2e-2
    assert torch.nn.functional.cosine_similarity(y.cpu().float().flatten(), ref.flatten(), dim=0) > 0.999


def test_int8_mlp_close_to_reference(golden):
    l1 = _int8.Int8Linear(256, 512, bias=False, group=0, device=DEV)
    l2 = _int8.Int8Linear(512, 256, bias=False, group=0, device=DEV)
    for layer, p in ((l1, "mlp_l1"), (l2, "mlp_l2")):
        layer.weight.copy_(torch.from_numpy(golden[f"{p}q"]))
        layer.scale_bits.copy_(torch.from_numpy(golden[f"{p}s"].view(np.int32)))
    x = bits_to_torch(golden["mlp_x"], torch.bfloat16).to(DEV)
    y = _int8.int8_mlp(x, l1, l2).cpu().float()
    ref = bits_to_torch(golden["mlp_y"], torch.bfloat16).float()
    assert (y - ref).abs().max() < 2e-2
    assert torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0) > 0.999


def test_config1_full_size_bit_exact_with_reference():
    """BASELINE config 1 (4096 x 3072 x 3072, bf16, bias, group 0): codes, scales, the int32
    accumulator and the bf16 output hash to the reference's (tests/golden/config1_sha256.json)."""
    meta = json.loads((GOLDEN / "config1_sha256.json").read_text())
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16)
    w = (torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(3072, generator=g) * 0.01).to(torch.bfloat16)
    assert _sha(x) == meta["x_sha256"]
    lin = nn.Linear(3072, 3072, bias=True).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(b)
    layer = _int8.Int8Linear.from_linear(lin.to(DEV), 0)
    assert _sha(layer.weight) == meta["wq_sha256"] and _sha(layer.scale) == meta["ws_sha256"]
    xd = x.to(DEV)
    qx, sx = _int8.quantize_activation(xd, 0)
    assert _sha(qx) == meta["qx_sha256"] and _sha(sx) == meta["sx_sha256"]
    assert _sha(_int8.int_mm(qx, layer.weight)) == meta["acc_sha256"]
    assert _sha(layer(xd)) == meta["y_sha256"]



# ─── mirrors of the reference's own module tests (tests/test_int8.py) ───────────────────

def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("k,n", [(2048, 2048), (768, 512), (1024, 8192)])
def test_kernels_match_reference_torch_ops(k, n):
    """tests/test_int8.py:141-153: the CUDA Int8Linear (default ConvRot group 256, fp16) against
    the reference's torch-op path (oracle/torch_ref.py, pinned to the reference's output hashes)
    within 2e-3 relative, and against the float linear within 2e-2."""
    from oracle import torch_ref
    torch.manual_seed(4)
    lin = nn.Linear(k, n, bias=n == 512).half()
    m = _int8.Int8Linear.from_linear(lin.to(DEV))
    x = torch.randn(3, 333, k, dtype=torch.float16)
    y = m(x.to(DEV)).cpu()
    bias = None if m.bias is None else m.bias.detach().cpu()
    y_ref = torch_ref.int8_linear(x, m.weight.cpu(), m.scale.cpu(), bias, m.group)
    assert y.dtype == torch.float16 and _rel(y, y_ref) < 2e-3
    with torch.no_grad():
        y_float = lin.cpu().float()(x.float())
    assert _rel(y, y_float) < 0.02


def test_fused_mlp_matches_reference_unfused():
    """tests/test_int8.py:156-166: int8_mlp against the torch-op l2(gelu(l1(x)))."""
    from oracle import torch_ref
    torch.manual_seed(5)
    l1 = _int8.Int8Linear.from_linear(nn.Linear(1024, 4096, bias=False).half().to(DEV))
    l2 = _int8.Int8Linear.from_linear(nn.Linear(4096, 1024, bias=False).half().to(DEV))
    x = torch.randn(2, 500, 1024, dtype=torch.float16)
    y = _int8.int8_mlp(x.to(DEV), l1, l2).cpu()
    h = torch_ref.int8_linear(x, l1.weight.cpu(), l1.scale.cpu(), None, l1.group)
    y_ref = torch_ref.int8_linear(torch.nn.functional.gelu(h), l2.weight.cpu(), l2.scale.cpu(), None, l2.group)
    assert _rel(y, y_ref) < 2e-3


@pytest.mark.parametrize("M,K,dtype", [(4096, 3072, torch.bfloat16), (300, 640, torch.float16), (5, 4096, torch.bfloat16),
                                       (129, 8, torch.float16), (64, 1000, torch.bfloat16)])
@pytest.mark.parametrize("division", ["ieee", "triton"])
def test_cta_per_row_quantizer_equals_warp_kernel(monkeypatch, M, K, dtype, division):
    """The CTA-per-row quantizer that plain 16-bit rows up to 4096 wide now take gives the warp-per-row
    kernel's codes and scales bit for bit (DC_QUANT_CTA=0 selects the latter), in both divisions."""
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * 3).to(dtype).to(DEV)
    _int8.set_quant_division(division)
    try:
        monkeypatch.setenv("DC_QUANT_CTA", "0")
        qw, sw = kernels.quant_rows(x, 0)
        monkeypatch.delenv("DC_QUANT_CTA")
        qc, sc = kernels.quant_rows(x, 0)
    finally:
        _int8.set_quant_division("ieee")
    assert torch.equal(qw, qc) and torch.equal(sw, sc)
