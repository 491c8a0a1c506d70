"""GPU parity of the INT8 attention through the C-ABI.

* The int8 codes, the per-row / per-block scales and (mode "ref") the K column sums are
  bit-exact with the CPU oracle, which restates the reference's prep kernels
  (src/diffucore/kernels/int8_attn_sm80.cu:38-142, :341-388).
* The output is within max-abs 2e-2 and cosine >= 0.999 of the oracle's exact-softmax attention
  over the same codes, and within the reference test's budget of exact fp32 attention
  (rel < 3e-2, cosine > 0.9995; tests/test_attention_dispatch.py:198-238).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from diffucore_b200 import _attention, _lib, kernels
from tests.conftest import DTAG, torch_to_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
MODES = {"ref": _lib.MODE_REF, "block64": _lib.MODE_BLOCK64}


@pytest.fixture(params=["two_tile", "single_tile"])
def kernel(request, monkeypatch):
    """Pins the main kernel the library would otherwise pick by grid size (DC_ATTN_KERNEL)."""
    monkeypatch.setenv("DC_ATTN_KERNEL", request.param)
    return request.param


def _inputs(B, Lq, Lk, H, D, dtype, seed=0, k_shift=0.5):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Lq, H, D, generator=g).to(dtype)
    k = (torch.randn(B, Lk, H, D, generator=g) + k_shift).to(dtype)
    v = torch.randn(B, Lk, H, D, generator=g).to(dtype)
    return q, k, v


def _bits(t):
    return torch_to_bits(t)


def _cos(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return float((a @ b) / (a.norm() * b.norm()))


@pytest.mark.parametrize("mode", ["ref", "block64"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Lq,Lk,H,D", [(1, 300, 77, 2, 128), (2, 130, 1000, 3, 128), (1, 257, 333, 2, 64),
                                         (1, 64, 4608, 1, 128)])
def test_prep_codes_bit_exact(mode, dtype, B, Lq, Lk, H, D):
    q, k, _ = _inputs(B, Lq, Lk, H, D, dtype)
    got = kernels.attn_int8_prep(q.to(DEV), k.to(DEV), MODES[mode])
    ref = oracle.attn_prep(_bits(q), _bits(k), DTAG[dtype], mode)
    for key in ("q_codes", "k_codes", "q_scale", "k_scale") + (("ksum",) if mode == "ref" else ()):
        a, b = got[key].cpu().numpy(), ref[key]
        assert a.shape == b.shape, key
        assert np.array_equal(a, b), f"{key}: {np.count_nonzero(a != b)} of {a.size} differ"


def _check_against_oracle(q, k, v, out, dtype, mode, sm_scale):
    ref = torch.from_numpy(oracle.attn_int8(_bits(q), _bits(k), _bits(v), DTAG[dtype], sm_scale, mode))
    o = out.float().cpu().reshape(ref.shape)
    assert torch.isfinite(o).all()
    assert (o - ref).abs().max() < 2e-2
    assert _cos(o, ref) >= 0.999


@pytest.mark.parametrize("mode", ["ref", "block64"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 1024, 1024, 4), (2, 1000, 1000, 2), (1, 700, 77, 4), (1, 70, 3953, 2)])
def test_attention_matches_oracle_and_sdpa(mode, dtype, B, Lq, Lk, H, kernel):
    """The reference test's shapes (unaligned lengths exercise query/key tails), K shifted +0.5."""
    q, k, v = _inputs(B, Lq, Lk, H, 128, dtype)
    out = _attention.attention_blhd(q.to(DEV), k.to(DEV), v.to(DEV), "int8_turing", quant_mode=mode)
    assert out.shape == (B, Lq, H * 128) and out.dtype == dtype
    _check_against_oracle(q, k, v, out, dtype, mode, 128 ** -0.5)
    ref = F.scaled_dot_product_attention(*(t.to(DEV).float().transpose(1, 2) for t in (q, k, v)))
    ref = ref.transpose(1, 2).reshape(B, Lq, -1)
    rel = float((out.float() - ref).norm() / ref.norm())
    assert rel < 3e-2
    assert _cos(out.float(), ref) > 0.9995


@pytest.mark.parametrize("mode", ["ref", "block64"])
@pytest.mark.parametrize("B,Lq,Lk,H", [(2, 4096, 4096, 2), (1, 1024, 77, 5), (1, 333, 1500, 3)])
def test_attention_head_dim_64(mode, B, Lq, Lk, H, kernel):
    """D = 64 (SDXL self-attention); the reference falls back to SDPA there."""
    q, k, v = _inputs(B, Lq, Lk, H, 64, torch.float16, seed=1, k_shift=0.0)
    out = _attention.attention_blhd(q.to(DEV), k.to(DEV), v.to(DEV), "int8_turing", quant_mode=mode)
    _check_against_oracle(q, k, v, out, torch.float16, mode, 64 ** -0.5)


def test_bhld_and_packed_strided_inputs(kernel):
    """(B, H, L, D) transposed views and a packed qkv projection (stride(2) = 3 * 128)
    (reference tests/test_attention_dispatch.py:216-226)."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 3, 600, 128, generator=g).half().to(DEV) for _ in range(3))
    out = _attention.attention_bhld(q, k, v, "int8_turing")
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float()).transpose(1, 2).reshape(1, 600, -1)
    assert float((out.float() - ref).norm() / ref.norm()) < 3e-2
    qkv = torch.randn(1, 500, 2, 3 * 128, generator=g).half().to(DEV)
    q, k, v = qkv[..., :128], qkv[..., 128:256], qkv[..., 256:]
    out = _attention.attention_blhd(q, k, v, "int8_turing")
    _check_against_oracle(q.cpu(), k.cpu(), v.cpu(), out, torch.float16, "ref", 128 ** -0.5)


def test_flat_scores_large_v_stay_finite(kernel):
    """Flat scores with large same-sign V (reference tests/test_attention_dispatch.py:229-238):
    fp32 P.V accumulation keeps every output finite and close."""
    g = torch.Generator().manual_seed(0)
    q = torch.zeros(1, 256, 2, 128).half().to(DEV)
    k = torch.randn(1, 1024, 2, 128, generator=g).half().to(DEV)
    v = (torch.rand(1, 1024, 2, 128, generator=g) * 200 + 900).half().to(DEV)
    out = _attention.attention_blhd(q, k, v, "int8_turing")
    assert torch.isfinite(out).all()
    ref = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                         v.float().transpose(1, 2)).transpose(1, 2).reshape(1, 256, -1)
    assert float((out.float() - ref).norm() / ref.norm()) < 1e-3


def test_ineligible_inputs_run_sdpa_exactly():
    """Head dims other than 64/128 and fp32 inputs take the reference's exact SDPA branch."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 256, 2, 96, generator=g).half().to(DEV)
    assert torch.equal(_attention.attention_blhd(q, q, q, "int8_turing"), _attention.attention_blhd(q, q, q, "sdpa"))
    q = torch.randn(1, 256, 2, 128, generator=g).to(DEV)
    assert torch.equal(_attention.attention_blhd(q, q, q, "int8_turing"), _attention.attention_blhd(q, q, q, "sdpa"))


def test_null_keys_equal_padded(kernel):
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 300, 4, 128, generator=g).half().to(DEV)
    k = torch.randn(1, 67, 4, 128, generator=g).half().to(DEV)
    v = torch.randn(1, 67, 4, 128, generator=g).half().to(DEV)
    kp, vp = F.pad(k, (0, 0, 0, 0, 0, 445)), F.pad(v, (0, 0, 0, 0, 0, 445))
    a = _attention.attention_blhd(q, k, v, "int8_turing", null_keys=445)
    b = _attention.attention_blhd(q, kp, vp, "int8_turing")
    assert torch.equal(a, b)


@pytest.mark.parametrize("mode", ["block64", "ref"])
def test_config2_full_size_properties(mode, kernel):
    """BASELINE config 2 at full size (B=1, H=24, S=4608, D=128, bf16, N(0,1)): finite, close to
    fp32 attention on the GPU, deterministic run to run, and its codes equal the oracle's."""
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 24, 4608, 128, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    out1 = _attention.attention_bhld(q, k, v, "int8_turing", quant_mode=mode)
    out2 = _attention.attention_bhld(q, k, v, "int8_turing", quant_mode=mode)
    assert torch.equal(out1, out2)
    assert torch.isfinite(out1).all()
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float()).transpose(1, 2).reshape(1, 4608, -1)
    assert _cos(out1.float(), ref) >= 0.999
    assert (out1.float() - ref).abs().max() < 5e-2
    qt, kt = q.transpose(1, 2), k.transpose(1, 2)
    got = kernels.attn_int8_prep(qt, kt, MODES[mode])
    want = oracle.attn_prep(_bits(qt.cpu()), _bits(kt.cpu()), "bf16", mode)
    assert np.array_equal(got["k_codes"].cpu().numpy(), want["k_codes"])
    assert np.array_equal(got["q_codes"].cpu().numpy(), want["q_codes"])


@pytest.mark.parametrize("mode", ["ref", "block64"])
def test_running_max_moves_every_tile(mode, kernel):
    """Scores that grow along the keys (K rows scaled up tile after tile) move every row's running
    max by far more than the lazy-rescale headroom at each 128-key tile, for some rows of a warp
    and not others: the O rescale path runs, warp-uniformly, and the result still matches the
    oracle's exact softmax."""
    g = torch.Generator().manual_seed(9)
    B, L, H, D = 1, 1024, 2, 128
    q = torch.randn(B, L, H, D, generator=g)
    q[:, ::2] *= 0.05                                          # half the rows barely move
    ramp = torch.linspace(0.2, 24.0, L).view(1, L, 1, 1)   # +9 (log2) per 128 keys for 2-sigma rows
    base = torch.randn(1, 1, H, D, generator=g)
    k = (base + 0.3 * torch.randn(B, L, H, D, generator=g)) * ramp
    v = torch.randn(B, L, H, D, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    out = _attention.attention_blhd(q.to(DEV), k.to(DEV), v.to(DEV), "int8_turing", quant_mode=mode)
    _check_against_oracle(q, k, v, out, torch.bfloat16, mode, D ** -0.5)


def test_fma_pipe_exp2_accuracy():
    """The polynomial exp2 the softmax runs on the FMA pipe for a third of the keys stays within
    1e-4 relative of CUDA's exp2f over the range P takes (arguments <= 8), and is 0 / tiny far below."""
    x = torch.cat([torch.linspace(-40.0, 8.0, 1 << 20), torch.tensor([-126.9, -127.0, -200.0, -1e30])]).cuda()
    poly, ref = kernels.selftest_exp2(x)
    rel = ((poly - ref).abs() / ref.clamp_min(1e-38))[: 1 << 20]
    assert float(rel.max()) < 1e-4
    assert torch.isfinite(poly).all() and float(poly[-1]) < 1e-37
