"""The CPU oracle's INT8 attention (oracle/dc_oracle.c restating src/diffucore/kernels/
int8_attn_sm80.cu) against the known answers the reference's own tests hold for that kernel
(tests/test_attention_dispatch.py:198-238): on its four shapes (unaligned lengths exercise the
query / key tails, K shifted by +0.5 exercises the mean subtraction) the int8 result stays within
rel 3e-2 and cosine 0.9995 of exact attention, packed q/k/v views give the same result, and flat
scores over large same-sign V stay within rel 1e-3. Also the prep invariants of both quant modes
(symmetric abs-max codes per token / per 64-row block, K's column mean subtracted in mode "ref")
and the exact path against torch's SDPA. The GPU tests compare the CUDA kernels with this oracle,
and tests/test_gpu_ref_pin.py pins its prep to the reference's own kernels bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle


def _inputs(B, Lq, Lk, H, D, dtype, seed=0, k_shift=0.5):
    g = np.random.default_rng(seed)
    q = g.standard_normal((B, Lq, H, D), dtype=np.float32)
    k = g.standard_normal((B, Lk, H, D), dtype=np.float32) + k_shift
    v = g.standard_normal((B, Lk, H, D), dtype=np.float32)
    return tuple(oracle.to_bits(t, dtype) for t in (q, k, v))


def _rel(a, b):
    return float(np.linalg.norm((a - b).ravel()) / np.linalg.norm(b.ravel()))


def _cos(a, b):
    a, b = a.ravel().astype(np.float64), b.ravel().astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.mark.parametrize("mode", ["ref", "block64"])
@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 1024, 1024, 4), (2, 1000, 1000, 2), (1, 700, 77, 4), (1, 70, 3953, 2)])
def test_int8_close_to_exact(B, Lq, Lk, H, mode):
    D = 128
    q, k, v = _inputs(B, Lq, Lk, H, D, "f16")
    got = oracle.attn_int8(q, k, v, "f16", D ** -0.5, mode)
    want = oracle.attn_exact(q, k, v, "f16", D ** -0.5)
    assert np.isfinite(got).all()
    assert _rel(got, want) < 3e-2 and _cos(got, want) > 0.9995, (_rel(got, want), _cos(got, want))


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("D", [64, 128])
def test_int8_close_to_exact_dtypes_and_head_dims(dtype, D):
    q, k, v = _inputs(1, 300, 333, 3, D, dtype, seed=D)
    for mode in ("ref", "block64"):
        got = oracle.attn_int8(q, k, v, dtype, D ** -0.5, mode)
        want = oracle.attn_exact(q, k, v, dtype, D ** -0.5)
        assert _rel(got, want) < 3e-2 and _cos(got, want) > 0.9995


def test_packed_views_equal_contiguous():
    g = np.random.default_rng(5)
    qkv = oracle.to_bits(g.standard_normal((1, 500, 2, 3 * 128), dtype=np.float32), "f16")
    q, k, v = qkv[..., :128], qkv[..., 128:256], qkv[..., 256:]
    for mode in ("ref", "block64"):
        a = oracle.attn_int8(q, k, v, "f16", 128 ** -0.5, mode)
        b = oracle.attn_int8(*(np.ascontiguousarray(t) for t in (q, k, v)), "f16", 128 ** -0.5, mode)
        assert np.array_equal(a, b)


def test_flat_scores_over_large_values():
    g = np.random.default_rng(7)
    q = oracle.to_bits(np.zeros((1, 256, 2, 128), np.float32), "f16")
    k = oracle.to_bits(g.standard_normal((1, 1024, 2, 128), dtype=np.float32), "f16")
    v = oracle.to_bits(g.random((1, 1024, 2, 128), dtype=np.float32) * 200 + 900, "f16")
    for mode in ("ref", "block64"):
        got = oracle.attn_int8(q, k, v, "f16", 128 ** -0.5, mode)
        want = oracle.attn_exact(q, k, v, "f16", 128 ** -0.5)
        assert np.isfinite(got).all() and _rel(got, want) < 1e-3


def test_exact_path_matches_torch_sdpa():
    q, k, v = _inputs(1, 200, 150, 2, 128, "bf16", seed=3)
    got = oracle.attn_exact(q, k, v, "bf16", 128 ** -0.5)
    tq, tk, tv = (torch.from_numpy(oracle.to_float(t, "bf16")).transpose(1, 2).double() for t in (q, k, v))
    want = F.scaled_dot_product_attention(tq, tk, tv).transpose(1, 2).float().numpy()
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6)


def _check_block_codes(x, codes, scale, block):
    """codes = rint(x / scale) with scale = amax / 127 per `block` rows of a head (the last block
    may be short); every non-zero block reaches +-127."""
    B, H, L, D = codes.shape
    for s in range(0, L, block):
        xs, cs, sc = x[:, :, s:s + block], codes[:, :, s:s + block].astype(np.int32), scale[:, :, s // block]
        amax = np.abs(xs).reshape(B, H, -1).max(axis=-1)
        np.testing.assert_allclose(sc, amax / 127, rtol=1e-6)
        assert np.abs(cs).max() <= 127
        assert (np.abs(cs).reshape(B, H, -1).max(axis=-1)[amax > 0] == 127).all()
        assert np.abs(cs - xs / sc[..., None, None]).max() <= 0.5 + 1e-3


@pytest.mark.parametrize("mode", ["ref", "block64"])
def test_prep_codes_are_symmetric_absmax(mode):
    B, Lq, Lk, H, D = 2, 150, 200, 3, 128
    q, k, _ = _inputs(B, Lq, Lk, H, D, "bf16", seed=9)
    prep = oracle.attn_prep(q, k, "bf16", mode)
    qf = oracle.to_float(q, "bf16").transpose(0, 2, 1, 3)           # [B, H, Lq, D]
    kf = oracle.to_float(k, "bf16").transpose(0, 2, 1, 3)
    if mode == "ref":
        # K per 64 keys after subtracting its per-channel mean (sum in fp32 times 1/L)
        np.testing.assert_allclose(prep["ksum"], kf.astype(np.float64).sum(axis=2), rtol=1e-5, atol=1e-3)
        kf = kf - prep["ksum"][:, :, None, :] * np.float32(1.0 / Lk)
        _check_block_codes(kf, prep["k_codes"], prep["k_scale"], 64)
        # Q per token
        _check_block_codes(qf, prep["q_codes"], prep["q_scale"], 1)
    else:
        _check_block_codes(kf, prep["k_codes"], prep["k_scale"], 64)
        qblk = prep["q_scale"][:, :, ::64]
        assert np.array_equal(np.repeat(qblk, 64, axis=2)[:, :, :Lq], prep["q_scale"])
        _check_block_codes(qf, prep["q_codes"], qblk, 64)
