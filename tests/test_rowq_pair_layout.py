"""CPU model of the index mapping of ``rowq_pair_kernel`` and ``rowq_cta_pair_kernel``
(diffucore_b200/csrc/rowquant.cuh).

The kernel computes two ConvRot groups per half-warp at once: lane L of half h holds, for
iteration j, value i of group ga = 4 j + h and of group gb = ga + 2 (layout X: element 16 i + L of
the group), applies the LayerNorm + modulation by column, rotates through two swizzled scratch
transposes and stores 16 codes per lane at 256 g + 16 L. This model follows those index formulas
with numpy float32 arithmetic (every operation IEEE round-to-nearest, as on the GPU) and must
reproduce the per-group reference: the oracle's butterfly quantizer on the modulated row. It
checks the mapping on CPU; the GPU test compares the kernel with the default one bit for bit.
The one-CTA-per-row form for wide rows gives half-warp hw of 16 the groups 32 j + hw and
32 j + hw + 16; every group of a row is computed exactly once under both mappings.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle

F = np.float32


def _rt(x: np.ndarray) -> np.ndarray:
    return oracle.to_float(oracle.to_bits(x.astype(F), "bf16"), "bf16")


def _sub_twice(s, x):
    return (s + (F(-2.0) * x).astype(F)).astype(F)


P0123, P0213, S0123 = 0, 1, 2


def _orders(K):
    """Summation order per stage (d3, d2, d1, d0) of the reference's Triton butterfly for a row of
    K elements (its block width is the next power of two >= K)."""
    block = 256
    while block < K:
        block *= 2
    if block <= 256:
        return P0213, P0213, P0213, P0123
    if block == 512:
        return P0123, P0213, P0213, S0123
    if block == 1024:
        return P0213, P0213, P0123, S0123
    return P0213, P0213, S0123, S0123


def _quad(x0, x1, x2, x3, ord_):
    if ord_ == P0213:
        return ((x0 + x2).astype(F) + (x1 + x3).astype(F)).astype(F)
    if ord_ == S0123:
        return (((x0 + x1).astype(F) + x2).astype(F) + x3).astype(F)
    return ((x0 + x1).astype(F) + (x2 + x3).astype(F)).astype(F)


def _r4_outer(x, ord_):               # x: [16, lanes]
    y = np.empty_like(x)
    for b in range(4):
        s = _quad(x[b], x[4 + b], x[8 + b], x[12 + b], ord_)
        for a in range(4):
            y[4 * a + b] = _sub_twice(s, x[4 * (3 - a) + b])
    return y


def _r4_inner(x, ord_):
    y = np.empty_like(x)
    for a in range(4):
        s = _quad(x[4 * a], x[4 * a + 1], x[4 * a + 2], x[4 * a + 3], ord_)
        for b in range(4):
            y[4 * a + b] = _sub_twice(s, x[4 * a + 3 - b])
    return y


def _rotate_half_warp(x, K):
    """rotate256_pair for one slot (.x or .y) of the 16 lanes of a row K wide: x [16 values, 16 lanes]."""
    o3, o2, o1, o0 = _orders(K)
    x = _r4_inner(_r4_outer(x, o3), o2)
    scr = np.zeros(256, dtype=F)
    for L in range(16):
        for i in range(16):
            scr[16 * i + (L ^ i)] = x[i, L]
    y = np.empty_like(x)
    for L in range(16):
        for c in range(16):
            y[c, L] = scr[16 * L + (c ^ L)]
    y = _r4_inner(_r4_outer(y, o1), o0)
    return (y * F(0.0625)).astype(F)


def _model_row(row, mod_a, mod_sh, mean, rstd, lnmod):
    """Codes and scale of one row as rowq_pair_kernel computes them."""
    K = row.size
    ng = K // 256
    nit2 = (ng + 3) // 4
    vals = {}
    for j in range(nit2):
        for h in range(2):
            ga, gb = 4 * j + h, 4 * j + h + 2
            slots = []
            for g in (ga, gb):
                live = g < ng
                x = np.zeros((16, 16), dtype=F)           # [value i, lane L]
                for L in range(16):
                    for i in range(16):
                        col = 256 * (g if live else 0) + 16 * i + L
                        v = row[col] if live else F(0)
                        if lnmod:
                            n = _rt(np.array([(v + F(-mean)) * F(rstd)], dtype=F))[0]
                            y = _rt(np.array([F(mod_a[col]) * n], dtype=F))[0]
                            v = _rt(np.array([y + F(mod_sh[col])], dtype=F))[0] if live else F(0)
                        x[i, L] = v
                slots.append((g, live, x))
            if 4 * j < ng:
                slots = [(g, live, _rotate_half_warp(x, K)) for g, live, x in slots]
            for g, live, x in slots:
                if live:
                    vals[g] = x                            # layout Y: lane L holds 16 L + c
    amax = max(float(np.abs(v).max()) for v in vals.values())
    scale = np.float32(max(F(amax) / F(127.0), F(1e-30)))
    codes = np.zeros(K, dtype=np.int8)
    for g, x in vals.items():
        for L in range(16):
            seg = (x[:, L] / scale).astype(F)
            codes[256 * g + 16 * L: 256 * g + 16 * L + 16] = np.clip(np.rint(seg), -128, 127).astype(np.int8)
    return codes, scale


@pytest.mark.parametrize("K", [256, 768, 1280, 3072])
def test_pair_layout_matches_butterfly_quantizer(K):
    rng = np.random.default_rng(K)
    x = _rt(rng.standard_normal((2, K)).astype(F) * F(2.0))
    ref_q, ref_s = oracle.quant_rows(oracle.to_bits(x, "bf16"), "bf16", 256)
    for m in range(2):
        q, s = _model_row(x[m], None, None, 0.0, 1.0, False)
        assert np.array_equal(q, ref_q[m]) and s == ref_s[m]


@pytest.mark.parametrize("K", [512, 3072])
def test_pair_layout_applies_modulation_by_column(K):
    """The modulation each element receives is its own column's: the model equals the butterfly
    quantizer on the row modulated element-wise beforehand."""
    rng = np.random.default_rng(K + 1)
    x = _rt(rng.standard_normal(K).astype(F) * F(3.0) + F(0.5))
    scale_v = _rt((rng.standard_normal(K) * 0.3).astype(F))
    shift_v = _rt((rng.standard_normal(K) * 0.3).astype(F))
    mod_a = _rt((F(1.0) + scale_v).astype(F))
    mean, rstd = F(x.mean(dtype=np.float64)), F(1.0 / np.sqrt(x.var(dtype=np.float64) + 1e-6))
    n = _rt(((x + F(-mean)).astype(F) * rstd).astype(F))
    y = _rt(_rt((mod_a * n).astype(F)) + shift_v)
    ref_q, ref_s = oracle.quant_rows(oracle.to_bits(y[None, :], "bf16"), "bf16", 256)
    q, s = _model_row(x, mod_a, shift_v, mean, rstd, True)
    assert np.array_equal(q, ref_q[0]) and s == ref_s[0]


def _model_row_cta(row):
    """rowq_cta_pair_kernel: half-warp hw of 16 computes groups 32 j + hw and 32 j + hw + 16."""
    K = row.size
    ng = K // 256
    nit2 = (ng + 31) // 32
    vals = {}
    for j in range(nit2):
        for hw in range(16):
            warp = hw // 2
            for g in (32 * j + hw, 32 * j + hw + 16):
                if g >= ng:
                    continue
                x = np.zeros((16, 16), dtype=F)
                for L in range(16):
                    for i in range(16):
                        x[i, L] = row[256 * g + 16 * i + L]
                assert 32 * j + 2 * warp < ng          # the warp-uniform rotate condition holds
                assert g not in vals
                vals[g] = _rotate_half_warp(x, K)
    assert sorted(vals) == list(range(ng))
    amax = max(float(np.abs(v).max()) for v in vals.values())
    scale = np.float32(max(F(amax) / F(127.0), F(1e-30)))
    codes = np.zeros(K, dtype=np.int8)
    for g, x in vals.items():
        for L in range(16):
            seg = (x[:, L] / scale).astype(F)
            codes[256 * g + 16 * L: 256 * g + 16 * L + 16] = np.clip(np.rint(seg), -128, 127).astype(np.int8)
    return codes, scale


@pytest.mark.parametrize("K", [4352, 12288, 15360, 16384])
def test_cta_pair_layout_matches_butterfly_quantizer(K):
    rng = np.random.default_rng(K)
    x = _rt(rng.standard_normal((1, K)).astype(F))
    ref_q, ref_s = oracle.quant_rows(oracle.to_bits(x, "bf16"), "bf16", 256)
    q, s = _model_row_cta(x[0])
    assert np.array_equal(q, ref_q[0]) and s == ref_s[0]


@pytest.mark.parametrize("ng", range(1, 65))
def test_pair_mappings_cover_every_group_once(ng):
    warp_groups = [g for j in range((ng + 3) // 4) for h in range(2) for g in (4 * j + h, 4 * j + h + 2) if g < ng]
    cta_groups = [g for j in range((ng + 31) // 32) for hw in range(16) for g in (32 * j + hw, 32 * j + hw + 16)
                  if g < ng]
    assert sorted(cta_groups) == list(range(ng))
    if ng <= 16:                                   # the warp kernel serves K <= 4096
        assert sorted(warp_groups) == list(range(ng))
