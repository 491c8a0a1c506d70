"""CPU model of the key-split attention's arithmetic (attn_int8_kernel<..., SPLIT> and
attn_split_combine_kernel): each key range runs the kernel's online softmax in the exp2 domain
(scores s * c, running max m started from the range's first 64-key half and moved only when a half's
max exceeds it by more than 8 -- the lazy rescale -- sum l and unnormalized O relative to m), and the
combine merges the ranges as sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s with M = max_s m_s.
For any range split, including one tile per range and a short last tile, that equals exact
softmax attention over all keys (fp64 here; the kernels differ from it only by fp32 / bf16
rounding, which the GPU tests bound)."""

from __future__ import annotations

import numpy as np
import pytest

LAZY = 8.0


def _range_partial(x, v, lo, hi):
    """(O, m, l) of one row over keys [lo, hi) of exp2-domain scores x, 64-key halves as the
    kernel's softmax warps take them."""
    m = None
    o = np.zeros(v.shape[1])
    l = 0.0
    for h0 in range(lo, hi, 64):
        xs, vs = x[h0:min(h0 + 64, hi)], v[h0:min(h0 + 64, hi)]
        mt = xs.max()
        if m is None:
            m = mt
        elif mt > m + LAZY:                  # move the max, rescale what was summed so far
            alpha = 2.0 ** (m - mt)
            o, l, m = o * alpha, l * alpha, mt
        p = 2.0 ** (xs - m)
        o = o + p @ vs
        l = l + p.sum()
    return o, m, l


def _combine(parts):
    M = max(m for _, m, _ in parts)
    num = sum(o * 2.0 ** (m - M) for o, m, _ in parts)
    den = sum(l * 2.0 ** (m - M) for _, m, l in parts)
    return num / den


def _ranges(n_tiles, nsplit):
    tps = -(-n_tiles // nsplit)
    return [(s * tps, min((s + 1) * tps, n_tiles)) for s in range(-(-n_tiles // tps))]


@pytest.mark.parametrize("Lk,nsplit", [(4608, 2), (3953, 4), (640, 5), (1000, 8), (129, 2), (300, 1)])
@pytest.mark.parametrize("growing", [False, True])
def test_split_softmax_equals_exact(Lk, nsplit, growing):
    rng = np.random.default_rng(Lk + nsplit)
    D = 32
    x = rng.standard_normal(Lk) * 3.0
    if growing:                              # the running max moves inside ranges and differs across them
        x = x + np.linspace(0.0, 60.0, Lk)
    v = rng.standard_normal((Lk, D))
    n_tiles = -(-Lk // 128)
    parts = [_range_partial(x, v, lo * 128, min(hi * 128, Lk)) for lo, hi in _ranges(n_tiles, nsplit)]
    got = _combine(parts)
    p = 2.0 ** (x - x.max())
    want = (p @ v) / p.sum()
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_ranges_cover_every_tile_once():
    for n in range(1, 80):
        for ns in range(1, n + 1):
            rs = _ranges(n, ns)
            assert rs[0][0] == 0 and rs[-1][1] == n and all(a < b for a, b in rs)
            assert all(rs[i][1] == rs[i + 1][0] for i in range(len(rs) - 1))
            assert len(rs) <= ns
