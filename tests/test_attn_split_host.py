"""Host side of the key-split attention (dc_attn_int8_main_split, kernels.attn_int8_split) on CPU:
the wave-count model that decides when to split, the partials size the library asks for, and the
argument checks that refuse bad calls before any launch. The kernel itself is checked on a B200
(tests/test_gpu_attention_split.py)."""

from __future__ import annotations

import ctypes

import pytest

from diffucore_b200 import _lib, kernels
from tests.conftest import has_b200


@pytest.mark.parametrize("B,H,L,want", [
    (1, 24, 4608, 1),      # 432 CTAs fill three waves; no split
    (1, 3, 4608, 1),       # FLUX 1024^2 on 8 GPUs: the combine pass costs what the split saves (measured)
    (1, 3, 16896, 2),      # FLUX 2048^2 on 8 GPUs: 198 CTAs, two waves at 67 % (measured 8 % faster split)
    (1, 6, 16896, 1),      # 2048^2 on 4 GPUs: 396 CTAs, the unsplit kernels do as well
    (1, 12, 16896, 1),
    (1, 6, 4608, 1),       # 1024^2 on 4 GPUs
])
def test_split_choice(B, H, L, want):
    assert kernels.choose_attn_split(B, H, L, L) == want


def test_split_choice_never_exceeds_the_key_tiles():
    for Lk in (1, 100, 128, 129, 300):
        n = -(-Lk // 128)
        assert 1 <= kernels.choose_attn_split(1, 1, 4608, Lk, max_split=8) <= n


@pytest.mark.parametrize("Lk,nsplit,ranges", [(4608, 2, 2), (4608, 4, 4), (3953, 4, 4), (4608, 5, 5), (1000, 8, 8),
                                              (1000, 7, 4), (640, 4, 3)])
def test_partials_size(Lk, nsplit, ranges):
    """ranges = ceil(n / ceil(n / nsplit)) key ranges of ceil(n / nsplit) tiles (n = ceil(Lk / 128)),
    each leaving fp32 O [B*H, Lq_pad, D] and (m, l) per row, Lq_pad = Lq rounded up to 256."""
    B, H, Lq, D = 1, 3, 700, 128
    n = -(-Lk // 128)
    tps = -(-n // nsplit)
    assert -(-n // tps) == ranges
    assert kernels.attn_split_partials_bytes(B, H, Lq, Lk, D, nsplit) == ranges * B * H * 768 * (D * 4 + 8)


def test_partials_size_refuses_bad_split():
    n = ctypes.c_size_t(0)
    lib = _lib.load()
    assert lib.dc_attn_split_partials_size(1, 3, 4608, 4608, 128, 0, ctypes.byref(n)) != 0
    assert b"nsplit" in lib.dc_last_error()
    assert lib.dc_attn_split_partials_size(1, 3, 4608, 4608, 128, 37, ctypes.byref(n)) != 0
    assert lib.dc_attn_split_partials_size(1, 3, 4608, 4608, 96, 2, ctypes.byref(n)) != 0
    assert b"head dim" in lib.dc_last_error()


@pytest.mark.skipif(has_b200(), reason="host-side validation only; fake addresses must never reach a GPU")
def test_main_split_validation_without_gpu():
    """Refused before any launch: null or too small or misaligned partials, nsplit out of range
    (the addresses are never dereferenced)."""
    lib = _lib.load()
    a16 = 0x10000
    strides = _lib.i64_array([4096 * 384, 384, 128])
    ws = ctypes.c_size_t(0)
    assert lib.dc_attn_workspace_size(1, 3, 4096, 4096, 128, 0, ctypes.byref(ws)) == 0
    need = kernels.attn_split_partials_bytes(1, 3, 4096, 4096, 128, 2)

    def call(nsplit, partials, pbytes):
        return lib.dc_attn_int8_main_split(a16, _lib.DTYPE_BF16, 1, 3, 4096, 4096, 128, strides, 0.088, 0, a16,
                                           strides, a16, ws.value, nsplit, partials, pbytes, None)

    assert call(2, None, need) != 0 and b"partials" in lib.dc_last_error()
    assert call(2, a16, need - 1) != 0 and b"partials" in lib.dc_last_error()
    assert call(2, a16 + 16, need) != 0 and b"aligned" in lib.dc_last_error()
    assert call(0, a16, need) != 0 and b"nsplit" in lib.dc_last_error()
    assert call(33, a16, need) != 0 and b"nsplit" in lib.dc_last_error()
    assert call(2, a16, need) != 0            # valid arguments: fails only at the device check
    assert b"sm_" in lib.dc_last_error() or b"device" in lib.dc_last_error() or b"CUDA" in lib.dc_last_error()
