"""The C-ABI library loads on CPU and exports every symbol include/diffucore_b200.h declares;
without a GPU every compute entry point returns an error status with a reason (no CPU path)."""

from __future__ import annotations

import ctypes
import re

import pytest

from diffucore_b200 import _lib
from tests.conftest import ROOT, has_b200

HEADER = ROOT / "include" / "diffucore_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(dc_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert _declared() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared():
        assert hasattr(lib, name), name
    assert _lib.load().dc_version() == _lib.ABI_VERSION


def test_abi_version_matches_header():
    m = re.search(r"#define DC_ABI_VERSION (\d+)", HEADER.read_text())
    assert int(m.group(1)) == _lib.ABI_VERSION


@pytest.mark.skipif(has_b200(), reason="checks the no-GPU error path")
def test_compute_calls_fail_loudly_without_gpu():
    lib = _lib.load()
    assert lib.dc_quant_rows(None, _lib.DTYPE_BF16, 4, 16, 16, 0, 0, None, None, None) != 0
    assert lib.dc_last_error()
    assert lib.dc_gemm_w8a8(None, 16, None, 16, None, None, None, None, 16, _lib.DTYPE_I32, 4, 16, 16, 0, None) != 0


def test_argument_validation_without_gpu():
    lib = _lib.load()
    assert lib.dc_quant_rows(None, _lib.DTYPE_BF16, 4, 100, 100, 256, 0, None, None, None) != 0
    assert b"ConvRot" in lib.dc_last_error()
    n = ctypes.c_size_t(0)
    assert lib.dc_attn_workspace_size(1, 24, 4608, 4608, 96, 0, ctypes.byref(n)) != 0
    assert b"head dim" in lib.dc_last_error()
    assert lib.dc_attn_workspace_size(1, 24, 4608, 4608, 128, 0, ctypes.byref(n)) == 0
    lay = (ctypes.c_int64 * 8)()
    assert lib.dc_attn_workspace_layout(1, 24, 4608, 4608, 128, 0, lay) == 0
    assert lay[0] == 4608 and lay[1] == 4608 and lay[7] == n.value
    # codes + scales + ksum for config 2
    assert n.value >= 2 * 24 * 4608 * 128 + 24 * 4608 * 4


@pytest.mark.skipif(has_b200(), reason="host-side validation only; fake addresses must never reach a GPU")
def test_pointer_validation_without_gpu():
    """Null and under-aligned pointers are refused before any launch (addresses here are never
    dereferenced: every call must fail in the host-side checks)."""
    lib = _lib.load()
    a16, odd = 0x10000, 0x10001
    # GEMM: null operand, odd bf16 output, odd scale pointer
    assert lib.dc_gemm_w8a8(None, 16, a16, 16, a16, a16, None, a16, 16, _lib.DTYPE_BF16, 4, 16, 16, 0, None) != 0
    assert b"null" in lib.dc_last_error()
    assert lib.dc_gemm_w8a8(a16, 16, a16, 16, a16, a16, None, odd, 16, _lib.DTYPE_BF16, 4, 16, 16, 0, None) != 0
    assert b"aligned" in lib.dc_last_error()
    assert lib.dc_gemm_w8a8(a16, 16, a16, 16, a16 + 2, a16, None, a16, 16, _lib.DTYPE_BF16, 4, 16, 16, 0,
                            None) != 0
    assert b"aligned" in lib.dc_last_error()
    # quantizer: odd scale output
    assert lib.dc_quant_rows(a16, _lib.DTYPE_BF16, 4, 16, 16, 0, 0, a16, a16 + 2, None) != 0
    assert b"aligned" in lib.dc_last_error()
    # rescale: null scales
    assert lib.dc_rescale(a16, 16, None, a16, None, a16, 16, _lib.DTYPE_BF16, 4, 16, None) != 0
    assert b"null" in lib.dc_last_error()
    # attention: null v
    strides = _lib.i64_array([4096, 1024, 128])
    n = ctypes.c_size_t(0)
    assert lib.dc_attn_workspace_size(1, 8, 32, 32, 128, 0, ctypes.byref(n)) == 0
    assert lib.dc_attn_int8_fwd(a16, a16, None, _lib.DTYPE_BF16, 1, 8, 32, 32, 128, strides, strides, strides,
                                0.088, 0, a16, strides, a16, n.value, None) != 0
    assert b"null" in lib.dc_last_error()
    # qk_norm_rope: scale vector not 8-byte aligned, pe not 16-byte aligned
    assert lib.dc_qk_norm_rope(a16, _lib.DTYPE_BF16, 4, 2, 128, 768, 0, 256, a16 + 4, a16, None, None, 4,
                               a16, 0, None) != 0
    assert b"8-byte" in lib.dc_last_error()
    assert lib.dc_qk_norm_rope(a16, _lib.DTYPE_BF16, 4, 2, 128, 768, 0, 256, a16, a16, None, None, 4,
                               a16 + 8, 0, None) != 0
    assert b"16-byte" in lib.dc_last_error()


def test_quant_division_setting_round_trips():
    """The quantizer's division mode is host state: settable and readable without a GPU, unknown
    modes refused, IEEE (the reference's CPU arithmetic) by default."""
    from diffucore_b200 import _int8
    lib = _lib.load()
    assert lib.dc_quant_division() == _lib.QDIV_IEEE
    assert lib.dc_set_quant_division(7) != 0 and b"division" in lib.dc_last_error()
    try:
        _int8.set_quant_division("triton")
        assert lib.dc_quant_division() == _lib.QDIV_FULL and _int8.quant_division() == "triton"
        with pytest.raises(ValueError):
            _int8.set_quant_division("fast")
    finally:
        _int8.set_quant_division("ieee")
    assert _int8.quant_division() == "ieee"
