"""CPU: the C-ABI library builds, loads, and exports every declared symbol.

No compute call is made here (there is no GPU); argument validation that
returns before any CUDA call is exercised where it needs no device.
"""
import ctypes

import pytest

from slang_b200 import _lib, build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_exports_every_header_symbol(lib):
    declared = _lib.header_symbols()
    assert len(declared) >= 9
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"
    assert set(_lib.SIGNATURES) == set(declared), "ctypes signatures out of sync with the header"


def test_version(lib):
    assert b"sm_100a" in lib.sb_version()


def test_argument_validation_is_host_side(lib):
    # bad bit width: rejected before any CUDA call
    rc = lib.sb_dequant_f16(None, 3, None, _lib.SB_F16, 32, None, 4, 32, None)
    assert rc == _lib.SB_ERR_ARG
    assert b"bits" in lib.sb_last_error()
    # GEMV k not a multiple of 32
    rc = lib.sb_gemv_q4(None, None, _lib.SB_F16, 32, None, _lib.SB_F32, None, 8, 1, 8, 40, None)
    assert rc == _lib.SB_ERR_ARG
    # GEMV m out of range
    rc = lib.sb_gemv_q4(None, None, _lib.SB_F16, 32, None, _lib.SB_F32, None, 8, 9, 8, 64, None)
    assert rc == _lib.SB_ERR_ARG
    # fused GEMM K must be a multiple of 64
    rc = lib.sb_gemm_q4(None, None, None, _lib.SB_F16, 32, None, 4, 4, 96, ctypes.c_float(1.0), 96, 4, None, 0, None)
    assert rc == _lib.SB_ERR_ARG
    # misaligned pointers
    rc = lib.sb_gemm_f16(ctypes.c_void_p(8), ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 4, 16,
                         ctypes.c_float(1.0), 1, 16, 16, 4, None)
    assert rc == _lib.SB_ERR_ALIGN
    # empty problems are no-ops
    assert lib.sb_gemm_f16(None, None, None, 0, 4, 16, ctypes.c_float(1.0), 1, 16, 16, 4, None) == 0


def test_workspace_size_zero_for_empty(lib):
    assert lib.sb_gemm_q4_workspace_size(0, 10, 64) == 0


def test_peer_wait_limit_is_bounded_by_the_default():
    """The exchange's wait limit can be shortened, never lengthened past 2 s (host-only call)."""
    lib = _lib.load()
    assert lib.sb_peer_set_wait_limit_ns(3_000_000_000) == _lib.SB_ERR_ARG
    assert lib.sb_peer_set_wait_limit_ns(0) == _lib.SB_OK
