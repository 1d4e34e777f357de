"""CPU: the C-ABI library loads, exports every declared symbol, and validates arguments on the host."""

import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include"))) if f.endswith(".h")]


def declared_functions():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(xm_[A-Za-z0-9_]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "xm_dequantize" in names and "xm_qgemv" in names and "xm_last_error" in names


def test_library_exports_every_declared_symbol():
    from xanosmerks_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes binding covers all of them
    assert set(declared_functions()) <= set(_lib.SIGNATURES), set(declared_functions()) - set(_lib.SIGNATURES)


def test_qtype_geometry_matches_table():
    from xanosmerks_b200 import _lib, qtypes
    for qt in qtypes.BY_NAME.values():
        qk, rec = ctypes.c_int(), ctypes.c_int()
        assert _lib.lib.xm_qtype_info(qt.type_id, ctypes.byref(qk), ctypes.byref(rec)) == 0
        assert (qk.value, rec.value) == (qt.qk, qt.record), qt.name
    for bad in (16, 17, 20, 28, 29, 34, 35, 99):   # IQ*, F64, TQ*, unknown
        assert _lib.lib.xm_qtype_info(bad, None, None) == _lib.XM_ERR_UNSUPPORTED


def test_host_side_validation_without_launch():
    """Argument errors are reported before any CUDA call (status + message)."""
    from xanosmerks_b200 import _lib
    L = _lib.lib
    # IQ2_XXS -> unsupported, as the reference raises NotImplementedError
    assert L.xm_dequantize(16, None, 0, 256, None, 1, None) == _lib.XM_ERR_UNSUPPORTED
    assert b"not implemented" in L.xm_last_error()
    # ragged element count / short buffer -> invalid (numpy ValueError in the reference)
    assert L.xm_dequantize(12, None, 144, 255, None, 1, None) == _lib.XM_ERR_INVALID
    assert L.xm_dequantize(12, None, 143, 256, None, 1, None) == _lib.XM_ERR_INVALID
    assert L.xm_dequantize(12, None, 144, 256, None, 7, None) == _lib.XM_ERR_INVALID
    # empty tensor is a no-op
    assert L.xm_dequantize(12, None, 0, 0, None, 1, None) == 0
    # qgemv shape checks
    assert L.xm_qgemv(12, None, 0, 4, 256, None, 0, 9, None, None, None, 0, None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemv(12, None, 0, 4, 200, None, 0, 1, None, None, None, 0, None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemv(0, None, 0, 4, 256, None, 0, 1, None, None, None, 0, None) == _lib.XM_ERR_UNSUPPORTED
    assert L.xm_qgemv(12, None, 100, 4, 256, None, 0, 1, None, None, None, 0, None) == _lib.XM_ERR_INVALID
    # a single row of 4096 also carries the lane-major copy of the split (9,216 B)
    assert L.xm_qgemv_workspace_size(4096, 1) == 128 * 80 + 9216
    assert L.xm_qgemv_workspace_size(4096, 2) == 2 * 128 * 80
    # fused-prologue GEMV: unknown prologue, RMSNorm without weights, short row pitch
    assert L.xm_qgemv_ex(14, None, 0, 4, 256, None, 0, 1, 256, 3, None, 1e-5, None, None, 0, None, 0,
                         None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemv_ex(14, None, 0, 4, 256, None, 0, 1, 256, _lib.PRO_RMSNORM, None, 1e-5, None, None, 0, None,
                         0, None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemv_ex(14, None, 0, 4, 256, None, 0, 1, 256, _lib.PRO_SWIGLU, None, 1e-5, None, None, 0, None,
                         0, None) == _lib.XM_ERR_INVALID
    # decoder kernels: head_dim other than 128 is unsupported, bad shapes are invalid
    assert L.xm_attention(None, 0, None, None, None, 1, 1, 32, 8, 64, 5e5, 16, None, 0, None, 0,
                          None) == _lib.XM_ERR_UNSUPPORTED
    assert L.xm_attention(None, 0, None, None, None, 1, 9, 32, 8, 128, 5e5, 16, None, 0, None, 0,
                          None) == _lib.XM_ERR_INVALID
    assert L.xm_attention(None, 0, None, None, None, 1, 1, 32, 3, 128, 5e5, 16, None, 0, None, 0,
                          None) == _lib.XM_ERR_INVALID
    assert L.xm_embed(0, None, 0, 10, 4096, None, 1, None, None) == _lib.XM_ERR_UNSUPPORTED
    assert L.xm_argmax(None, 0, 10, None, None) == _lib.XM_ERR_INVALID
    assert L.xm_qgemv_workspace_size(100, 1) == 0
