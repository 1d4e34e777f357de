"""ctypes binding of ``libxm_gguf.so`` (the C ABI declared in ``include/xm_gguf.h``).

The library is required: there is no CPU fallback.  Importing this module
fails with ``ImportError`` when the shared library has not been built
(``python -m xanosmerks_b200.build``).
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libxm_gguf.so")

XM_OK = 0
XM_ERR_INVALID = -1
XM_ERR_UNSUPPORTED = -2
XM_ERR_CUDA = -3

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
PRO_NONE, PRO_RMSNORM, PRO_SWIGLU = 0, 1, 2
# expert activations of the MoE entry points, by the reference's names (primitives.py:52-62)
ACT = {"silu": 0, "swish": 0, "gelu": 1, "relu": 2, "identity": 3}

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "xm_abi_version": (_int, []),
    "xm_last_error": (ctypes.c_char_p, []),
    "xm_qtype_info": (_int, [_int, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "xm_device_status": (_int, [_int]),
    "xm_device_status_async": (_int, [_vp, _vp]),
    "xm_dequantize": (_int, [_int, _vp, _i64, _i64, _vp, _int, _vp]),
    "xm_qgemv_workspace_size": (_i64, [_i64, _i64]),
    "xm_qgemv": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp, _i64, _vp]),
    "xm_qgemv_exact": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp]),
    "xm_split_activation": (_int, [_vp, _int, _i64, _i64, _vp, _i64, _vp]),
    "xm_qgemv_presplit": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "xm_qgemm_workspace_size": (_i64, [_i64, _i64]),
    "xm_qgemm_workspace_size_n": (_i64, [_i64, _i64, _i64]),
    "xm_qgemm": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp, _i64, _vp]),
    "xm_qgemm_ex": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _i64, _int, _vp, _f32, _vp, _vp, _int,
                           _vp, _i64, _vp]),
    "xm_qgemm_ex_pitched": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _vp, _int, _i64, _i64, _int, _vp, _f32, _vp,
                                   _vp, _int, _vp, _i64, _vp]),
    "xm_moe_workspace_size": (_i64, [_i64, _i64, _i64, _int, _int]),
    "xm_moe_forward": (_int, [_vp, _int, _i64, _i64, _vp, _int, _int, _i64, ctypes.POINTER(_vp),
                              ctypes.POINTER(_vp), ctypes.POINTER(_vp), _int, _int, _vp, _vp, _i64, _vp]),
    "xm_qgemv_noalloc": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _vp, _vp, _vp]),
    "xm_qgemv_ex": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _int, _i64, _i64, _int, _vp, _f32, _vp, _vp, _int,
                           _vp, _i64, _vp]),
    "xm_embed": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "xm_attention_workspace_size": (_i64, [_i64, _int, _i64]),
    "xm_attention": (_int, [_vp, _i64, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _f32, _i64, _vp, _i64, _vp,
                            _i64, _vp]),
    "xm_argmax": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "xm_moe_dispatch": (_int, [_vp, _int, _i64, _i64, _vp, _int, _int, _i64, _vp, _vp, _vp, _i64, _vp]),
    "xm_moe_experts_workspace_size": (_i64, [_i64, _i64, _i64]),
    "xm_moe_experts": (_int, [_vp, _int, _i64, _i64, _i64, _int, _vp, _vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                              ctypes.POINTER(_vp), _int, _int, _i64, _vp, _vp, _i64, _vp]),
    "xm_moe_combine": (_int, [_vp, _i64, _i64, _int, _int, _i64, _vp, _vp, _vp]),
    "xm_comm_buffer_size": (_i64, [_i64]),
    "xm_comm_create": (_int, [_int, _int, _i64, _int, ctypes.POINTER(_vp), _vp]),
    "xm_comm_open_peer": (_int, [_vp, _int, _vp]),
    "xm_comm_open_local": (_int, [_vp, _int, _vp]),
    "xm_comm_set_wait_limit": (_int, [_vp, _i64]),
    "xm_rmsnorm": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _f32, _vp, _vp]),
    "xm_comm_destroy": (_int, [_vp]),
    "xm_allreduce_add": (_int, [_vp, _vp, _vp, _i64, _vp]),
}


class XMError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with `python -m xanosmerks_b200.build` "
            f"(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check_device(what: str = "") -> None:
    """Raise if a bounded wait inside a kernel on the current device gave up
    (the device error word is non-zero), and clear the word.  Synchronises the
    device (the word is read with a blocking copy)."""
    st = lib.xm_device_status(1)
    if st < 0:
        raise XMError(f"{what}: {lib.xm_last_error().decode(errors='replace')}")
    if st:
        raise XMError(f"{what}: a bounded wait inside a kernel gave up (device error word {st}); the results of "
                      f"the calls since the last check are not valid")


def check(status: int, what: str = "") -> None:
    """Map an XM_* status to the exception the reference raises for the same condition."""
    if status == XM_OK:
        return
    msg = lib.xm_last_error().decode(errors="replace")
    if what:
        msg = f"{what}: {msg}"
    if status == XM_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status == XM_ERR_INVALID:
        raise ValueError(msg)
    raise XMError(msg)
