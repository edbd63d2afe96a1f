"""ctypes binding of the native library ``libca_b200.so``.

The library exports the C ABI declared in ``include/continuum_attention_b200.h``.
This module only loads it and declares argument types; it never falls back to
anything else: if the library is missing, every operator call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libca_b200.so")

CA_DTYPE_F32, CA_DTYPE_BF16, CA_DTYPE_F16 = 0, 1, 2
CA_IMPL_AUTO, CA_IMPL_SIMT, CA_IMPL_TCGEN05 = 0, 1, 2
CA_LAYOUT_BHTD, CA_LAYOUT_BTHD = 0, 1
CA_BWD_DETERMINISTIC = 1
STATUS_NAMES = {0: "CA_OK", 1: "CA_ERR_INVALID_ARGUMENT", 2: "CA_ERR_UNSUPPORTED", 3: "CA_ERR_CUDA",
                4: "CA_ERR_WORKSPACE", 5: "CA_ERR_DEVICE_TIMEOUT"}

# every function the header declares, with (restype, argtypes)
_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "ca_abi_version": (_int, []),
    "ca_last_error": (ctypes.c_char_p, []),
    "ca_row_stats_floats": (_int, []),
    "ca_forward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "ca_forward_ex": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp]),
    "ca_backward_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _int]),
    "ca_backward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                           _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "ca_backward_ex": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                              _i64, _i64, _i64, _i64, _int, _int, _int, _vp]),
    "ca_backward_ex2": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                               _i64, _i64, _i64, _i64, _int, _int, _int, _int, _vp]),
    "ca_backward_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "ca_device_status": (_int, [_int]),
    "ca_last_launch_count": (_int, []),
    "ca_rope_qkv_forward": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp]),
    "ca_rope_qkv_backward": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp]),
    "ca_selftest_wait_timeout": (_int, [_i64, _vp]),
    "ca_rmsnorm_workspace_size": (_sz, [_i64, _i64]),
    "ca_rmsnorm_forward": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int, _int, _vp]),
    "ca_rmsnorm_backward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _int, _int, _vp]),
    "ca_add_rmsnorm_forward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "ca_add_rmsnorm_backward": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _vp]),
    "ca_gelu_tanh_forward": (_int, [_vp, _vp, _i64, _int, _vp]),
    "ca_gelu_tanh_backward": (_int, [_vp, _vp, _vp, _i64, _int, _vp]),
}

_lock = threading.Lock()
_lib = None


class CANativeError(RuntimeError):
    """A non-zero status returned by the native library."""

    def __init__(self, func: str, status: int, message: str):
        self.status = status
        super().__init__(f"{func} failed with {STATUS_NAMES.get(status, status)}: {message}")


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"native library {LIB_PATH} is missing: build it with "
                    "`python -m continuum_attention_b200.build` (no CPU fallback exists)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(func: str, status: int) -> None:
    if status != 0:
        msg = lib().ca_last_error().decode("utf-8", "replace")
        raise CANativeError(func, status, msg)
