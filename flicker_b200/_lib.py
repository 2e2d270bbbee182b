"""ctypes binding of libflicker_b200.so (the C ABI declared in include/flicker_b200.h).

The library is loaded from this package directory. There is no fallback: if
the shared object is missing or cannot be loaded, ``lib()`` raises, so a
product call never silently runs anything but the sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libflicker_b200.so")

FLK_OK = 0
FLK_ERR_INVALID_ARGUMENT = -1
FLK_ERR_UNSUPPORTED = -2
FLK_ERR_CUDA = -3
FLK_ERR_WORKSPACE = -4
FLK_ERR_DEVICE_TIMEOUT = -5
FLK_ERR_NO_DEVICE = -6

_u16p = ctypes.c_void_p
_f32p = ctypes.c_void_p
_int = ctypes.c_int

# name -> (restype, argtypes), mirroring include/flicker_b200.h
SIGNATURES = {
    "flk_qk_prep": (_int, [_u16p, _u16p, _u16p, _f32p, _f32p, ctypes.c_float, _int, _int, _int, _int,
                           _u16p, _u16p, _u16p, ctypes.c_void_p]),
    "flk_qk_prep_into": (_int, [_u16p, _u16p, _u16p, _f32p, _f32p, ctypes.c_float, _int, _int, _int, _int,
                                _u16p, _u16p, _u16p, _int, _int, ctypes.c_void_p]),
    "flk_attend_merged": (_int, [_u16p, _u16p, _u16p, _int, _int, _int, _int, _u16p, ctypes.c_void_p,
                                 ctypes.c_size_t, ctypes.c_void_p]),
    "flk_attend_gather": (_int, [_u16p, _u16p, _u16p, _int, _int, _int, _int, ctypes.POINTER(ctypes.c_void_p),
                                 _int, _int, _int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "flk_attend_gather_multicast": (_int, [_u16p, _u16p, _u16p, _int, _int, _int, _int, _u16p, _int, _int,
                                           ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "flk_linear": (_int, [_u16p, _u16p, _int, _int, _int, _u16p, ctypes.c_void_p]),
    "flk_linear_qk_prep": (_int, [_u16p, _u16p, _int, _int, _int, _u16p, _u16p, _f32p, _f32p, ctypes.c_float,
                                  _int, _int, _int, _int, _u16p, _u16p, _u16p, _int, _int, ctypes.c_void_p,
                                  ctypes.c_void_p]),
    "flk_attend": (_int, [_u16p, _u16p, _u16p, _int, _int, _int, _int, _u16p, ctypes.c_void_p,
                          ctypes.c_size_t, ctypes.c_void_p]),
    "flk_attend_workspace_size": (ctypes.c_size_t, [_int, _int, _int, _int]),
    "flk_attend_schedule": (_int, [_int, _int, _int, _int, _int, ctypes.POINTER(ctypes.c_longlong)]),
    "flk_attend_noalloc": (_int, [_u16p, _u16p, _u16p, _int, _int, _int, _int, _u16p, ctypes.c_void_p]),
    "flk_w8a8_quantize_act": (_int, [_u16p, _f32p, _int, _int, ctypes.c_void_p, _f32p, ctypes.c_void_p]),
    "flk_w8a8_gemm": (_int, [ctypes.c_void_p, ctypes.c_void_p, _f32p, _f32p, _int, _int, _int, _u16p,
                             ctypes.c_void_p]),
    "flk_i8_gemm_s32": (_int, [ctypes.c_void_p, ctypes.c_void_p, _int, _int, _int, ctypes.c_void_p,
                               ctypes.c_void_p]),
    "flk_logit_bound": (_int, [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float), _int,
                               ctypes.POINTER(ctypes.c_float)]),
    "flk_device_status": (_int, []),
    "flk_selftest_wait_timeout": (_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "flk_selftest_quotient": (_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_void_p]),
    "flk_selftest_exp2": (_int, [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p]),
    "flk_kernel_binary_version": (_int, []),
    "flk_error_string": (ctypes.c_char_p, [_int]),
    "flk_abi_version": (_int, []),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class FlickerError(RuntimeError):
    """A flk_* entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int):
        self.code = code
        msg = lib().flk_error_string(code).decode()
        super().__init__(f"{fn} failed with {code}: {msg}")


def lib() -> ctypes.CDLL:
    """Load (once) and return the library with argument types bound."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m flicker_b200.build` "
                        "(this package has no non-CUDA fallback)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(fn: str, code: int) -> None:
    if code != FLK_OK:
        raise FlickerError(fn, code)
