"""ctypes binding of the C ABI declared in include/mg_gemm.h.

The product path has exactly one implementation: the sm_100a kernels in
libmg_gemm.so. If the library is missing or cannot load, every entry point
raises; there is no CPU or library fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

MG_OK = 0
MG_ERR_INVALID = 1
MG_ERR_UNSUPPORTED = 2
MG_ERR_CUDA = 3
MG_ERR_ALLOC = 4
MG_ERR_TIMEOUT = 5
MG_ERR_NO_KERNEL = 6

MG_MODE_TF32X3 = 0
MG_MODE_TF32 = 1
MG_MODE_DEFAULT = -1

MG_EPI_BIAS = 1
MG_EPI_CAUSAL = 2
MG_EPI_SOFTMAX = 4

MG_MAX_BATCH_DIMS = 6

_STATUS_NAMES = {
    MG_OK: "MG_OK",
    MG_ERR_INVALID: "MG_ERR_INVALID",
    MG_ERR_UNSUPPORTED: "MG_ERR_UNSUPPORTED",
    MG_ERR_CUDA: "MG_ERR_CUDA",
    MG_ERR_ALLOC: "MG_ERR_ALLOC",
    MG_ERR_TIMEOUT: "MG_ERR_TIMEOUT",
    MG_ERR_NO_KERNEL: "MG_ERR_NO_KERNEL",
}


class MacrogradError(RuntimeError):
    """A failing library call: carries the mg_status and the library's message
    (the counterpart of MACROGRAD_ERROR in macrograd/include/macrograd_error.h:95,
    which prints and aborts; here the error is raised instead)."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{_STATUS_NAMES.get(status, status)}: {message}")


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int32), ("N", ctypes.c_int32), ("K", ctypes.c_int32),
        ("trans_a", ctypes.c_int32), ("trans_b", ctypes.c_int32),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("batch_rank", ctypes.c_int32),
        ("batch", ctypes.c_int32 * MG_MAX_BATCH_DIMS),
        ("a_batch_stride", ctypes.c_int64 * MG_MAX_BATCH_DIMS),
        ("b_batch_stride", ctypes.c_int64 * MG_MAX_BATCH_DIMS),
        ("c_batch_stride", ctypes.c_int64 * MG_MAX_BATCH_DIMS),
        ("bias_batch_stride", ctypes.c_int64 * MG_MAX_BATCH_DIMS),
        ("bias_rs", ctypes.c_int64), ("bias_cs", ctypes.c_int64),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("epilogue", ctypes.c_int32), ("mode", ctypes.c_int32),
    ]


_lock = threading.Lock()
_lib = None

# name -> (restype, argtypes), exactly the declarations of include/mg_gemm.h
_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_I32 = ctypes.c_int32
SIGNATURES = {
    "mg_gemm_desc_init": (None, [ctypes.POINTER(GemmDesc), _I32, _I32, _I32, _I32, _I32]),
    "mg_gemm": (ctypes.c_int, [ctypes.POINTER(GemmDesc), _P, _P, _P, _P, _P]),
    "mg_matmul": (ctypes.c_int, [_P, _P, _P, _I32P, _I32P, _I32P, _I32, _I32, _I32, _P]),
    "mg_matmul_bias": (ctypes.c_int, [_P, _P, _P, _P, _I32P, _I32P, _I32P, _I32P, _I32, _I32, _I32, _P]),
    "mg_matmul_accumulate": (ctypes.c_int, [_P, _P, _P, _I32P, _I32P, _I32P, _I32, _I32, _I32, ctypes.c_float,
                                            _P]),
    "mg_sum_into": (ctypes.c_int, [_P, _P, _I32P, _I32P, _I32, ctypes.c_float, _P]),
    "mg_matmul_softmax": (ctypes.c_int, [_P, _P, _P, _P, _I32P, _I32P, _I32P, _I32P, _I32, _I32, _I32,
                                         ctypes.c_float, _I32, _P]),
    "mg_matmul_softmax_backward": (ctypes.c_int, [_P, _P, _P, _P, _I32P, _I32P, _I32P, _I32, _I32, _I32,
                                                  ctypes.c_float, _P]),
    "mg_matmul_noalloc": (ctypes.c_int, [_P, _P, _P, _I32P, _I32P, _I32P, _I32, _I32, _I32, _P]),
    "mg_gemm_scatter_rows": (ctypes.c_int, [ctypes.POINTER(GemmDesc), _P, _P, _P, ctypes.POINTER(_P), _I32,
                                            ctypes.c_int64, ctypes.c_int64, _P]),
    "mg_ipc_export": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
    "mg_ipc_import": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(_P)]),
    "mg_ipc_close": (ctypes.c_int, [_P]),
    "mg_set_allocator": (None, [_P, _P, _P]),
    "mg_set_mode": (ctypes.c_int, [_I32]),
    "mg_get_mode": (ctypes.c_int32, []),
    "mg_last_error": (ctypes.c_char_p, []),
    "mg_device_status": (ctypes.c_int, [_I32P, _I32]),
    "mg_launch_count": (ctypes.c_uint64, []),
    "mg_version": (ctypes.c_char_p, []),
}


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = False):
    """Loads libmg_gemm.so (building it first if asked and it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if build_if_missing:
                _build.build()
            else:
                raise MacrogradError(MG_ERR_NO_KERNEL,
                                     f"{path} is missing: build it with `python -m macrograd_b200.build`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != MG_OK:
        msg = load().mg_last_error()
        raise MacrogradError(status, msg.decode() if msg else "")


def i32_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int32 * max(1, len(vals)))(*vals)
