"""ctypes binding of libnvfp4_b200.so (the C ABI in include/nvfp4_b200.h).

The library is required: there is no CPU or PyTorch fallback.  ``lib()`` raises
when the shared object is missing, and ``check()`` turns a non-zero status into
a ``RuntimeError`` carrying the library's own message, mirroring the
reference's ``TORCH_CHECK`` failures (blackwell_nvfp4_gemv.cu:55-58).
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libnvfp4_b200.so")

_lock = threading.Lock()
_lib = None

I64 = ctypes.c_int64
VP = ctypes.c_void_p

class Group(ctypes.Structure):
    """struct nvfp4_group (include/nvfp4_b200.h)."""
    _fields_ = [("a", VP), ("b", VP), ("sfa", VP), ("sfb", VP), ("c", VP),
                ("M", I64), ("N", I64), ("K", I64), ("lda", I64), ("ldb", I64), ("ldc", I64)]


# name -> argtypes; every entry point returns int (status).
SIGNATURES: dict[str, list] = {
    "nvfp4_gemv": [VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, VP],
    "nvfp4_device_errors": [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int],
    "nvfp4_selftest_wait_timeout": [ctypes.c_uint64, VP],
    "nvfp4_selftest_wait_timeout_noalloc": [ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(ctypes.c_int), VP],
    "nvfp4_version": [],
    "nvfp4_dual_gemm": [VP, VP, VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, VP],
    "nvfp4_grouped_gemm": [ctypes.POINTER(Group), ctypes.c_int, VP],
    "nvfp4_mma_peak": [ctypes.c_int, VP],
    "nvfp4_mma_peak_pattern": [ctypes.c_int, ctypes.c_int, VP],
    "nvfp4_quantize": [VP, I64, I64, I64, VP, I64, VP, VP],
    "nvfp4_gemm_skinny": [VP, VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, VP],
    "nvfp4_gemv_grid": [I64, I64, I64, ctypes.POINTER(I64)],
    "nvfp4_set_peer_wait_ns": [ctypes.c_uint64],
    "nvfp4_gemv_allgather": [VP, VP, VP, VP, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                             VP, I64, I64, I64, I64, ctypes.POINTER(VP), ctypes.c_int, ctypes.c_int,
                             ctypes.c_uint32, VP],
}

STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "ALIGNMENT", 3: "CUDA", 4: "TIMEOUT", 5: "UNSUPPORTED"}


class Nvfp4Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"nvfp4 {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is not built; run `python __graft_entry__.py build` "
                    "(the CUDA library is required, there is no fallback)")
            l = ctypes.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                f = getattr(l, name)
                f.argtypes = args
                f.restype = ctypes.c_int
            l.nvfp4_last_error.argtypes = []
            l.nvfp4_last_error.restype = ctypes.c_char_p
            _lib = l
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().nvfp4_last_error().decode(errors="replace")
        raise Nvfp4Error(status, msg)


def device_errors(clear: bool = True) -> int:
    v = ctypes.c_uint32(0)
    check(lib().nvfp4_device_errors(ctypes.byref(v), int(clear)))
    return v.value
