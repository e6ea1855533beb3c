"""ctypes binding of librustane_cuda.so (declared in include/rustane_cuda.h).

The library is the product; this module only loads it and declares argument
types.  It raises if the shared object is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("librustane_cuda.so")
HEADER = Path(__file__).resolve().parent.parent / "include" / "rustane_cuda.h"

RT_OK = 0
ERRORS = {
    -1: "RT_ERR_ARG", -2: "RT_ERR_SHAPE", -3: "RT_ERR_CUDA", -4: "RT_ERR_OOM", -5: "RT_ERR_TOKEN",
    -6: "RT_ERR_DEVICE", -7: "RT_ERR_NCCL", -8: "RT_ERR_STATE", -9: "RT_ERR_NONFINITE",
}

EPI_BF16, EPI_F32, EPI_F32_ACC, EPI_RESIDUAL, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD = range(7)

c_int, c_int64, c_float, c_void_p, c_uint32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint32
c_float_p = ctypes.POINTER(ctypes.c_float)
c_uint32_p = ctypes.POINTER(ctypes.c_uint32)

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "rt_kernel_gemm": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int,
                               c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_float, c_int,
                               c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
}

_lib = None


class RustaneError(RuntimeError):
    def __init__(self, code: int, msg: str = ""):
        self.code = code
        super().__init__(f"{ERRORS.get(code, code)}{': ' + msg if msg else ''}")


def lib() -> ctypes.CDLL:
    """Load librustane_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m rustane_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(code: int, msg: str = "") -> None:
    if code != RT_OK:
        raise RustaneError(code, msg)
