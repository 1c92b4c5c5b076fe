"""Device-memory copies for the GPU tests: raw pointers the library hands out (the
engine's KV arena) to and from numpy, through the CUDA runtime that ships with torch's
wheels (the same driver context libtqb200.so uses).  Test infrastructure only."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_rt = None


def _cudart():
    global _rt
    if _rt is None:
        import nvidia.cuda_runtime as cr
        base = list(cr.__path__)[0]
        _rt = C.CDLL(os.path.join(base, "lib", "libcudart.so.12"))
        _rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        _rt.cudaMemcpy.restype = C.c_int
    return _rt


def d2h(ptr: int, nbytes: int) -> np.ndarray:
    """nbytes from device address ptr as a uint8 array."""
    out = np.empty(nbytes, np.uint8)
    rc = _cudart().cudaMemcpy(out.ctypes.data, ptr, nbytes, 2)  # cudaMemcpyDeviceToHost
    assert rc == 0, f"cudaMemcpy D2H failed ({rc})"
    return out


def h2d(ptr: int, arr: np.ndarray) -> None:
    """The bytes of arr to device address ptr."""
    a = np.ascontiguousarray(arr)
    rc = _cudart().cudaMemcpy(ptr, a.ctypes.data, a.nbytes, 1)  # cudaMemcpyHostToDevice
    assert rc == 0, f"cudaMemcpy H2D failed ({rc})"
