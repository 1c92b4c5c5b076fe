"""ctypes binding of libtqb200.so: the host-side mirror of the reference's
operator interface for the quantised decode path.

Function names and argument meaning follow the reference's dispatch entry
points (kernels/dispatch.h): ``matvec_i4(w, x, out_dim, in_dim, group_size)``
computes what ``tinyqwen::matvec_i4`` computes and returns ``y``.  A non-zero
status from the library raises ``TQB200Error`` carrying the library's message
(the reference aborts; kernels/dispatch.cpp:393-398).  If the shared library is
missing the import fails loudly: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import abi

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libtqb200.so")

_u8 = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i, _fl, _vp = C.c_int, C.c_float, C.c_void_p


class TQB200Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"tqb200 status {status}: {msg}")
        self.status = status


# name -> (argtypes, restype); every symbol include/tqb200.h declares appears here
PROTOTYPES = {
    "tqb200_version": ([], _i),
    "tqb200_last_error": ([], C.c_char_p),
    "tqb200_status_string": ([_i], C.c_char_p),
    "tqb200_device_count": ([C.POINTER(_i)], _i),
    "tqb200_set_resident_weights": ([_i], _i),
    "tqb200_clear_resident_weights": ([], _i),
    "tqb200_matvec_i4": ([_u8, _f, _f, _i, _i, _i], _i),
    "tqb200_matvec_pair_i4": ([_u8, _u8, _f, _f, _f, _i, _i, _i], _i),
    "tqb200_matvec_qkv_i4": ([_u8, _u8, _u8, _f, _f, _f, _f, _i, _i, _i, _i], _i),
    "tqb200_matvec_i4_sym": ([_u8, _f, _f, _i, _i, _i], _i),
    "tqb200_dequant_i4": ([_u8, _i, _i, _i, _f], _i),
    "tqb200_dev_matvec_i4": ([_vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_dev_matvec_i4_sym": ([_vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_dev_dequant_i4": ([_vp, _i, _i, _i, _vp, _vp], _i),
}

_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load (once) and type the library.  Raises OSError if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise OSError(f"{path} not built: run tiny-llm_b200/build.py (no CPU fallback exists)")
        L = C.CDLL(path)
        for name, (args, res) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _check(status: int):
    if status != 0:
        L = load()
        raise TQB200Error(status, (L.tqb200_last_error() or b"").decode(errors="replace"))


def device_count() -> int:
    n = C.c_int(0)
    load().tqb200_device_count(C.byref(n))
    return n.value


def set_resident_weights(on: bool):
    _check(load().tqb200_set_resident_weights(1 if on else 0))


def clear_resident_weights():
    _check(load().tqb200_clear_resident_weights())


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8a(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


# ---------------------------------------------------------------- i4
def matvec_i4(w, x, out_dim: int, in_dim: int, group_size: int) -> np.ndarray:
    y = np.zeros(out_dim, np.float32)
    _check(load().tqb200_matvec_i4(_u8a(w), _f32(x), y, out_dim, in_dim, group_size))
    return y


def matvec_pair_i4(w1, w2, x, out_dim: int, in_dim: int, group_size: int):
    y1 = np.zeros(out_dim, np.float32)
    y2 = np.zeros(out_dim, np.float32)
    _check(load().tqb200_matvec_pair_i4(_u8a(w1), _u8a(w2), _f32(x), y1, y2, out_dim, in_dim,
                                        group_size))
    return y1, y2


def matvec_qkv_i4(wq, wk, wv, x, q_dim: int, kv_dim: int, in_dim: int, group_size: int):
    yq = np.zeros(q_dim, np.float32)
    yk = np.zeros(kv_dim, np.float32)
    yv = np.zeros(kv_dim, np.float32)
    _check(load().tqb200_matvec_qkv_i4(_u8a(wq), _u8a(wk), _u8a(wv), _f32(x), yq, yk, yv, q_dim,
                                       kv_dim, in_dim, group_size))
    return yq, yk, yv


def matvec_i4_sym(w, x, out_dim: int, in_dim: int, group_size: int) -> np.ndarray:
    y = np.zeros(out_dim, np.float32)
    _check(load().tqb200_matvec_i4_sym(_u8a(w), _f32(x), y, out_dim, in_dim, group_size))
    return y


def dequant_i4(w, rows: int, dim: int, group_size: int) -> np.ndarray:
    out = np.zeros((rows, dim), np.float32)
    _check(load().tqb200_dequant_i4(_u8a(w), rows, dim, group_size, out))
    return out


# ---------------------------------------------------------------- device-pointer twins
def _stream(stream):
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:
            return None
    return stream


def dev_matvec_i4(w_ptr: int, x_ptr: int, y_ptr: int, out_dim: int, in_dim: int,
                  group_size: int, stream=None):
    _check(load().tqb200_dev_matvec_i4(w_ptr, x_ptr, y_ptr, out_dim, in_dim, group_size,
                                       _stream(stream)))


def dev_matvec_i4_sym(w_ptr: int, x_ptr: int, y_ptr: int, out_dim: int, in_dim: int,
                      group_size: int, stream=None):
    _check(load().tqb200_dev_matvec_i4_sym(w_ptr, x_ptr, y_ptr, out_dim, in_dim, group_size,
                                           _stream(stream)))


def dev_dequant_i4(w_ptr: int, rows: int, dim: int, group_size: int, out_ptr: int, stream=None):
    _check(load().tqb200_dev_dequant_i4(w_ptr, rows, dim, group_size, out_ptr, _stream(stream)))
