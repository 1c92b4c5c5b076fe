"""The C-ABI library itself, without a GPU: it builds for sm_100a, loads, and
exports every entry point include/*.h declares; host-side argument checks
report errors instead of aborting.  CPU only."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "tiny-llm_b200", "libtqb200.so")


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        syms |= set(re.findall(r"\b(tqb200_\w+)\s*\(", src))
    # static inline helpers in headers are not exported symbols
    return {s for s in syms if not s.endswith("_bytes")}


@pytest.fixture(scope="module")
def built():
    if not os.path.exists(LIB):
        from tqb200 import __name__ as _  # noqa: F401
        import importlib.util
        spec = importlib.util.spec_from_file_location("tqb200_build",
                                                      os.path.join(ROOT, "tiny-llm_b200", "build.py"))
        m = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(m)
        m.build()
    return LIB


def test_library_exports_declared_symbols(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\b(tqb200_\w+)$", out, flags=re.M))
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_python_binding_covers_header(built):
    from tqb200 import lib
    assert declared_symbols() <= set(lib.PROTOTYPES), \
        sorted(declared_symbols() - set(lib.PROTOTYPES))
    lib.load()


def test_no_device_is_an_error_not_an_abort(built):
    from tqb200 import lib
    L = lib.load()
    if lib.device_count() > 0:
        pytest.skip("a GPU is visible")
    y = np.zeros(4, np.float32)
    st = L.tqb200_matvec_i4(np.zeros(6, np.uint8), np.ones(4, np.float32), y, 1, 4, 4)
    assert st == 4  # TQB200_ERR_NO_DEVICE
    assert b"no CUDA device" in L.tqb200_last_error()
    with pytest.raises(lib.TQB200Error):
        lib.matvec_i4(np.zeros(6, np.uint8), np.ones(4, np.float32), 1, 4, 4)


def test_bad_arguments_rejected_before_device(built):
    from tqb200 import lib
    L = lib.load()
    y = np.zeros(4, np.float32)
    st = L.tqb200_matvec_i4(np.zeros(6, np.uint8), np.ones(4, np.float32), y, 1, 4, 3)
    assert st == 1  # odd group size
    assert b"group_size" in L.tqb200_last_error()
    assert L.tqb200_status_string(5) == b"device wait timed out"
    # the tensor-core matmul needs whole 32-column groups
    yy = np.zeros(8, np.float32)
    st = L.tqb200_matmul_i4(np.zeros(64, np.uint8), np.ones(32, np.float32), yy, 1, 16, 2, 16)
    assert st == 1 and b"not 32, 64 or 128" in L.tqb200_last_error()
    # weights in 256-row tile blocks, then two bf16 planes of (G + 16) slots per group
    # and 16-padded column
    assert L.tqb200_matmul_i4_scratch_bytes(768, 2048, 37, 64) == 3 * 32 * 256 * 36 + 2 * 32 * 80 * 48 * 2
    assert L.tqb200_matmul_i4_scratch_bytes(768, 2048, 37, 48) == 0


def test_prefill_arguments_rejected_before_device(built):
    """tqb200_engine_prefill / _profile_prefill validate their arguments on the host."""
    import ctypes as C
    from tqb200 import lib
    L = lib.load()
    toks = np.array([1, 2, 3], np.int32)
    nxt = C.c_int(-1)
    assert L.tqb200_engine_prefill(None, toks, 3, C.byref(nxt)) == 1
    assert b"prefill" in L.tqb200_last_error()
    ms = np.zeros(14, np.float32)
    assert L.tqb200_engine_profile_prefill(None, toks, 3, ms, 14, C.byref(nxt)) == 1
