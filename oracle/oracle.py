"""ctypes front-end of the CPU checkers.  TEST INFRASTRUCTURE ONLY.

``Oracle``  loads oracle/_build/libtqoracle.so, the C restatement (tq_oracle.c).
``RefLib``  loads oracle/_ref/libtqref.so, the reference's own CPU sources built
            by oracle/Makefile (present only where the reference tree was
            available at build time; it then travels with the built tree).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))
from tqb200 import abi  # noqa: E402

ORACLE_SO = os.path.join(HERE, "_build", "libtqoracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtqref.so")

_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8 = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32 = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_vp = C.c_void_p
_i = C.c_int
_fl = C.c_float


def build_oracle(ref: bool = False) -> None:
    """Compile the checkers (make -C oracle oracle [ref])."""
    targets = ["oracle"] + (["ref"] if ref else [])
    subprocess.check_call(["make", "-s", "-C", HERE, "-j8"] + targets)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8a(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


class _Common:
    """Shared numpy-level wrappers; subclasses bind the C symbols."""

    def matvec_i4(self, w, x, out_dim, in_dim, group_size):
        y = np.zeros(out_dim, np.float32)
        self._matvec_i4(_u8a(w), _f32(x), y, out_dim, in_dim, group_size)
        return y

    def matvec_vq2(self, w, x, out_dim, in_dim):
        y = np.zeros(out_dim, np.float32)
        self._matvec_vq2(_u8a(w), _f32(x), y, out_dim, in_dim)
        return y

    def matmul_i4(self, w, x_cols, M, K, N, group_size):
        """x_cols: [N, K] (one token per row == column-major X[K, N]); returns [N, M]."""
        y = np.zeros((N, M), np.float32)
        self._matmul_i4(_u8a(w), _f32(x_cols), y, M, K, N, group_size)
        return y

    def biip_rotate(self, x, scale, sign, block_size):
        x = _f32(x)
        y = np.zeros_like(x)
        self._biip(x, y, x.size, None if scale is None else _f32(scale).ctypes.data,
                   _f32(sign).ctypes.data, block_size)
        return y

    def rmsnorm(self, x, w, eps):
        x = _f32(x)
        y = np.zeros_like(x)
        self._rmsnorm(x, _f32(w), y, x.size, eps)
        return y

    def rope(self, q, k, n_heads, n_kv_heads, head_dim, pos, theta):
        q = _f32(q).copy()
        k = _f32(k).copy()
        self._rope(q, k, n_heads, n_kv_heads, head_dim, pos, theta)
        return q, k

    def attention(self, q, kc, vc, seq_len, max_seq_len, n_heads, n_kv_heads, head_dim, scale):
        out = np.zeros(n_heads * head_dim, np.float32)
        self._attn(_f32(q), _f32(kc), _f32(vc), seq_len, max_seq_len, n_heads, n_kv_heads,
                   head_dim, scale, out)
        return out

    def swiglu(self, g, u):
        g = _f32(g).copy()
        self._swiglu(g, _f32(u), g.size)
        return g

    def argmax(self, logits):
        l = _f32(logits)
        return int(self._argmax(l, l.size))

    def _bind_gdn_gptq(self, sig, pre):
        self._gptq = sig(pre + "matvec_gptq", [_u8, _f, _f, _i, _i, _i])
        self._l2n = sig(pre + "l2norm_inplace", [_f, _i, _fl])
        self._conv = sig(pre + "causal_conv1d_update", [_f, _f, _f, _f, _i, _i])
        self._gdn = sig(pre + "gdn_step", [_f, _f, _f, _f, _fl, _fl, _f, _i, _i])
        self._rmsg = sig(pre + "rmsnorm_gated", [_f, _f, _f, _f, _i, _fl])
        self._prope = sig(pre + "partial_rope", [_f, _f, _i, _i, _i, _i, _i, _fl])

    def matvec_gptq(self, w, x, out_dim, in_dim, group_size):
        y = np.zeros(out_dim, np.float32)
        self._gptq(_u8a(w), _f32(x), y, out_dim, in_dim, group_size)
        return y

    def matmul_gptq(self, w, x_cols, M, K, N, group_size):
        """x_cols [N, K]; returns [N, M] (matmul_gptq_ref: one matvec per column)."""
        return np.stack([self.matvec_gptq(w, x_cols[n], M, K, group_size) for n in range(N)])

    def l2norm_inplace(self, x, eps):
        x = _f32(x).copy()
        self._l2n(x, x.size, eps)
        return x

    def causal_conv1d_update(self, x, state, weight, dim, kernel_size):
        st = _f32(state).copy()
        out = np.zeros(dim, np.float32)
        self._conv(_f32(x), st, _f32(weight), out, dim, kernel_size)
        return out, st

    def gdn_step(self, S, q, k, v, g, beta, qk_dim, v_dim):
        S2 = _f32(S).copy()
        o = np.zeros(v_dim, np.float32)
        self._gdn(S2, _f32(q), _f32(k), _f32(v), g, beta, o, qk_dim, v_dim)
        return o, S2

    def rmsnorm_gated(self, x, gate, weight, eps):
        x = _f32(x)
        y = np.zeros_like(x)
        self._rmsg(x, _f32(gate), _f32(weight), y, x.size, eps)
        return y

    def partial_rope(self, q, k, n_heads, n_kv_heads, head_dim, rotary_dim, pos, theta):
        q, k = _f32(q).copy(), _f32(k).copy()
        self._prope(q, k, n_heads, n_kv_heads, head_dim, rotary_dim, pos, theta)
        return q, k

    def topk_softmax(self, logits, k):
        l = _f32(logits)
        idx = np.zeros(k, np.int32)
        w = np.zeros(k, np.float32)
        self._topk(l, l.size, k, idx, w)
        return idx, w


class Oracle(_Common):
    """The C restatement (oracle/tq_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build_oracle()
        L = C.CDLL(path)
        self.lib = L

        def sig(name, args, res=None):
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
            return fn

        self._matvec_i4 = sig("tqo_matvec_i4", [_u8, _f, _f, _i, _i, _i])
        self._matvec_w4a8 = sig("tqo_matvec_i4_w4a8", [_u8, _f, _f, _i, _i, _i])
        self._matmul_i4 = sig("tqo_matmul_i4", [_u8, _f, _f, _i, _i, _i, _i])
        self._dequant = sig("tqo_dequant_i4", [_u8, _i, _i, _i, _f])
        self._matvec_vq2 = sig("tqo_matvec_vq2", [_u8, _f, _f, _i, _i])
        self._matvec_f32 = sig("tqo_matvec_f32", [_f, _f, _f, _i, _i])
        self._biip = sig("tqo_biip_rotate", [_f, _f, _i, _vp, _vp, _i])
        self._rmsnorm = sig("tqo_rmsnorm", [_f, _f, _f, _i, _fl])
        self._rope = sig("tqo_rope", [_f, _f, _i, _i, _i, _i, _fl])
        self._attn = sig("tqo_attention_decode", [_f, _f, _f, _i, _i, _i, _i, _i, _fl, _f])
        self._attn16 = sig("tqo_attention_decode_f16kv",
                           [_f, _u16, _u16, _i, _i, _i, _i, _i, _fl, _f])
        self._swiglu = sig("tqo_swiglu", [_f, _f, _i])
        self._argmax = sig("tqo_argmax", [_f, _i], _i)
        self._topk = sig("tqo_topk_softmax", [_f, _i, _i, _i32, _f])
        self._f2h = sig("tqo_float_to_half", [_fl], C.c_uint16)
        self._h2f = sig("tqo_half_to_float", [C.c_uint16], _fl)
        self._bind_gdn_gptq(sig, "tqo_")
        sig("tqo_set_threads", [_i])
        sig("tqo_model_create", [C.POINTER(abi.ModelDesc), _i, _i], _vp)
        sig("tqo_model_step", [_vp, _i], _i)
        sig("tqo_model_logits", [_vp], C.POINTER(C.c_float))
        sig("tqo_model_hidden", [_vp], C.POINTER(C.c_float))
        sig("tqo_model_reset", [_vp])
        sig("tqo_model_destroy", [_vp])
        sig("tqo_model_set_partial", [_vp, _i, _i])
        sig("tqo_model_kv", [_vp, C.POINTER(C.c_size_t)], _vp)
        sig("tqo_model_set_position", [_vp, _i], _i)
        sig("tqo_model_set_kv_guide", [_vp, _vp, _fl])
        sig("tqo_model_kv_guide_counts", [_vp, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong),
                                           C.POINTER(C.c_double)])

    def set_threads(self, n: int):
        self.lib.tqo_set_threads(n)

    def matvec_i4_w4a8(self, w, x, out_dim, in_dim, group_size):
        y = np.zeros(out_dim, np.float32)
        self._matvec_w4a8(_u8a(w), _f32(x), y, out_dim, in_dim, group_size)
        return y

    def dequant_i4(self, w, rows, dim, group_size):
        out = np.zeros((rows, dim), np.float32)
        self._dequant(_u8a(w), rows, dim, group_size, out)
        return out

    def matvec_f32(self, w, x):
        w = _f32(w)
        y = np.zeros(w.shape[0], np.float32)
        self._matvec_f32(w, _f32(x), y, w.shape[0], w.shape[1])
        return y

    def attention_f16kv(self, q, kc16, vc16, seq_len, max_seq_len, n_heads, n_kv_heads,
                        head_dim, scale):
        out = np.zeros(n_heads * head_dim, np.float32)
        self._attn16(_f32(q), np.ascontiguousarray(kc16, np.uint16),
                     np.ascontiguousarray(vc16, np.uint16), seq_len, max_seq_len, n_heads,
                     n_kv_heads, head_dim, scale, out)
        return out

    def float_to_half(self, a) -> np.ndarray:
        a = _f32(a).ravel()
        return np.array([self._f2h(float(v)) for v in a], np.uint16)

    def model(self, synth_model, max_seq_len: int, kv_fp16: bool = False) -> "OracleModel":
        return OracleModel(self, synth_model, max_seq_len, kv_fp16)


class OracleModel:
    def __init__(self, orc: Oracle, sm, max_seq_len: int, kv_fp16: bool):
        self.orc = orc
        self.sm = sm  # keeps the weights alive
        self.vocab = sm.spec.vocab
        self.kv_fp16 = kv_fp16
        self.h = orc.lib.tqo_model_create(C.byref(sm.desc), max_seq_len, 1 if kv_fp16 else 0)

    def step(self, token: int) -> int:
        return int(self.orc.lib.tqo_model_step(self.h, token))

    def logits(self) -> np.ndarray:
        p = self.orc.lib.tqo_model_logits(self.h)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def set_partial(self, n_layers: int, head: bool):
        self.orc.lib.tqo_model_set_partial(self.h, n_layers, 1 if head else 0)

    def reset(self):
        self.orc.lib.tqo_model_reset(self.h)

    def kv(self) -> np.ndarray:
        """The KV arena as a writable numpy view (uint16 bits for fp16, else float32)."""
        n = C.c_size_t()
        p = self.orc.lib.tqo_model_kv(self.h, C.byref(n))
        raw = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value,))
        return raw.view(np.uint16 if self.kv_fp16 else np.float32)

    def set_kv_guide(self, guide, tol: float = 1e-5):
        """Another implementation's fp16 arena (uint16, this model's layout) after the
        same step: the next steps write their K/V rows from it, measuring how far this
        model's own rounding is (beyond one ulp, in units of the head row's largest
        magnitude; above tol is a mismatch).  None: off."""
        self._guide = None if guide is None else np.ascontiguousarray(guide, np.uint16)
        self.orc.lib.tqo_model_set_kv_guide(self.h, None if self._guide is None else
                                            self._guide.ctypes.data, tol)

    def kv_guide_counts(self):
        """(differing elements, mismatches beyond tol, largest distance beyond one ulp)."""
        f, m, d = C.c_longlong(0), C.c_longlong(0), C.c_double(0.0)
        self.orc.lib.tqo_model_kv_guide_counts(self.h, C.byref(f), C.byref(m), C.byref(d))
        return f.value, m.value, d.value

    def set_position(self, pos: int):
        if self.orc.lib.tqo_model_set_position(self.h, pos) != 0:
            raise ValueError(f"position {pos} out of range")

    def close(self):
        if self.h:
            self.orc.lib.tqo_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class RefLib(_Common):
    """The reference's own CPU code (oracle/_ref/libtqref.so)."""

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def __init__(self, path: str = REF_SO):
        L = C.CDLL(path)
        self.lib = L

        def sig(name, args, res=None):
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
            return fn

        self._matvec_i4 = sig("tqref_matvec_i4", [_u8, _f, _f, _i, _i, _i])
        self._matmul_i4 = sig("tqref_matmul_i4", [_u8, _f, _f, _i, _i, _i, _i])
        self._dequant_row = sig("tqref_dequant_i4_row", [_u8, _i, _i, _i, _f])
        self._matvec_vq2 = sig("tqref_matvec_vq2", [_u8, _f, _f, _i, _i])
        self._biip = sig("tqref_biip_rotate", [_f, _f, _i, _vp, _vp, _i])
        self._rmsnorm = sig("tqref_rmsnorm", [_f, _f, _f, _i, _fl])
        self._rope = sig("tqref_rope", [_f, _f, _i, _i, _i, _i, _fl])
        self._attn = sig("tqref_attention_decode", [_f, _f, _f, _i, _i, _i, _i, _i, _fl, _f])
        self._swiglu = sig("tqref_swiglu", [_f, _f, _i])
        self._argmax = sig("tqref_argmax", [_f, _i], _i)
        self._topk = sig("tqref_topk_softmax", [_f, _i, _i, _i32, _f])
        self._f2h = sig("tqref_float_to_half", [_fl], C.c_uint16)
        self._h2f = sig("tqref_half_to_float", [C.c_uint16], _fl)
        self._bind_gdn_gptq(sig, "tqref_")
        self._w4a8 = sig("tqref_matvec_i4_w4a8_naive", [_u8, _f, _f, _i, _i, _i])
        self._pack_sym = sig("tqref_pack_i4_rtn_symmetric", [_f, _i, _i, _i, _u8])
        self._random_vec = sig("tqref_random_vec", [C.c_size_t, C.c_uint32, _f])
        sig("tqref_model_open", [C.c_char_p, _i, _i, C.c_char_p, _i], _vp)
        sig("tqref_model_step", [_vp, _i], _i)
        sig("tqref_model_logits", [_vp], C.POINTER(C.c_float))
        sig("tqref_model_reset", [_vp])
        sig("tqref_model_close", [_vp])

    def dequant_i4(self, w, rows, dim, group_size):
        out = np.zeros((rows, dim), np.float32)
        w = _u8a(w)
        row = np.zeros(dim, np.float32)
        for r in range(rows):
            self._dequant_row(w, r, dim, group_size, row)
            out[r] = row
        return out

    def float_to_half(self, a) -> np.ndarray:
        a = _f32(a).ravel()
        return np.array([self._f2h(float(v)) for v in a], np.uint16)

    def matvec_i4_w4a8_naive(self, w, x, out_dim, in_dim, group_size):
        """The reference test's symmetric W4A8 checker (tests/test_matvec_i4.cpp:252-306)."""
        y = np.zeros(out_dim, np.float32)
        self._w4a8(_u8a(w), _f32(x), y, out_dim, in_dim, group_size)
        return y

    def pack_i4_rtn_symmetric(self, w, out_dim, in_dim, group_size):
        """The reference test's symmetric packer (tests/test_matvec_i4.cpp:403-438)."""
        ng = (in_dim + group_size - 1) // group_size
        dst = np.zeros(out_dim * ng * (4 + group_size // 2), np.uint8)
        self._pack_sym(_f32(w).ravel(), out_dim, in_dim, group_size, dst)
        return dst.reshape(out_dim, -1)

    def random_vec(self, n, seed):
        """The reference test's N(0,1) inputs (tests/test_matvec_i4.cpp:144-152)."""
        out = np.zeros(n, np.float32)
        self._random_vec(n, seed, out)
        return out

    def open_model(self, path: str, max_seq_len: int, vocab: int, kv_fp16: bool = False):
        err = C.create_string_buffer(512)
        h = self.lib.tqref_model_open(path.encode(), max_seq_len, 1 if kv_fp16 else 0, err, 512)
        if not h:
            raise RuntimeError("reference model load failed: " + err.value.decode())
        return RefModelHandle(self, h, vocab)


class RefModelHandle:
    def __init__(self, lib: RefLib, h, vocab: int):
        self.lib, self.h, self.vocab = lib, h, vocab

    def step(self, token: int) -> int:
        return int(self.lib.lib.tqref_model_step(self.h, token))

    def logits(self) -> np.ndarray:
        p = self.lib.lib.tqref_model_logits(self.h)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()

    def close(self):
        if self.h:
            self.lib.lib.tqref_model_close(self.h)
            self.h = None

    def __del__(self):
        self.close()
