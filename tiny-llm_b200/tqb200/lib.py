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
_d = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
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
    "tqb200_dev_matvec_i4_pdl": ([_vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_dev_matvec_i4_sym": ([_vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_dev_dequant_i4": ([_vp, _i, _i, _i, _vp, _vp], _i),
    "tqb200_matmul_i4": ([_u8, _f, _f, _i, _i, _i, _i], _i),
    "tqb200_matmul_i4_scratch_bytes": ([_i, _i, _i, _i], C.c_size_t),
    "tqb200_dev_matmul_i4": ([_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "tqb200_matvec_vq2": ([_u8, _f, _f, _i, _i], _i),
    "tqb200_biip_rotate": ([_f, _f, _i, _vp, _vp, _i], _i),
    "tqb200_matvec_vq2_rot": ([_u8, _f, _f, _i, _i, _vp, _vp, _i], _i),
    "tqb200_dev_matvec_vq2_rot": ([_vp, _vp, _vp, _i, _i, _vp, _vp, _i, _vp], _i),
    "tqb200_rmsnorm": ([_f, _f, _f, _i, _fl], _i),
    "tqb200_rope": ([_f, _f, _i, _i, _i, _i, _fl], _i),
    "tqb200_attention_decode": ([_f, _f, _f, _i, _i, _i, _i, _i, _fl, _f], _i),
    "tqb200_dev_attention_decode_noalloc": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _fl, _vp, _vp], _i),
    "tqb200_attention_decode_f16kv": ([_f, _u16, _u16, _i, _i, _i, _i, _i, _fl, _f], _i),
    "tqb200_swiglu": ([_f, _f, _i], _i),
    "tqb200_argmax": ([_f, _i, C.POINTER(_i)], _i),
    "tqb200_topk_softmax": ([_f, _i, _i, _i32, _f], _i),
    "tqb200_engine_default_opts": ([_vp], None),
    "tqb200_nccl_unique_id": ([_vp], _i),
    "tqb200_engine_create": ([C.POINTER(abi.ModelDesc), _vp, C.POINTER(_vp)], _i),
    "tqb200_engine_step": ([_vp, _i, C.POINTER(_i)], _i),
    "tqb200_engine_reset": ([_vp], _i),
    "tqb200_engine_destroy": ([_vp], _i),
    "tqb200_engine_logits": ([_vp], _vp),
    "tqb200_engine_copy_logits": ([_vp, _f, _i], _i),
    "tqb200_engine_position": ([_vp], _i),
    "tqb200_engine_set_position": ([_vp, _i], _i),
    "tqb200_engine_stream": ([_vp, C.POINTER(_vp)], _i),
    "tqb200_engine_kv_cache": ([_vp, C.POINTER(_vp), C.POINTER(C.c_size_t)], _i),
    "tqb200_engine_weight_bytes": ([_vp, C.POINTER(C.c_size_t)], _i),
    "tqb200_engine_prefill_copy_bytes": ([_vp, C.POINTER(C.c_size_t)], _i),
    "tqb200_engine_generate": ([_vp, _i, _i, _i32, C.POINTER(_fl)], _i),
    "tqb200_engine_prefill": ([_vp, _i32, _i, C.POINTER(_i)], _i),
    "tqb200_engine_profile_prefill": ([_vp, _i32, _i, _f, _i, C.POINTER(_i)], _i),
    "tqb200_engine_profile_step": ([_vp, _i, _f, _i, C.POINTER(_i)], _i),
    "tqb200_engine_set_timeline": ([_vp, _i], _i),
    "tqb200_engine_exchange_handle": ([_vp, _vp], _i),
    "tqb200_engine_open_exchange": ([_vp, _vp, _i], _i),
    "tqb200_l2norm_inplace": ([_f, _i, _fl], _i),
    "tqb200_causal_conv1d_update": ([_f, _f, _f, _f, _i, _i], _i),
    "tqb200_gdn_step": ([_f, _f, _f, _f, _fl, _fl, _f, _i, _i], _i),
    "tqb200_dev_gdn_step": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_rmsnorm_gated": ([_f, _f, _f, _f, _i, _fl], _i),
    "tqb200_partial_rope": ([_f, _f, _i, _i, _i, _i, _i, _fl], _i),
    "tqb200_matvec_gptq": ([_u8, _f, _f, _i, _i, _i], _i),
    "tqb200_matmul_gptq": ([_u8, _f, _f, _i, _i, _i, _i], _i),
    "tqb200_dev_matvec_gptq": ([_vp, _i, _vp, _vp, _i, _i, _i, _vp], _i),
    "tqb200_matvec_f32": ([_f, _f, _f, _i, _i], _i),
    "tqb200_matvec_f16": ([_u16, _f, _f, _i, _i], _i),
    "tqb200_engine_timeline": ([_vp, _i, _d, _d, _i32, C.POINTER(_i), C.POINTER(C.c_double)], _i),
    "tqb200_engine_timeline_launches": ([_vp, _i, _i, _i32, _d, C.POINTER(_i)], _i),
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


def matmul_i4(w, x_cols, M: int, K: int, N: int, group_size: int) -> np.ndarray:
    """MatmulI4Fn: x_cols is X column-major ([N][K] in memory); returns Y as [N][M]."""
    y = np.zeros(M * N, np.float32)
    _check(load().tqb200_matmul_i4(_u8a(w), _f32(x_cols), y, M, K, N, group_size))
    return y.reshape(N, M)


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


# ---------------------------------------------------------------- VQ2 + BiIP
def matvec_vq2(w, x, out_dim: int, in_dim: int) -> np.ndarray:
    y = np.zeros(out_dim, np.float32)
    _check(load().tqb200_matvec_vq2(_u8a(w), _f32(x), y, out_dim, in_dim))
    return y


def _ptr_or_none(a):
    return None if a is None else _f32(a).ctypes.data


def biip_rotate(x, scale, sign, block_size: int) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    sc = None if scale is None else _f32(scale)
    sg = _f32(sign)
    _check(load().tqb200_biip_rotate(x, y, x.size, None if sc is None else sc.ctypes.data,
                                     sg.ctypes.data, block_size))
    return y


def matvec_vq2_rot(w, x, out_dim: int, in_dim: int, scale, sign, block_size: int) -> np.ndarray:
    y = np.zeros(out_dim, np.float32)
    sc = None if scale is None else _f32(scale)
    sg = None if sign is None else _f32(sign)
    _check(load().tqb200_matvec_vq2_rot(_u8a(w), _f32(x), y, out_dim, in_dim,
                                        None if sc is None else sc.ctypes.data,
                                        None if sg is None else sg.ctypes.data, block_size))
    return y


# ---------------------------------------------------------------- decode ops
def rmsnorm(x, weight, eps: float) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    _check(load().tqb200_rmsnorm(x, _f32(weight), y, x.size, eps))
    return y


def rope(q, k, n_heads: int, n_kv_heads: int, head_dim: int, pos: int, theta: float):
    q = _f32(q).copy()
    k = _f32(k).copy()
    _check(load().tqb200_rope(q, k, n_heads, n_kv_heads, head_dim, pos, theta))
    return q, k


def attention_decode(q, k_cache, v_cache, seq_len, max_seq_len, n_heads, n_kv_heads, head_dim,
                     scale) -> np.ndarray:
    out = np.zeros(n_heads * head_dim, np.float32)
    _check(load().tqb200_attention_decode(_f32(q), _f32(k_cache), _f32(v_cache), seq_len,
                                          max_seq_len, n_heads, n_kv_heads, head_dim, scale, out))
    return out


def attention_decode_f16kv(q, k_cache16, v_cache16, seq_len, max_seq_len, n_heads, n_kv_heads,
                           head_dim, scale) -> np.ndarray:
    out = np.zeros(n_heads * head_dim, np.float32)
    _check(load().tqb200_attention_decode_f16kv(
        _f32(q), np.ascontiguousarray(k_cache16, np.uint16),
        np.ascontiguousarray(v_cache16, np.uint16), seq_len, max_seq_len, n_heads, n_kv_heads,
        head_dim, scale, out))
    return out


def swiglu(gate, up) -> np.ndarray:
    g = _f32(gate).copy()
    _check(load().tqb200_swiglu(g, _f32(up), g.size))
    return g


def argmax(logits) -> int:
    l = _f32(logits)
    i = C.c_int(-1)
    _check(load().tqb200_argmax(l, l.size, C.byref(i)))
    return i.value


def topk_softmax(logits, k: int):
    l = _f32(logits)
    idx = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    _check(load().tqb200_topk_softmax(l, l.size, k, idx, w))
    return idx, w


# ---------------------------------------------------------------- engine
class EngineOpts(C.Structure):
    _fields_ = [("max_seq_len", C.c_int), ("kv_fp16", C.c_int), ("use_graph", C.c_int),
                ("pdl", C.c_int), ("device", C.c_int), ("tp_size", C.c_int), ("tp_rank", C.c_int),
                ("nccl_id", C.c_ubyte * 128), ("reserved", C.c_int * 8)]


def l2norm_inplace(x, eps: float) -> np.ndarray:
    """l2norm_inplace_ref (kernels/gdn/gdn_ops_ref.cpp:44-57); returns the normalised copy."""
    x = _f32(x).copy()
    _check(load().tqb200_l2norm_inplace(x, x.size, eps))
    return x


def causal_conv1d_update(x, state, weight, dim: int, kernel_size: int):
    """causal_conv1d_update_ref (:82-105); returns (out, new state)."""
    st = _f32(state).copy()
    out = np.zeros(dim, np.float32)
    _check(load().tqb200_causal_conv1d_update(_f32(x), st, _f32(weight), out, dim, kernel_size))
    return out, st


def gdn_step(S, q, k, v, g: float, beta: float, qk_dim: int, v_dim: int):
    """gdn_step_ref (:134-176); returns (o, new S)."""
    S2 = _f32(S).copy()
    o = np.zeros(v_dim, np.float32)
    _check(load().tqb200_gdn_step(S2, _f32(q), _f32(k), _f32(v), g, beta, o, qk_dim, v_dim))
    return o, S2


def rmsnorm_gated(x, gate, weight, eps: float) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    _check(load().tqb200_rmsnorm_gated(x, _f32(gate), _f32(weight), y, x.size, eps))
    return y


def partial_rope(q, k, n_heads: int, n_kv_heads: int, head_dim: int, rotary_dim: int, pos: int,
                 theta: float):
    q, k = _f32(q).copy(), _f32(k).copy()
    _check(load().tqb200_partial_rope(q, k, n_heads, n_kv_heads, head_dim, rotary_dim, pos, theta))
    return q, k


def matvec_gptq(w, x, out_dim: int, in_dim: int, group_size: int) -> np.ndarray:
    y = np.zeros(out_dim, np.float32)
    _check(load().tqb200_matvec_gptq(_u8a(w), _f32(x), y, out_dim, in_dim, group_size))
    return y


def matmul_gptq(w, x_cols, M: int, K: int, N: int, group_size: int) -> np.ndarray:
    """x_cols [N, K] (column-major X [K, N]); returns [N, M]."""
    y = np.zeros((N, M), np.float32)
    _check(load().tqb200_matmul_gptq(_u8a(w), _f32(x_cols), y, M, K, N, group_size))
    return y


def matvec_f32(w, x) -> np.ndarray:
    w = _f32(w)
    y = np.zeros(w.shape[0], np.float32)
    _check(load().tqb200_matvec_f32(w, _f32(x), y, w.shape[0], w.shape[1]))
    return y


def matvec_f16(w, x) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint16)
    y = np.zeros(w.shape[0], np.float32)
    _check(load().tqb200_matvec_f16(w, _f32(x), y, w.shape[0], w.shape[1]))
    return y


def nccl_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    _check(load().tqb200_nccl_unique_id(buf))
    return bytes(buf)


class Engine:
    """GPU decode engine (the reference's GpuDecode* registry entry, kernels/dispatch.h:353-378)."""

    def __init__(self, model, max_seq_len: int = 512, kv_fp16: bool = False,
                 use_graph: bool = True, pdl: bool = True, device: int = -1,
                 tp_size: int = 1, tp_rank: int = 0, nccl_id: bytes = b""):
        L = load()
        self.model = model  # keeps the host weights alive through create()
        self.vocab = model.spec.vocab
        o = EngineOpts()
        L.tqb200_engine_default_opts(C.byref(o))
        o.max_seq_len, o.kv_fp16 = max_seq_len, 1 if kv_fp16 else 0
        o.use_graph, o.pdl, o.device = 1 if use_graph else 0, 1 if pdl else 0, device
        o.tp_size, o.tp_rank = tp_size, tp_rank
        if tp_size > 1:
            assert len(nccl_id) == 128, "tensor parallel needs the 128-byte NCCL id"
            C.memmove(o.nccl_id, nccl_id, 128)
        h = C.c_void_p()
        _check(L.tqb200_engine_create(C.byref(model.desc), C.byref(o), C.byref(h)))
        self.h = h

    def step(self, token: int) -> int:
        nxt = C.c_int(-1)
        _check(load().tqb200_engine_step(self.h, int(token), C.byref(nxt)))
        return nxt.value

    def prefill(self, tokens) -> int:
        """QwenModel::forward_prefill: the prompt as one batch; returns the greedy next token."""
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = C.c_int(-1)
        _check(load().tqb200_engine_prefill(self.h, toks, len(toks), C.byref(nxt)))
        return nxt.value

    def logits(self) -> np.ndarray:
        out = np.zeros(self.vocab, np.float32)
        _check(load().tqb200_engine_copy_logits(self.h, out, self.vocab))
        return out

    def logits_ptr(self) -> int:
        return load().tqb200_engine_logits(self.h)

    def generate(self, token: int, n_steps: int):
        """n greedy steps with device-side token feedback; returns (tokens, device_ms)."""
        out = np.zeros(max(1, n_steps), np.int32)
        ms = C.c_float(0.0)
        _check(load().tqb200_engine_generate(self.h, int(token), n_steps, out, C.byref(ms)))
        return out[:n_steps].tolist(), ms.value

    KINDS = ("embed", "qkv", "qk_rope_kv", "attention", "o_proj", "gate_up", "down", "lm_head",
             "router", "moe_combine", "rmsnorm", "x_pack", "moe_plan", "swiglu")

    def profile_prefill(self, tokens):
        """A prefill launched kernel by kernel, CUDA events between launches; returns
        (next token, {kind: ms})."""
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        ms = np.zeros(len(self.KINDS), np.float32)
        nxt = C.c_int(-1)
        _check(load().tqb200_engine_profile_prefill(self.h, toks, len(toks), ms, len(self.KINDS),
                                                    C.byref(nxt)))
        return nxt.value, dict(zip(self.KINDS, ms.tolist()))

    def profile_step(self, token: int):
        """One kernel-by-kernel step timed with CUDA events; returns (next, {kind: ms})."""
        ms = np.zeros(len(self.KINDS), np.float32)
        nxt = C.c_int(-1)
        _check(load().tqb200_engine_profile_step(self.h, int(token), ms, ms.size, C.byref(nxt)))
        return nxt.value, dict(zip(self.KINDS, ms.tolist()))

    def exchange_handle(self) -> bytes:
        """This rank's activation arena as a 64-byte CUDA IPC handle (peer exchange)."""
        buf = (C.c_ubyte * 64)()
        _check(load().tqb200_engine_exchange_handle(self.h, buf))
        return bytes(buf)

    def open_exchange(self, handles):
        """Maps every other rank's arena (handles[r] = rank r's exchange_handle()); from the
        next step on the all-gathers run inside the producing kernels over NVLink."""
        blob = b"".join(handles)
        assert len(blob) == 64 * len(handles)
        buf = (C.c_ubyte * len(blob)).from_buffer_copy(blob)
        _check(load().tqb200_engine_open_exchange(self.h, buf, len(handles)))

    def set_timeline(self, max_steps: int):
        """Stamp every launch of the first max_steps steps of each generate() (0: off)."""
        _check(load().tqb200_engine_set_timeline(self.h, int(max_steps)))

    def timeline(self):
        """The last generate()'s in-graph timeline: (steps, span_ms, {kind: (excl_ms,
        incl_ms, launches)}) per step, for the kinds with launches."""
        n = len(self.KINDS)
        ex, inc = np.zeros(n, np.float64), np.zeros(n, np.float64)
        cnt = np.zeros(n, np.int32)
        steps, span = C.c_int(0), C.c_double(0.0)
        _check(load().tqb200_engine_timeline(self.h, n, ex, inc, cnt, C.byref(steps), C.byref(span)))
        kinds = {k: (float(ex[i]), float(inc[i]), int(cnt[i]))
                 for i, k in enumerate(self.KINDS) if cnt[i] > 0}
        return steps.value, span.value, kinds

    def timeline_launches(self, step: int = 0, max_launches: int = 4096):
        """[(kind, entry_first, entry_last, wait_first, wait_last, exit_first, exit_last)] in
        microseconds from the step's first stamp, for one recorded step."""
        kinds = np.zeros(max_launches, np.int32)
        us = np.zeros(6 * max_launches, np.float64)
        n = C.c_int(0)
        _check(load().tqb200_engine_timeline_launches(self.h, step, max_launches, kinds, us,
                                                      C.byref(n)))
        return [(self.KINDS[kinds[i]],) + tuple(us[6 * i: 6 * i + 6]) for i in range(n.value)]

    def reset(self):
        _check(load().tqb200_engine_reset(self.h))

    @property
    def position(self) -> int:
        return load().tqb200_engine_position(self.h)

    def set_position(self, pos: int):
        _check(load().tqb200_engine_set_position(self.h, pos))

    def stream(self) -> int:
        s = C.c_void_p()
        _check(load().tqb200_engine_stream(self.h, C.byref(s)))
        return s.value or 0

    def kv_cache(self):
        p, n = C.c_void_p(), C.c_size_t()
        _check(load().tqb200_engine_kv_cache(self.h, C.byref(p), C.byref(n)))
        return p.value, n.value

    def weight_bytes(self) -> int:
        n = C.c_size_t()
        _check(load().tqb200_engine_weight_bytes(self.h, C.byref(n)))
        return n.value

    def prefill_copy_bytes(self) -> int:
        """Bytes of repacked weight copies the batched prefill made (0: all read in place)."""
        n = C.c_size_t()
        _check(load().tqb200_engine_prefill_copy_bytes(self.h, C.byref(n)))
        return n.value

    def close(self):
        if getattr(self, "h", None):
            load().tqb200_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
