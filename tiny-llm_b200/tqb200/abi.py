"""ctypes mirrors of include/tqb200_model.h (plain-C model description)."""
from __future__ import annotations

import ctypes as C

DT_F32 = 0
DT_F16 = 1
DT_I4 = 3
DT_VQ2 = 4

MODEL_QWEN2 = 0
MODEL_QWEN3_MOE = 3


class Matrix(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int), ("rows", C.c_int), ("cols", C.c_int)]


class Rotation(C.Structure):
    _fields_ = [("sign", C.c_void_p), ("scale", C.c_void_p), ("block_size", C.c_int)]


class Layer(C.Structure):
    _fields_ = [
        ("input_ln", C.c_void_p), ("post_ln", C.c_void_p),
        ("q_proj", Matrix), ("k_proj", Matrix), ("v_proj", Matrix), ("o_proj", Matrix),
        ("q_bias", C.c_void_p), ("k_bias", C.c_void_p), ("v_bias", C.c_void_p),
        ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
        ("gate_proj", Matrix), ("up_proj", Matrix), ("down_proj", Matrix),
        ("rot_q", Rotation), ("rot_k", Rotation), ("rot_v", Rotation), ("rot_o", Rotation),
        ("rot_gate", Rotation), ("rot_up", Rotation), ("rot_down", Rotation),
        ("router", Matrix),
        ("expert_gate", C.POINTER(Matrix)), ("expert_up", C.POINTER(Matrix)),
        ("expert_down", C.POINTER(Matrix)),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("model_type", C.c_int), ("n_layers", C.c_int), ("hidden", C.c_int), ("inter", C.c_int),
        ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int),
        ("group_size", C.c_int), ("max_seq_len", C.c_int),
        ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("n_experts", C.c_int), ("experts_per_tok", C.c_int), ("moe_inter", C.c_int),
        ("embed", Matrix), ("lm_head", Matrix), ("final_norm", C.c_void_p),
        ("layers", C.POINTER(Layer)),
    ]
