"""Synthetic tinyqwen decoders: seeded weights under the reference's tensor names,
a plain-C descriptor for them (include/tqb200_model.h), and a .tqwen writer.

Tensor names and shapes are the ones QwenModel::create binds
(runtime/qwen_model.cpp:438-649).  Weights follow the survey's synthetic recipe:
linear weights N(0, 0.02) quantised by RTN g64 (or drawn directly as codes for
multi-GB timing models), biases N(0, 0.02), a tied compact-i4 embedding used as
lm_head (``lm_head_is_i4_``, runtime/qwen_model.cpp:456-468).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional

import numpy as np

from . import abi
from .synth import (hadamard_block_size, i4_row_bytes, quantize_i4_rtn, random_i4_fast,
                    random_vq2)


@dataclass
class ModelSpec:
    name: str = "tiny"
    model_type: int = abi.MODEL_QWEN2
    n_layers: int = 2
    hidden: int = 128
    inter: int = 256
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 32
    vocab: int = 1000
    group_size: int = 64
    max_seq_len: int = 512
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    n_experts: int = 0
    experts_per_tok: int = 0
    moe_inter: int = 0
    weight_dtype: str = "i4"          # "i4" | "vq2"
    embed_dtype: str = "i4"           # "i4" | "f32" | "f16"
    tied: bool = True                 # lm_head == embed
    qkv_bias: bool = False            # Qwen2
    qk_norm: bool = False             # Qwen3
    rotated: bool = False             # BiIP rotations on every projection input
    router_dtype: str = "f32"         # MoE router matrix dtype
    norm_noise: float = 0.0           # 0 -> norm weights exactly 1 (make_fake_model.py)
    weights: str = "rtn"              # "rtn" (N(0,.02) -> RTN) | "codes" (direct random codes)
    expert_layers: int = 0            # > 0: layer l reuses the expert tensors of layer
                                      # l % expert_layers (host memory of a large MoE model)


# The benchmark configurations' model shapes (Qwen2.5-0.5B, Qwen3-4B, Qwen3-0.6B VQ2,
# Qwen3-30B-A3B); vocab 151936 everywhere.
QWEN25_05B = ModelSpec(name="qwen2.5-0.5b-i4", n_layers=24, hidden=896, inter=4864, n_heads=14,
                       n_kv_heads=2, head_dim=64, vocab=151936, max_seq_len=512, qkv_bias=True)
QWEN3_4B = ModelSpec(name="qwen3-4b-i4", n_layers=36, hidden=2560, inter=9728, n_heads=32,
                     n_kv_heads=8, head_dim=128, vocab=151936, max_seq_len=4096, qk_norm=True)
QWEN3_06B_VQ2 = ModelSpec(name="qwen3-0.6b-vq2", n_layers=28, hidden=1024, inter=3072,
                          n_heads=16, n_kv_heads=8, head_dim=128, vocab=151936,
                          max_seq_len=512, qk_norm=True, weight_dtype="vq2", rotated=True)
QWEN3_30B_A3B = ModelSpec(name="qwen3-30b-a3b-i4", model_type=abi.MODEL_QWEN3_MOE, n_layers=48,
                          hidden=2048, inter=6144, n_heads=32, n_kv_heads=4, head_dim=128,
                          vocab=151936, max_seq_len=1024, qk_norm=True, n_experts=128,
                          experts_per_tok=8, moe_inter=768, tied=False)


@dataclass
class Tensor:
    name: str
    dtype: int
    shape: tuple
    data: np.ndarray          # contiguous bytes/values in the file layout


class SynthModel:
    """Weights in memory plus a ctypes descriptor pointing at them."""

    def __init__(self, spec: ModelSpec, seed: int = 0):
        self.spec = spec
        self.seed = seed
        self.tensors: Dict[str, Tensor] = {}
        self._build()
        self._desc_keep: List[object] = []
        self.desc = self._make_desc()

    # -------------------------------------------------------------- weights
    def _rng(self, idx: int) -> np.random.Generator:
        return np.random.default_rng([self.seed, idx])

    def _quant(self, idx: int, rows: int, cols: int) -> Tensor:
        s = self.spec
        rng = self._rng(idx)
        if s.weight_dtype == "vq2":
            return Tensor("", abi.DT_VQ2, (rows, cols), random_vq2(rng, rows, cols))
        if s.weights == "codes":
            blob = random_i4_fast(rng, rows, cols, s.group_size)
        else:
            w = rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32)
            blob = quantize_i4_rtn(w, s.group_size)
        return Tensor("", abi.DT_I4, (rows, cols), blob)

    def _vec(self, idx: int, n: int, mean: float, sigma: float) -> np.ndarray:
        if sigma == 0.0:
            return np.full(n, mean, dtype=np.float32)
        return (mean + self._rng(idx).normal(0.0, sigma, n)).astype(np.float32)

    def _add(self, name: str, t: Tensor):
        t.name = name
        self.tensors[name] = t

    def _build(self):
        s = self.spec
        H, qd, kvd = s.hidden, s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
        idx = 0

        def nxt():
            nonlocal idx
            idx += 1
            return idx

        # embedding (compact i4 / f32 / f16)
        if s.embed_dtype == "i4":
            sp = replace(s, weight_dtype="i4")
            rng = self._rng(nxt())
            if sp.weights == "codes":
                blob = random_i4_fast(rng, s.vocab, H, s.group_size)
            else:
                blob = quantize_i4_rtn(rng.normal(0.0, 0.02, (s.vocab, H)).astype(np.float32),
                                       s.group_size)
            self._add("model.embed_tokens.weight", Tensor("", abi.DT_I4, (s.vocab, H), blob))
        else:
            e = self._rng(nxt()).normal(0.0, 0.02, (s.vocab, H)).astype(np.float32)
            if s.embed_dtype == "f16":
                self._add("model.embed_tokens.weight",
                          Tensor("", abi.DT_F16, (s.vocab, H), e.astype(np.float16)))
            else:
                self._add("model.embed_tokens.weight", Tensor("", abi.DT_F32, (s.vocab, H), e))
        self._add("model.norm.weight", Tensor("", abi.DT_F32, (H,), self._vec(nxt(), H, 1.0, s.norm_noise)))
        if not s.tied:
            spi = self.spec
            rng = self._rng(nxt())
            if spi.weights == "codes":
                blob = random_i4_fast(rng, s.vocab, H, s.group_size)
            else:
                blob = quantize_i4_rtn(rng.normal(0.0, 0.02, (s.vocab, H)).astype(np.float32),
                                       s.group_size)
            self._add("lm_head.weight", Tensor("", abi.DT_I4, (s.vocab, H), blob))

        for li in range(s.n_layers):
            p = f"model.layers.{li}."
            self._add(p + "input_layernorm.weight",
                      Tensor("", abi.DT_F32, (H,), self._vec(nxt(), H, 1.0, s.norm_noise)))
            self._add(p + "post_attention_layernorm.weight",
                      Tensor("", abi.DT_F32, (H,), self._vec(nxt(), H, 1.0, s.norm_noise)))
            self._add(p + "self_attn.q_proj.weight", self._quant(nxt(), qd, H))
            self._add(p + "self_attn.k_proj.weight", self._quant(nxt(), kvd, H))
            self._add(p + "self_attn.v_proj.weight", self._quant(nxt(), kvd, H))
            self._add(p + "self_attn.o_proj.weight", self._quant(nxt(), H, qd))
            if s.qkv_bias:
                for nm, n in (("q", qd), ("k", kvd), ("v", kvd)):
                    self._add(p + f"self_attn.{nm}_proj.bias",
                              Tensor("", abi.DT_F32, (n,), self._vec(nxt(), n, 0.0, 0.02)))
            if s.qk_norm:
                for nm in ("q", "k"):
                    self._add(p + f"self_attn.{nm}_norm.weight",
                              Tensor("", abi.DT_F32, (s.head_dim,),
                                     self._vec(nxt(), s.head_dim, 1.0, s.norm_noise)))
            if s.model_type == abi.MODEL_QWEN3_MOE:
                if s.router_dtype == "i4":
                    rt = self._quant(nxt(), s.n_experts, H)
                else:
                    # N(0, 1/sqrt(H)) gives router logits ~ N(0, 1) on a unit-RMS input
                    rt = Tensor("", abi.DT_F32, (s.n_experts, H),
                                self._rng(nxt()).normal(0.0, 1.0 / np.sqrt(H), (s.n_experts, H))
                                .astype(np.float32))
                self._add(p + "mlp.gate.weight", rt)
                src = li % s.expert_layers if s.expert_layers > 0 else li
                for e in range(s.n_experts):
                    pe = p + f"mlp.experts.{e}."
                    if src != li:  # the same tensors (bytes) as layer `src`
                        ps = f"model.layers.{src}.mlp.experts.{e}."
                        for nm in ("gate_proj.weight", "up_proj.weight", "down_proj.weight"):
                            self._add(pe + nm, replace(self.tensors[ps + nm]))
                        continue
                    self._add(pe + "gate_proj.weight", self._quant(nxt(), s.moe_inter, H))
                    self._add(pe + "up_proj.weight", self._quant(nxt(), s.moe_inter, H))
                    self._add(pe + "down_proj.weight", self._quant(nxt(), H, s.moe_inter))
            else:
                self._add(p + "mlp.gate_proj.weight", self._quant(nxt(), s.inter, H))
                self._add(p + "mlp.up_proj.weight", self._quant(nxt(), s.inter, H))
                self._add(p + "mlp.down_proj.weight", self._quant(nxt(), H, s.inter))
            if s.rotated:
                for nm, dim in (("self_attn.q_proj", H), ("self_attn.k_proj", H),
                                ("self_attn.v_proj", H), ("self_attn.o_proj", qd),
                                ("mlp.gate_proj", H), ("mlp.up_proj", H),
                                ("mlp.down_proj", s.inter)):
                    rng = self._rng(nxt())
                    sign = rng.choice(np.array([-1.0, 1.0], dtype=np.float32), dim)
                    scale = (np.abs(rng.normal(0.0, 1.0, dim)) + 1e-3).astype(np.float32)
                    self._add(p + nm + ".rot_sign", Tensor("", abi.DT_F32, (dim,), sign))
                    self._add(p + nm + ".rot_scale", Tensor("", abi.DT_F32, (dim,), scale))

    # ------------------------------------------------------------ descriptor
    def _ptr(self, name: Optional[str]):
        if name is None or name not in self.tensors:
            return None
        return self.tensors[name].data.ctypes.data

    def _mat(self, name: str) -> abi.Matrix:
        if name not in self.tensors:
            return abi.Matrix(None, 0, 0, 0)
        t = self.tensors[name]
        return abi.Matrix(t.data.ctypes.data, t.dtype, t.shape[0], t.shape[1])

    def _rot(self, prefix: str, dim: int) -> abi.Rotation:
        if prefix + ".rot_sign" not in self.tensors:
            return abi.Rotation(None, None, 0)
        return abi.Rotation(self._ptr(prefix + ".rot_sign"), self._ptr(prefix + ".rot_scale"),
                            hadamard_block_size(dim))

    def _make_desc(self) -> abi.ModelDesc:
        s = self.spec
        H, qd = s.hidden, s.n_heads * s.head_dim
        layers = (abi.Layer * s.n_layers)()
        for li in range(s.n_layers):
            p = f"model.layers.{li}."
            L = layers[li]
            L.input_ln = self._ptr(p + "input_layernorm.weight")
            L.post_ln = self._ptr(p + "post_attention_layernorm.weight")
            for nm in ("q", "k", "v", "o"):
                setattr(L, f"{nm}_proj", self._mat(p + f"self_attn.{nm}_proj.weight"))
            L.q_bias = self._ptr(p + "self_attn.q_proj.bias")
            L.k_bias = self._ptr(p + "self_attn.k_proj.bias")
            L.v_bias = self._ptr(p + "self_attn.v_proj.bias")
            L.q_norm = self._ptr(p + "self_attn.q_norm.weight")
            L.k_norm = self._ptr(p + "self_attn.k_norm.weight")
            L.gate_proj = self._mat(p + "mlp.gate_proj.weight")
            L.up_proj = self._mat(p + "mlp.up_proj.weight")
            L.down_proj = self._mat(p + "mlp.down_proj.weight")
            L.rot_q = self._rot(p + "self_attn.q_proj", H)
            L.rot_k = self._rot(p + "self_attn.k_proj", H)
            L.rot_v = self._rot(p + "self_attn.v_proj", H)
            L.rot_o = self._rot(p + "self_attn.o_proj", qd)
            L.rot_gate = self._rot(p + "mlp.gate_proj", H)
            L.rot_up = self._rot(p + "mlp.up_proj", H)
            L.rot_down = self._rot(p + "mlp.down_proj", s.inter)
            if s.model_type == abi.MODEL_QWEN3_MOE:
                L.router = self._mat(p + "mlp.gate.weight")
                eg = (abi.Matrix * s.n_experts)()
                eu = (abi.Matrix * s.n_experts)()
                ed = (abi.Matrix * s.n_experts)()
                for e in range(s.n_experts):
                    pe = p + f"mlp.experts.{e}."
                    eg[e] = self._mat(pe + "gate_proj.weight")
                    eu[e] = self._mat(pe + "up_proj.weight")
                    ed[e] = self._mat(pe + "down_proj.weight")
                self._desc_keep += [eg, eu, ed]
                L.expert_gate = C.cast(eg, C.POINTER(abi.Matrix))
                L.expert_up = C.cast(eu, C.POINTER(abi.Matrix))
                L.expert_down = C.cast(ed, C.POINTER(abi.Matrix))
        self._desc_keep.append(layers)
        d = abi.ModelDesc()
        d.model_type = s.model_type
        d.n_layers, d.hidden, d.inter = s.n_layers, H, s.inter
        d.n_heads, d.n_kv_heads, d.head_dim, d.vocab = s.n_heads, s.n_kv_heads, s.head_dim, s.vocab
        d.group_size, d.max_seq_len = s.group_size, s.max_seq_len
        d.rms_eps, d.rope_theta = s.rms_eps, s.rope_theta
        d.n_experts, d.experts_per_tok, d.moe_inter = s.n_experts, s.experts_per_tok, s.moe_inter
        d.embed = self._mat("model.embed_tokens.weight")
        d.lm_head = self._mat("lm_head.weight") if not s.tied else self._mat("model.embed_tokens.weight")
        d.final_norm = self._ptr("model.norm.weight")
        d.layers = C.cast(layers, C.POINTER(abi.Layer))
        return d

    def weight_bytes(self) -> int:
        return sum(t.data.nbytes for t in self.tensors.values())

    # ----------------------------------------------------------- .tqwen file
    def write_tqwen(self, path: str):
        write_tqwen(path, self)


_ALIGN = 64


def _align(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


def write_tqwen(path: str, m: SynthModel):
    """Write a .tqwen v3 file (runtime/tiny_format.h:41-322): 192-byte header with the
    v2 (64 B) and v3 (32 B) extensions in its reserved tail, a table of 120-byte
    entries, then 64-byte aligned tensor payloads."""
    s = m.spec
    file_dtype = abi.DT_VQ2 if s.weight_dtype == "vq2" else abi.DT_I4
    tensors = list(m.tensors.values())
    table_off = 192
    data_off = _align(table_off + 120 * len(tensors))
    offsets = []
    cur = data_off
    for t in tensors:
        offsets.append(cur)
        cur = _align(cur + t.data.nbytes)
    total = offsets[-1] + tensors[-1].data.nbytes if tensors else data_off
    is_moe = s.model_type == abi.MODEL_QWEN3_MOE
    v2 = struct.pack("<7IfII I20s", s.model_type, 0, 0, 0, 0, 0, 0, 0.0, 0, 0, s.group_size,
                     b"\0" * 20)
    v3 = struct.pack("<8I", s.n_experts if is_moe else 0, s.experts_per_tok if is_moe else 0,
                     s.moe_inter if is_moe else 0, 0, 0, 1,
                     s.group_size if is_moe else 0, 0)
    assert len(v2) == 64 and len(v3) == 32
    hdr = struct.pack("<8s2I10I2f4Q", b"TINYQWEN", 3, file_dtype, s.n_layers, s.hidden,
                      s.inter, s.n_heads, s.n_kv_heads, s.head_dim, s.vocab, s.max_seq_len,
                      1 if s.tied else 0, 0, s.rms_eps, s.rope_theta, len(tensors), table_off,
                      data_off, total) + v2 + v3
    assert len(hdr) == 192
    with open(path, "wb") as f:
        f.write(hdr)
        for t, off in zip(tensors, offsets):
            name = t.name.encode()
            assert len(name) <= 64
            shape = list(t.shape) + [0] * (4 - len(t.shape))
            f.write(struct.pack("<64s2I4Q2Q", name, t.dtype, len(t.shape), *shape, off,
                                t.data.nbytes))
        for t, off in zip(tensors, offsets):
            f.seek(off)
            f.write(np.ascontiguousarray(t.data).tobytes())
        f.truncate(total)
