"""Model cases shared by the golden-fixture generator and the tests."""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))

from tqb200.model import ModelSpec  # noqa: E402

PROMPT = [1, 17, 300, 999, 5, 42]

# (name, spec, kv_fp16, seed)
MODEL_CASES = [
    ("qwen2_bias", ModelSpec(name="qwen2_bias", qkv_bias=True, norm_noise=0.1), False, 11),
    ("qwen3_f16kv", ModelSpec(name="qwen3_f16kv", qk_norm=True, norm_noise=0.1), True, 12),
    ("untied_f32embed", ModelSpec(name="untied", embed_dtype="f32", tied=False, qkv_bias=True),
     False, 13),
    ("vq2_rot", ModelSpec(name="vq2_rot", weight_dtype="vq2", rotated=True, qk_norm=True,
                          hidden=256, inter=512, n_heads=8, head_dim=32), False, 14),
    ("moe", ModelSpec(name="moe", model_type=3, qk_norm=True, n_experts=16, experts_per_tok=4,
                      moe_inter=64, tied=False), False, 15),
]


def model_tokens(m, steps: int = 10):
    """Feed PROMPT then greedy-decode up to `steps` tokens; returns (tokens, logits list)."""
    toks, logits = [], []
    nxt = None
    for i in range(steps):
        t = PROMPT[i] if i < len(PROMPT) else nxt
        nxt = m.step(t)
        toks.append(nxt)
        logits.append(m.logits())
    return toks, logits


# ----------------------------------------------------------------------------
# Seeded op cases.  Inputs are regenerated from the seed by the functions below
# (numpy PCG64); the fixture stores the outputs plus a checksum of the inputs
# so a change in the generator is detected instead of silently compared.
import hashlib  # noqa: E402

import numpy as np  # noqa: E402

from tqb200 import synth  # noqa: E402

I4_CASES = [(64, 256, 128), (64, 256, 64), (32, 200, 64), (33, 200, 48), (96, 384, 64)]
VQ2_CASES = [(32, 128), (96, 384), (33, 200)]
# symmetric W4A8: (rows, cols, weight seed, activation seed) of the reference's sdot5 tests
# (tests/test_matvec_i4.cpp:441-477), inputs drawn by the reference test's random_vec
W4A8_CASES = [(96, 384, 9901, 9902), (512, 896, 9903, 9904)]
BIIP_CASES = [(896, 128, True), (896, 128, False), (4864, 256, True), (256, 64, True),
              (128, 128, False)]
RMS_CASES = [896, 2560, 128]
ROPE_CASES = [(14, 2, 64, 0), (14, 2, 64, 37), (32, 8, 128, 4095), (16, 8, 128, 511)]
ATTN_CASES = [(14, 2, 64, 1, 8), (14, 2, 64, 96, 128), (32, 8, 128, 300, 512), (4, 1, 32, 17, 17)]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _seed(tag: str, *nums) -> np.random.Generator:
    base = int(hashlib.md5(tag.encode()).hexdigest()[:8], 16)
    return np.random.default_rng([base] + [int(n) for n in nums])


def i4_case(M, K, G):
    r = _seed("i4", M, K, G)
    return synth.random_i4(r, M, K, G), r.normal(size=K).astype(np.float32)


def vq2_case(M, K):
    r = _seed("vq2", M, K)
    return synth.random_vq2(r, M, K), r.normal(size=K).astype(np.float32)


def matmul_case():
    r = _seed("mm")
    return synth.random_i4(r, 48, 256, 64), r.normal(size=(5, 256)).astype(np.float32)


def biip_case(dim, bs):
    r = _seed("biip", dim, bs)
    x = r.normal(size=dim).astype(np.float32)
    sign = r.choice(np.array([-1.0, 1.0], np.float32), dim)
    scale = (np.abs(r.normal(size=dim)) + 1e-3).astype(np.float32)
    return x, sign, scale


def rms_case(n):
    r = _seed("rms", n)
    return r.normal(size=n).astype(np.float32), (1 + 0.1 * r.normal(size=n)).astype(np.float32)


def rope_case(H, KVH, hd, pos):
    r = _seed("rope", H, KVH, hd, pos)
    return r.normal(size=H * hd).astype(np.float32), r.normal(size=KVH * hd).astype(np.float32)


def attn_case(H, KVH, hd, seq, maxs):
    r = _seed("attn", H, KVH, hd, seq, maxs)
    q = r.normal(size=H * hd).astype(np.float32)
    kc = r.normal(size=KVH * maxs * hd).astype(np.float32)
    vc = r.normal(size=KVH * maxs * hd).astype(np.float32)
    return q, kc, vc


def swiglu_case():
    r = _seed("swiglu")
    return (r.normal(size=4864) * 4).astype(np.float32), r.normal(size=4864).astype(np.float32)


def argmax_case():
    r = _seed("argmax")
    l = r.normal(size=151936).astype(np.float32)
    l[[7, 90000]] = l.max() + 1.0
    return l


def topk_case():
    r = _seed("topk")
    gl = r.normal(size=128).astype(np.float32)
    gl[[3, 9]] = gl.max() + 0.5
    return gl


def f2h_case():
    r = _seed("f2h")
    vals = np.concatenate([r.normal(size=4000) * np.float32(10.0) ** r.integers(-9, 6, 4000),
                           [65504, 65519, 65520, 65536, 1e-8, 3e-8, 6e-8, -2.9e-8, 5.9604645e-08,
                            2.9802322e-08, 6.1035156e-05, 6.0975552e-05]])
    return vals.astype(np.float32)


# GPTQ-INT4 (rows, cols, group, act-order) and the Qwen3.5 GDN ops
GPTQ_CASES = [(96, 512, 128, False), (64, 256, 64, True), (33, 384, 128, True)]
GDN_CONV = (512, 4)          # channels, kernel size
GDN_HEAD = (128, 128)        # qk_dim, v_dim
PROPE_CASE = (8, 2, 256, 64, 77, 1e7)  # heads, kv heads, head_dim, rotary_dim, pos, theta


def gptq_case(M, K, G, act_order):
    r = _seed("gptq", M, K, G, int(act_order))
    return synth.random_gptq(r, M, K, G, act_order), r.normal(size=K).astype(np.float32)


def gdn_case():
    """l2norm vector, conv (x, state, weight), one head (S, q, k, v, g, beta), gated RMSNorm
    (x, gate, weight), partial RoPE (q, k)."""
    r = _seed("gdn")
    dim, ks = GDN_CONV
    dk, dv = GDN_HEAD
    H, KVH, hd = PROPE_CASE[:3]
    f = lambda *s: r.normal(size=s).astype(np.float32)
    return dict(l2=f(dk), cx=f(dim), cst=f(dim, ks - 1), cw=f(dim, ks) * np.float32(0.5),
                S=f(dk, dv) * np.float32(0.1), q=f(dk), k=f(dk) * np.float32(0.1), v=f(dv),
                g=np.float32(-0.25), beta=np.float32(0.6),
                rx=f(dv), rg=f(dv), rw=(1 + 0.1 * f(dv)).astype(np.float32),
                pq=f(H * hd), pk=f(KVH * hd))
