"""Generate tests/golden/golden_ref.npz from the reference's own CPU code.

Runs the reference's kernels and QwenModel::forward_token, compiled from the
reference tree by oracle/Makefile into oracle/_ref/libtqref.so, on the seeded
inputs of golden_cases.py, and stores the outputs with a checksum of the
inputs.  The fixtures pin the C restatement in oracle/ (tests/test_oracle.py)
and, through it, the CUDA path.  Re-run with:

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))

from oracle.oracle import RefLib  # noqa: E402
from tqb200 import synth  # noqa: E402
from tqb200.model import SynthModel  # noqa: E402

import golden_cases as gc  # noqa: E402


def _s(h: str) -> np.ndarray:
    return np.frombuffer(h.encode(), np.uint8)


def main():
    ref = RefLib()
    out = {}
    for (M, K, G) in gc.I4_CASES:
        w, x = gc.i4_case(M, K, G)
        k = f"i4_{M}x{K}g{G}"
        out[k + "_sha"] = _s(gc.sha(w, x))
        out[k + "_y"] = ref.matvec_i4(w, x, M, K, G)
        out[k + "_deq"] = ref.dequant_i4(w, M, K, G)
    w, x = synth.config1_matvec(0)
    out["cfg1_sha"] = _s(gc.sha(w, x))
    out["cfg1_y"] = ref.matvec_i4(w, x, 4864, 896, 64)
    w, X = gc.matmul_case()
    out["mm_sha"] = _s(gc.sha(w, X))
    out["mm_y"] = ref.matmul_i4(w, X, 48, 256, 5, 64)
    for (M, K) in gc.VQ2_CASES:
        w, x = gc.vq2_case(M, K)
        out[f"vq2_{M}x{K}_sha"] = _s(gc.sha(w, x))
        out[f"vq2_{M}x{K}_y"] = ref.matvec_vq2(w, x, M, K)
    w, x, sign, scale = synth.config3_vq2(0)
    out["cfg3_sha"] = _s(gc.sha(w, x, sign, scale))
    out["cfg3_y"] = ref.matvec_vq2(w, x, 3072, 1024)
    out["cfg3_rot"] = ref.biip_rotate(x, scale, sign, 256)
    for (dim, bs, ws) in gc.BIIP_CASES:
        x, sign, scale = gc.biip_case(dim, bs)
        k = f"biip_{dim}_{bs}_{int(ws)}"
        out[k + "_sha"] = _s(gc.sha(x, sign, scale))
        out[k + "_y"] = ref.biip_rotate(x, scale if ws else None, sign, bs)
    for n in gc.RMS_CASES:
        x, wt = gc.rms_case(n)
        out[f"rms_{n}_sha"] = _s(gc.sha(x, wt))
        out[f"rms_{n}_y"] = ref.rmsnorm(x, wt, 1e-6)
    for (H, KVH, hd, pos) in gc.ROPE_CASES:
        q, k = gc.rope_case(H, KVH, hd, pos)
        qo, ko = ref.rope(q, k, H, KVH, hd, pos, 1e6)
        key = f"rope_{H}_{KVH}_{hd}_{pos}"
        out[key + "_sha"] = _s(gc.sha(q, k))
        out[key + "_qo"], out[key + "_ko"] = qo, ko
    for (H, KVH, hd, seq, maxs) in gc.ATTN_CASES:
        q, kc, vc = gc.attn_case(H, KVH, hd, seq, maxs)
        key = f"attn_{H}_{KVH}_{hd}_{seq}_{maxs}"
        out[key + "_sha"] = _s(gc.sha(q, kc, vc))
        out[key + "_o"] = ref.attention(q, kc, vc, seq, maxs, H, KVH, hd,
                                        float(np.float32(1.0) / np.sqrt(np.float32(hd))))
    # symmetric W4A8 ("sdot5"): the reference test's own inputs, symmetric packer and
    # checker (tests/test_matvec_i4.cpp:441-477 use these seeds and shapes)
    for (M, K, sw, sx) in gc.W4A8_CASES:
        w = ref.pack_i4_rtn_symmetric(ref.random_vec(M * K, sw), M, K, 64)
        x = ref.random_vec(K, sx)
        key = f"w4a8_{M}x{K}"
        out[key + "_w"], out[key + "_x"] = w, x
        out[key + "_y"] = ref.matvec_i4_w4a8_naive(w, x, M, K, 64)
    # GPTQ-INT4 and the Qwen3.5 GDN ops (kernels/matvec/matvec_gptq_ref.cpp, kernels/gdn/)
    for (M, K, G, ao) in gc.GPTQ_CASES:
        w, x = gc.gptq_case(M, K, G, ao)
        key = f"gptq_{M}x{K}g{G}_{int(ao)}"
        out[key + "_sha"] = _s(gc.sha(w, x))
        out[key + "_y"] = ref.matvec_gptq(w, x, M, K, G)
    c = gc.gdn_case()
    out["gdn_sha"] = _s(gc.sha(*[np.asarray(v) for v in c.values()]))
    out["gdn_l2"] = ref.l2norm_inplace(c["l2"], 1e-6)
    dim, ks = gc.GDN_CONV
    out["gdn_conv_out"], out["gdn_conv_state"] = ref.causal_conv1d_update(c["cx"], c["cst"], c["cw"],
                                                                          dim, ks)
    dk, dv = gc.GDN_HEAD
    out["gdn_step_o"], out["gdn_step_S"] = ref.gdn_step(c["S"], c["q"], c["k"], c["v"], float(c["g"]),
                                                        float(c["beta"]), dk, dv)
    out["gdn_rmsg"] = ref.rmsnorm_gated(c["rx"], c["rg"], c["rw"], 1e-6)
    H, KVH, hd, rd, pos, theta = gc.PROPE_CASE
    out["prope_q"], out["prope_k"] = ref.partial_rope(c["pq"], c["pk"], H, KVH, hd, rd, pos, theta)
    g, u = gc.swiglu_case()
    out["swiglu_sha"], out["swiglu_y"] = _s(gc.sha(g, u)), ref.swiglu(g, u)
    l = gc.argmax_case()
    out["argmax_sha"], out["argmax_i"] = _s(gc.sha(l)), np.array([ref.argmax(l)], np.int32)
    gl = gc.topk_case()
    out["topk_sha"] = _s(gc.sha(gl))
    out["topk_i"], out["topk_w"] = ref.topk_softmax(gl, 8)
    out["topk5_i"], out["topk5_w"] = ref.topk_softmax(gl[:5], 8)
    v = gc.f2h_case()
    out["f2h_sha"], out["f2h_h"] = _s(gc.sha(v)), ref.float_to_half(v)

    with tempfile.TemporaryDirectory() as td:
        for name, spec, kv16, seed in gc.MODEL_CASES:
            sm = SynthModel(spec, seed=seed)
            path = os.path.join(td, name + ".tqwen")
            sm.write_tqwen(path)
            rm = ref.open_model(path, 64, spec.vocab, kv16)
            toks, logits = gc.model_tokens(rm, steps=10)
            out[f"model_{name}_tokens"] = np.array(toks, np.int32)
            out[f"model_{name}_logits_last"] = logits[-1]
            out[f"model_{name}_logits_sha"] = _s(gc.sha(np.stack(logits)))
            out[f"model_{name}_weights_sha"] = _s(gc.sha(*[t.data for t in sm.tensors.values()]))
            rm.close()

    path = os.path.join(HERE, "golden_ref.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes,", len(out), "arrays")


if __name__ == "__main__":
    main()
