"""GPTQ-INT4 matvec / matmul, dense f32 / f16 matvec and the Qwen3.5 GDN ops on the GPU,
through the C ABI, against the oracle (pinned to the reference's fixtures in
tests/test_oracle.py) and the reference's golden outputs.

Bars: GPTQ and dense matvecs max relative error 1e-4 (fp32 accumulation against the
reference's double sums); the GDN ops with fp32 sums in the reference's order bit-exact
(gdn_step, partial RoPE, the conv state) or within a few ulp where CUDA's expf enters
(SiLU in conv1d and the gated RMSNorm) or a double sum is associated differently
(l2norm)."""
from __future__ import annotations

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4
ULPS = 4e-7  # a few float ulp, relative to the vector's largest magnitude


@pytest.mark.parametrize("M,K,G,ao", gc.GPTQ_CASES + [(4864, 896, 128, False), (2048, 4096, 128, True),
                                                      (1, 64, 64, False)])
def test_matvec_gptq_vs_oracle(tq, oracle, golden, M, K, G, ao):
    rng = np.random.default_rng(M + K + G)
    w = synth.random_gptq(rng, M, K, G, ao)
    x = rng.normal(size=K).astype(np.float32)
    assert max_rel(tq.matvec_gptq(w, x, M, K, G), oracle.matvec_gptq(w, x, M, K, G)) < TOL
    key = f"gptq_{M}x{K}g{G}_{int(ao)}"
    if key + "_y" in golden:
        w, x = gc.gptq_case(M, K, G, ao)
        assert max_rel(tq.matvec_gptq(w, x, M, K, G), golden[key + "_y"]) < TOL


def test_matmul_gptq_columns(tq, oracle):
    rng = np.random.default_rng(3)
    M, K, N, G = 512, 1024, 5, 128
    w = synth.random_gptq(rng, M, K, G, True)
    X = rng.normal(size=(N, K)).astype(np.float32)
    assert max_rel(tq.matmul_gptq(w, X, M, K, N, G), oracle.matmul_gptq(w, X, M, K, N, G)) < TOL


def test_gptq_rejects_bad_group(tq):
    w = np.zeros(8 + 2 * 4 * 64 * 2 + 60 * 64 * 4, np.uint8)
    with pytest.raises(tq.TQB200Error):
        tq.matvec_gptq(w, np.zeros(100, np.float32), 64, 100, 25)


@pytest.mark.parametrize("M,K", [(128, 2048), (37, 100), (151, 1024)])
def test_dense_matvec_vs_oracle(tq, oracle, M, K):
    rng = np.random.default_rng(M * K)
    w = rng.normal(0, 0.02, (M, K)).astype(np.float32)
    x = rng.normal(size=K).astype(np.float32)
    assert max_rel(tq.matvec_f32(w, x), oracle.matvec_f32(w, x)) < TOL
    w16 = w.astype(np.float16).view(np.uint16)
    y16 = tq.matvec_f16(w16, x)
    exp16 = (w16.view(np.float16).astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    assert max_rel(y16, exp16) < TOL


def test_gdn_ops_vs_reference_golden(tq, oracle, golden):
    c = gc.gdn_case()
    rel = lambda a, b: float(np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30))
    assert rel(tq.l2norm_inplace(c["l2"], 1e-6), golden["gdn_l2"]) <= ULPS
    dim, ks = gc.GDN_CONV
    out, st = tq.causal_conv1d_update(c["cx"], c["cst"], c["cw"], dim, ks)
    assert np.array_equal(st, golden["gdn_conv_state"])
    assert rel(out, golden["gdn_conv_out"]) <= ULPS
    dk, dv = gc.GDN_HEAD
    o, S = tq.gdn_step(c["S"], c["q"], c["k"], c["v"], float(c["g"]), float(c["beta"]), dk, dv)
    assert np.array_equal(S, golden["gdn_step_S"]) and np.array_equal(o, golden["gdn_step_o"])
    assert rel(tq.rmsnorm_gated(c["rx"], c["rg"], c["rw"], 1e-6), golden["gdn_rmsg"]) <= ULPS
    H, KVH, hd, rd, pos, theta = gc.PROPE_CASE
    q, k = tq.partial_rope(c["pq"], c["pk"], H, KVH, hd, rd, pos, theta)
    assert np.array_equal(q, golden["prope_q"]) and np.array_equal(k, golden["prope_k"])


@pytest.mark.parametrize("dk,dv", [(128, 128), (64, 256), (100, 512), (16, 7), (200, 64)])
def test_gdn_step_shapes_bit_exact(tq, oracle, dk, dv):
    rng = np.random.default_rng(dk * 1000 + dv)
    S = (rng.normal(size=(dk, dv)) * 0.1).astype(np.float32)
    q, k = rng.normal(size=dk).astype(np.float32), (rng.normal(size=dk) * 0.1).astype(np.float32)
    v = rng.normal(size=dv).astype(np.float32)
    o, S2 = tq.gdn_step(S, q, k, v, -0.7, 0.3, dk, dv)
    oo, OS = oracle.gdn_step(S, q, k, v, -0.7, 0.3, dk, dv)
    assert np.array_equal(S2, OS) and np.array_equal(o, oo)


def test_gdn_step_rejects_wide_values(tq):
    with pytest.raises(tq.TQB200Error):
        tq.gdn_step(np.zeros((4, 600), np.float32), np.zeros(4), np.zeros(4), np.zeros(600), 0.0, 1.0,
                    4, 600)


def test_dev_gdn_step_many_heads(tq, oracle):
    """The device-pointer form runs all heads of a layer in one launch."""
    import torch
    nh, dk, dv = 16, 128, 128
    rng = np.random.default_rng(16)
    S = (rng.normal(size=(nh, dk, dv)) * 0.1).astype(np.float32)
    q = rng.normal(size=(nh, dk)).astype(np.float32)
    k = (rng.normal(size=(nh, dk)) * 0.1).astype(np.float32)
    v = rng.normal(size=(nh, dv)).astype(np.float32)
    g = (-np.abs(rng.normal(size=nh))).astype(np.float32)
    beta = rng.uniform(0, 1, nh).astype(np.float32)
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.argtypes, libm.expf.restype = [ctypes.c_float], ctypes.c_float
    dec = np.array([libm.expf(float(x)) for x in g], np.float32)  # the host libm, as the oracle
    t = {n: torch.from_numpy(a).cuda() for n, a in dict(S=S, q=q, k=k, v=v, d=dec, b=beta).items()}
    o = torch.zeros(nh, dv, device="cuda")
    L = tq.load()
    st = L.tqb200_dev_gdn_step(t["S"].data_ptr(), t["q"].data_ptr(), t["k"].data_ptr(),
                               t["v"].data_ptr(), t["d"].data_ptr(), t["b"].data_ptr(),
                               o.data_ptr(), nh, dk, dv, None)
    assert st == 0, L.tqb200_last_error()
    torch.cuda.synchronize()
    for h in range(nh):
        oo, OS = oracle.gdn_step(S[h], q[h], k[h], v[h], float(g[h]), float(beta[h]), dk, dv)
        assert np.array_equal(t["S"][h].cpu().numpy(), OS)
        assert np.array_equal(o[h].cpu().numpy(), oo)
