"""i4 matvec family on the GPU vs the oracle (max relative error, as
benchmarks/bench_kernels.cpp:474-479 defines it).  Tolerance 1e-4: the
north-star bound for fp32-accumulating kernels vs the double-accumulating
reference.  Dequantised weights: bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.mark.parametrize("M,K,G", gc.I4_CASES + [(4864, 896, 64), (1, 64, 64), (7, 2560, 64),
                                                 (300, 9728, 64), (129, 4096, 128), (5, 96, 32)])
def test_matvec_i4_vs_oracle(tq, oracle, M, K, G):
    rng = np.random.default_rng(M * 7 + K)
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=K).astype(np.float32)
    y = tq.matvec_i4(w, x, M, K, G)
    assert max_rel(y, oracle.matvec_i4(w, x, M, K, G)) < TOL


def test_matvec_i4_golden_config1(tq, golden):
    w, x = synth.config1_matvec(0)
    assert max_rel(tq.matvec_i4(w, x, 4864, 896, 64), golden["cfg1_y"]) < TOL


def test_matvec_i4_rtn_weights(tq, oracle):
    rng = np.random.default_rng(5)
    w = synth.quantize_i4_rtn(rng.normal(0, 0.02, (512, 2560)).astype(np.float32), 64)
    x = rng.normal(size=2560).astype(np.float32)
    assert max_rel(tq.matvec_i4(w, x, 512, 2560, 64), oracle.matvec_i4(w, x, 512, 2560, 64)) < TOL


def test_pair_and_qkv_match_single(tq, oracle):
    rng = np.random.default_rng(9)
    K, G = 896, 64
    wq, wk, wv = (synth.random_i4(rng, n, K, G) for n in (896, 128, 128))
    x = rng.normal(size=K).astype(np.float32)
    yq, yk, yv = tq.matvec_qkv_i4(wq, wk, wv, x, 896, 128, K, G)
    assert max_rel(yq, oracle.matvec_i4(wq, x, 896, K, G)) < TOL
    assert max_rel(yk, oracle.matvec_i4(wk, x, 128, K, G)) < TOL
    assert max_rel(yv, oracle.matvec_i4(wv, x, 128, K, G)) < TOL
    g1, g2 = synth.random_i4(rng, 4864, K, G), synth.random_i4(rng, 4864, K, G)
    y1, y2 = tq.matvec_pair_i4(g1, g2, x, 4864, K, G)
    assert max_rel(y1, oracle.matvec_i4(g1, x, 4864, K, G)) < TOL
    assert max_rel(y2, oracle.matvec_i4(g2, x, 4864, K, G)) < TOL


@pytest.mark.parametrize("M,K,G", gc.I4_CASES)
def test_dequant_bit_exact(tq, golden, M, K, G):
    w, x = gc.i4_case(M, K, G)
    assert np.array_equal(tq.dequant_i4(w, M, K, G), golden[f"i4_{M}x{K}g{G}_deq"])


def test_symmetric_w4a8_vs_naive(tq, oracle):
    # tests/test_matvec_i4.cpp:441-477: sdot5 vs the symmetric W4A8 naive, abs err < 1e-4
    rng = np.random.default_rng(9901)
    for (M, K) in [(96, 384), (512, 896)]:
        wf = rng.normal(size=(M, K)).astype(np.float32)
        w = synth.quantize_i4_rtn(wf, 64, symmetric=True)
        x = rng.normal(size=K).astype(np.float32)
        y = tq.matvec_i4_sym(w, x, M, K, 64)
        ref = oracle.matvec_i4_w4a8(w, x, M, K, 64)
        assert np.abs(y.astype(np.float64) - ref).max() < 1e-4


@pytest.mark.parametrize("M,K,sw,sx", gc.W4A8_CASES)
def test_symmetric_w4a8_vs_reference_golden(tq, golden, M, K, sw, sx):
    # the reference test's own inputs and checker output (golden from oracle/_ref):
    # tests/test_matvec_i4.cpp:441-477 holds sdot5 to abs err < 1e-4 against it
    key = f"w4a8_{M}x{K}"
    y = tq.matvec_i4_sym(golden[key + "_w"], golden[key + "_x"], M, K, 64)
    assert np.abs(y.astype(np.float64) - golden[key + "_y"]).max() < 1e-4


def _heavy_tailed(rng, K, kind):
    """Activation vectors whose magnitudes span several decades."""
    x = rng.normal(size=K).astype(np.float32)
    if kind == "spikes":        # a few channels 1e3x and 1e4x the rest (outlier channels)
        idx = rng.choice(K, 8, replace=False)
        x[idx[:4]] *= 1e3
        x[idx[4:]] *= 1e4
    elif kind == "swiglu":      # SwiGLU of N(0,3) gate and up: heavy-tailed products
        g, u = rng.normal(0, 3, K), rng.normal(0, 3, K)
        x = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
    elif kind == "tiny_bulk":   # the bulk 1e-4 of a single large channel
        x *= 1e-4
        x[rng.integers(K)] = 1.0
    return x


@pytest.mark.parametrize("kind", ["spikes", "swiglu", "tiny_bulk"])
@pytest.mark.parametrize("M,K", [(2560, 9728), (4096, 2560), (4864, 896)])
def test_matvec_i4_heavy_tailed_activations(tq, oracle, kind, M, K):
    """The kernel's activation digits share one scale per vector (max |x|); inputs
    spanning 4 decades stay within the 1e-4 bound."""
    rng = np.random.default_rng(M + K + len(kind))
    w = synth.random_i4(rng, M, K, 64)
    x = _heavy_tailed(rng, K, kind)
    assert max_rel(tq.matvec_i4(w, x, M, K, 64), oracle.matvec_i4(w, x, M, K, 64)) < TOL


def test_pair_heavy_tailed_activations(tq, oracle):
    rng = np.random.default_rng(77)
    K, M = 2560, 9728
    g1, g2 = synth.random_i4_fast(rng, M, K, 64), synth.random_i4_fast(rng, M, K, 64)
    x = _heavy_tailed(rng, K, "spikes")
    y1, y2 = tq.matvec_pair_i4(g1, g2, x, M, K, 64)
    assert max_rel(y1, oracle.matvec_i4(g1, x, M, K, 64)) < TOL
    assert max_rel(y2, oracle.matvec_i4(g2, x, M, K, 64)) < TOL


@pytest.mark.parametrize("M,K", [(16384, 2560), (20011, 2560), (151936, 2560)])
def test_matvec_i4_multi_pass(tq, oracle, M, K):
    """CTA shares above 100 KB run in several passes (lm_head: 151936 rows, ~1 MB per
    CTA); 20011 rows leave a ragged last pass."""
    rng = np.random.default_rng(M)
    w = synth.random_i4_fast(rng, M, K, 64)
    x = rng.normal(size=K).astype(np.float32)
    assert max_rel(tq.matvec_i4(w, x, M, K, 64), oracle.matvec_i4(w, x, M, K, 64)) < TOL


def test_resident_weight_cache(tq, oracle):
    rng = np.random.default_rng(3)
    w = synth.random_i4(rng, 256, 512, 64)
    x = rng.normal(size=512).astype(np.float32)
    tq.set_resident_weights(True)
    try:
        y1 = tq.matvec_i4(w, x, 256, 512, 64)
        y2 = tq.matvec_i4(w, x, 256, 512, 64)
        assert np.array_equal(y1, y2)
        assert max_rel(y1, oracle.matvec_i4(w, x, 256, 512, 64)) < TOL
    finally:
        tq.set_resident_weights(False)
        tq.clear_resident_weights()


def test_device_pointer_path(tq, oracle):
    import torch
    rng = np.random.default_rng(4)
    M, K, G = 2048, 2560, 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=K).astype(np.float32)
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(M, device="cuda", dtype=torch.float32)
    tq.dev_matvec_i4(dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, G)
    torch.cuda.synchronize()
    assert max_rel(dy.cpu().numpy(), oracle.matvec_i4(w, x, M, K, G)) < TOL


@pytest.mark.parametrize("M,K", [(4864, 896), (2048, 2560)])
def test_pdl_launch_after_producer(tq, oracle, M, K):
    """tqb200_dev_matvec_i4_pdl right after a kernel that writes x: the matvec may start
    early and read its weights, but must read the x that kernel wrote."""
    import torch
    from tqb200 import lib
    rng = np.random.default_rng(M + K)
    G = 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=K).astype(np.float32)
    dw = torch.from_numpy(w).cuda()
    src = torch.from_numpy(x).cuda()
    dx = torch.zeros(K, device="cuda", dtype=torch.float32)
    dy = torch.empty(M, device="cuda", dtype=torch.float32)
    s = torch.cuda.current_stream()
    for _ in range(2):
        dx.zero_()
        torch.cuda.synchronize()
        dx.copy_(src * 1.0)  # a kernel on the stream that produces x
        st = lib.load().tqb200_dev_matvec_i4_pdl(dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), M,
                                                 K, G, s.cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        assert max_rel(dy.cpu().numpy(), oracle.matvec_i4(w, x, M, K, G)) < TOL


@pytest.mark.parametrize("K", [64, 896, 1792])
def test_small_rows_single_pair_qkv(tq, oracle, K):
    """Short rows (one to 28 groups) in single, paired and q/k/v launches, against the
    oracle."""
    rng = np.random.default_rng(K)
    G = 64
    M = 333
    w1, w2, w3 = (synth.random_i4(rng, M, K, G) for _ in range(3))
    x = rng.normal(size=K).astype(np.float32)
    assert max_rel(tq.matvec_i4(w1, x, M, K, G), oracle.matvec_i4(w1, x, M, K, G)) < TOL
    y1, y2 = tq.matvec_pair_i4(w1, w2, x, M, K, G)
    assert max_rel(y1, oracle.matvec_i4(w1, x, M, K, G)) < TOL
    assert max_rel(y2, oracle.matvec_i4(w2, x, M, K, G)) < TOL
    wk = synth.random_i4(rng, 77, K, G)
    wv = synth.random_i4(rng, 77, K, G)
    q, k, v = tq.matvec_qkv_i4(w1, wk, wv, x, M, 77, K, G)
    assert max_rel(q, oracle.matvec_i4(w1, x, M, K, G)) < TOL
    assert max_rel(k, oracle.matvec_i4(wk, x, 77, K, G)) < TOL
    assert max_rel(v, oracle.matvec_i4(wv, x, 77, K, G)) < TOL
