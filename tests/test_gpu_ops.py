"""Decode ops on the GPU vs the oracle (rmsnorm, rope, attention fp32/fp16 KV,
swiglu, argmax, top-k softmax).  Bars: rmsnorm bit-exact up to the double
reduction order (<= 1 ulp); ops that call expf/powf/cosf/sinf within a few
ulp (CUDA libm vs glibc); argmax and top-k indices exact."""
from __future__ import annotations

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel

pytestmark = pytest.mark.gpu


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.mark.parametrize("n", gc.RMS_CASES + [1, 9728])
def test_rmsnorm(tq, oracle, n):
    rng = np.random.default_rng(n)
    x = rng.normal(size=n).astype(np.float32) * 3
    w = (1 + 0.1 * rng.normal(size=n)).astype(np.float32)
    assert ulp_diff(tq.rmsnorm(x, w, 1e-6), oracle.rmsnorm(x, w, 1e-6)).max() <= 1


@pytest.mark.parametrize("H,KVH,hd,pos", gc.ROPE_CASES)
def test_rope(tq, golden, H, KVH, hd, pos):
    q, k = gc.rope_case(H, KVH, hd, pos)
    qo, ko = tq.rope(q, k, H, KVH, hd, pos, 1e6)
    key = f"rope_{H}_{KVH}_{hd}_{pos}"
    # bit-exact: the cos/sin row is the reference's own powf/cosf/sinf values
    assert np.array_equal(qo, golden[key + "_qo"]) and np.array_equal(ko, golden[key + "_ko"])


@pytest.mark.parametrize("H,KVH,hd,seq,maxs", gc.ATTN_CASES + [(32, 8, 128, 4096, 4096),
                                                              (14, 2, 64, 3, 512)])
def test_attention_fp32_kv(tq, oracle, H, KVH, hd, seq, maxs):
    q, kc, vc = gc.attn_case(H, KVH, hd, seq, maxs)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    out = tq.attention_decode(q, kc, vc, seq, maxs, H, KVH, hd, scale)
    assert max_rel(out, oracle.attention(q, kc, vc, seq, maxs, H, KVH, hd, scale)) < 1e-5


@pytest.mark.parametrize("H,KVH,hd,seq,maxs", [(32, 8, 128, 4095, 4096), (32, 8, 128, 77, 4096),
                                              (8, 2, 64, 301, 512), (28, 4, 64, 333, 512),
                                              (16, 8, 128, 1000, 1024), (8, 8, 32, 5, 64)])
def test_attention_fp16_kv(tq, oracle, H, KVH, hd, seq, maxs):
    # the reference's fp16-KV check: store halves, decode, attention_decode_ref
    # (tests/test_attention.cpp:192-226); shapes with partial tiles and groups of 1-8 heads
    q, kc, vc = gc.attn_case(H, KVH, hd, seq, maxs)
    k16, v16 = kc.astype(np.float16).view(np.uint16), vc.astype(np.float16).view(np.uint16)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    out = tq.attention_decode_f16kv(q, k16, v16, seq, maxs, H, KVH, hd, scale)
    ref = oracle.attention_f16kv(q, k16, v16, seq, maxs, H, KVH, hd, scale)
    assert max_rel(out, ref) < 1e-5


def test_attention_known_answer(tq):
    # tests/test_attention.cpp:62-73 (two positions, hand-computed)
    out = tq.attention_decode(np.array([1, 0], np.float32), np.array([1, 0, 0, 1], np.float32),
                              np.array([1, 0, 0, 1], np.float32), 2, 2, 1, 1, 2, 1.0)
    e = np.e
    np.testing.assert_allclose(out, [e / (e + 1), 1 / (e + 1)], atol=1e-6)


def test_swiglu(tq, golden):
    g, u = gc.swiglu_case()
    assert ulp_diff(tq.swiglu(g, u), golden["swiglu_y"]).max() <= 4


def test_argmax(tq, golden):
    assert tq.argmax(gc.argmax_case()) == int(golden["argmax_i"][0]) == 7
    assert tq.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    rng = np.random.default_rng(0)
    for n in (1, 31, 1000, 151936):
        l = rng.normal(size=n).astype(np.float32)
        assert tq.argmax(l) == int(np.argmax(l))


def test_topk_softmax(tq, oracle):
    rng = np.random.default_rng(1)
    for n, k in [(128, 8), (16, 4), (60, 8), (5, 8)]:
        l = rng.normal(size=n).astype(np.float32)
        idx, w = tq.topk_softmax(l, k)
        ridx, rw = oracle.topk_softmax(l, k)
        assert np.array_equal(idx, ridx)
        assert ulp_diff(w, rw).max() <= 1
