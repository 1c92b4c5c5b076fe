"""VQ2 codebook matvec and BiIP rotation on the GPU vs the reference's golden
outputs and the oracle.  BiIP is bit-exact (same butterfly order, IEEE
division); the VQ2 dot accumulates in fp32 (reference: double), 1e-4 max
relative error."""
from __future__ import annotations

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.mark.parametrize("M,K", gc.VQ2_CASES + [(3072, 1024), (1024, 3072), (1, 4), (7, 12)])
def test_vq2_vs_oracle(tq, oracle, M, K):
    rng = np.random.default_rng(M + 13 * K)
    w = synth.random_vq2(rng, M, K)
    x = rng.normal(size=K).astype(np.float32)
    assert max_rel(tq.matvec_vq2(w, x, M, K), oracle.matvec_vq2(w, x, M, K)) < TOL


def test_vq2_handcrafted(tq):
    # tests/test_matvec_vq2.cpp:154-166
    cb = np.zeros((256, 4), np.float16)
    cb[5] = 5.0
    w = np.concatenate([cb.view(np.uint8).ravel(), np.array([5], np.uint8)])
    assert tq.matvec_vq2(w, np.ones(4, np.float32), 1, 4)[0] == 20.0


def test_vq2_golden_config3(tq, golden):
    w, x, sign, scale = synth.config3_vq2(0)
    assert max_rel(tq.matvec_vq2(w, x, 3072, 1024), golden["cfg3_y"]) < TOL
    assert np.array_equal(tq.biip_rotate(x, scale, sign, 256), golden["cfg3_rot"])
    fused = tq.matvec_vq2_rot(w, x, 3072, 1024, scale, sign, 256)
    assert max_rel(fused, tq.matvec_vq2(w, golden["cfg3_rot"], 3072, 1024)) < 1e-6


@pytest.mark.parametrize("dim,bs,ws", gc.BIIP_CASES)
def test_biip_bit_exact(tq, golden, dim, bs, ws):
    x, sign, scale = gc.biip_case(dim, bs)
    y = tq.biip_rotate(x, scale if ws else None, sign, bs)
    assert np.array_equal(y, golden[f"biip_{dim}_{bs}_{int(ws)}_y"])


def test_biip_partial_block_tail(tq, oracle):
    # dim not a multiple of the block: the tail keeps (x/scale)*sign (biip_rotate.cpp:50)
    rng = np.random.default_rng(2)
    dim = 200
    x = rng.normal(size=dim).astype(np.float32)
    sign = rng.choice(np.array([-1, 1], np.float32), dim)
    scale = (np.abs(rng.normal(size=dim)) + 1e-3).astype(np.float32)
    assert np.array_equal(tq.biip_rotate(x, scale, sign, 64), oracle.biip_rotate(x, scale, sign, 64))
