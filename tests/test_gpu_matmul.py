"""Batched i4 matmul (MatmulI4Fn, the prefill / grouped-expert contraction) on the tensor
cores vs the oracle's matmul_i4 (a restatement of matmul_i4_ref,
kernels/matvec/matmul_i4_ref.cpp:53-114: per-column matvec, double accumulation).
Tolerance 1e-4 max relative (the north-star bound for fp32 accumulation); the
reference's own matmul test (tests/test_matvec_i4.cpp:514-536) uses 1e-4 absolute
against matvec_i4 on its 48x128x2 case, which is checked here as well."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import max_rel
from tqb200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4

CASES = [
    (48, 128, 2, 64),      # the reference's own matmul_i4_matches_matvec shape
    (4864, 896, 32, 64),   # config-1 matrix, a prompt's worth of columns
    (768, 2048, 37, 64),   # a config-5 expert gate/up, ragged column count
    (2048, 768, 5, 64),    # a config-5 expert down
    (129, 4096, 17, 128),  # group 128, one row past a tile
    (5, 96, 3, 32),        # group 32, K tail inside the stage
    (100, 200, 9, 64),     # K tail group of 8 columns
    (256, 2560, 300, 64),  # three column tiles, last one partial
    (1, 64, 1, 64),
    (384, 1024, 256, 64),  # exactly two full column tiles
]


@pytest.mark.parametrize("M,K,N,G", CASES)
def test_matmul_i4_vs_oracle(tq, oracle, M, K, N, G):
    rng = np.random.default_rng(M * 31 + K * 7 + N)
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=(N, K)).astype(np.float32)  # column-major X[K, N]
    y = tq.matmul_i4(w, x, M, K, N, G)
    ref = oracle.matmul_i4(w, x, M, K, N, G)
    assert max_rel(y, ref) < TOL
    # every column on its own as well (a column of tiny outputs must not hide)
    for n in range(0, N, max(1, N // 7)):
        assert max_rel(y[n], ref[n]) < TOL


def test_matmul_i4_reference_test_shape_abs(tq, oracle):
    """tests/test_matvec_i4.cpp:514-536: RTN-packed random weights, N = 2, each column
    within 1e-4 (absolute) of matvec_i4 on that column."""
    rng = np.random.default_rng(99)
    M, K, N, G = 48, 128, 2, 64
    w = synth.quantize_i4_rtn(rng.uniform(-1, 1, (M, K)).astype(np.float32), G)
    x = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    y = tq.matmul_i4(w, x, M, K, N, G)
    for n in range(N):
        assert np.abs(y[n] - oracle.matvec_i4(w, x[n], M, K, G)).max() < 1e-4


def test_matmul_i4_vs_reference_build(tq, reflib):
    rng = np.random.default_rng(3)
    M, K, N, G = 300, 1024, 40, 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=(N, K)).astype(np.float32)
    y = tq.matmul_i4(w, x, M, K, N, G)
    assert max_rel(y, reflib.matmul_i4(w, x, M, K, N, G)) < TOL


def test_matmul_i4_large_activations(tq, oracle):
    """Hidden states far from unit scale keep the relative bound (bf16 keeps fp32's range)."""
    rng = np.random.default_rng(11)
    M, K, N, G = 256, 2048, 24, 64
    w = synth.random_i4(rng, M, K, G)
    x = (rng.normal(size=(N, K)) * 300.0).astype(np.float32)
    x[:, ::97] *= 50.0
    assert max_rel(tq.matmul_i4(w, x, M, K, N, G), oracle.matmul_i4(w, x, M, K, N, G)) < TOL


def test_dev_matmul_i4_device_pointers(tq, oracle):
    import torch
    rng = np.random.default_rng(4)
    M, K, N, G = 640, 2048, 48, 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=(N, K)).astype(np.float32)
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((N, M), float("nan"), device="cuda")
    L = tq.load()
    sb = L.tqb200_matmul_i4_scratch_bytes(M, K, N, G)
    scr = torch.empty(sb, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.tqb200_dev_matmul_i4(dw.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, N, G,
                                  scr.data_ptr(), st) == 0
    torch.cuda.synchronize()
    assert max_rel(dy.cpu().numpy(), oracle.matmul_i4(w, x, M, K, N, G)) < TOL
