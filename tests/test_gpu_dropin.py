"""The drop-in boundary itself: the reference's own decode loop
(QwenModel::forward_token and the GPU decode registry), built from the reference
sources with tiny-llm_b200/host/b200_variants.cpp registered, run three ways on the
same .tqwen file: reference CPU kernels, the "b200" per-op variants inside
forward_token (--matvec-impl b200 --ops-impl b200), and the "b200" whole-step
engine (--engine b200).  Greedy tokens must be identical.  The checker binary is
built where the reference tree exists (tiny-llm_b200/host/Makefile); the test is
skipped where it was not built."""
from __future__ import annotations

import os
import subprocess

import pytest

import golden_cases as gc
from tqb200.model import SynthModel

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tiny-llm_b200", "host", "_build", "drop_in_check")


@pytest.mark.parametrize("case", [c for c in gc.MODEL_CASES if c[0] in ("qwen2_bias", "vq2_rot")],
                         ids=lambda c: c[0])
def test_reference_decode_loop_with_b200_variants(tmp_path, case):
    if not os.path.exists(BIN):
        pytest.skip("drop_in_check not built (needs the reference tree at build time)")
    name, spec, kv16, seed = case
    path = str(tmp_path / f"{name}.tqwen")
    SynthModel(spec, seed=seed).write_tqwen(path)
    args = ["64", "6"] + [str(t) for t in gc.PROMPT]
    run = lambda mode: subprocess.run([BIN, path, mode] + args, capture_output=True, text=True,
                                      timeout=300)
    ref = run("ref")
    assert ref.returncode == 0, ref.stderr
    ops = run("ops")
    assert ops.returncode == 0, ops.stderr
    assert ops.stdout.split() == ref.stdout.split()
    eng = run("engine")
    assert eng.returncode == 0, eng.stderr
    assert eng.stdout.split() == ref.stdout.split()
    be = run("backend")  # every IBackend op on the GPU (create_b200_backend)
    assert be.returncode == 0, be.stderr
    assert be.stdout.split() == ref.stdout.split()


@pytest.mark.parametrize("case", [c for c in gc.MODEL_CASES if c[0] in ("qwen3_f16kv", "moe")],
                         ids=lambda c: c[0])
def test_reference_forward_token_on_b200_backend_f16kv(tmp_path, tq, oracle, case):
    """QwenModel::forward_token with its fp16 KV cache (--kv-f16) on the b200 IBackend: the
    attention goes through IBackend::attention_decode_f16kv (runtime/backend.h:246-249),
    which the reference's x86 CPU backend cannot run.  Greedy tokens identical to the
    b200 engine with an fp16 cache and to the oracle (the reference's method for fp16-KV
    attention on x86, tests/test_attention.cpp:192)."""
    if not os.path.exists(BIN):
        pytest.skip("drop_in_check not built (needs the reference tree at build time)")
    name, spec, _, seed = case
    sm = SynthModel(spec, seed=seed)
    path = str(tmp_path / f"{name}.tqwen")
    sm.write_tqwen(path)
    n_new = 8
    r = subprocess.run([BIN, path, "backend-f16kv", "64", str(n_new)] + [str(t) for t in gc.PROMPT],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = [int(t) for t in r.stdout.split()]
    eng = tq.Engine(sm, max_seq_len=64, kv_fp16=True)
    om = oracle.model(sm, 64, True)
    exp_e, exp_o = [], []
    ne = no = None
    for i in range(len(gc.PROMPT) + n_new - 1):
        t = gc.PROMPT[i] if i < len(gc.PROMPT) else ne
        to = gc.PROMPT[i] if i < len(gc.PROMPT) else no
        ne, no = eng.step(t), om.step(to)
        exp_e.append(ne)
        exp_o.append(no)
    eng.close()
    om.close()
    assert got == exp_e == exp_o, (got, exp_e, exp_o)


def test_reference_matmul_dispatch_reaches_b200(tmp_path, oracle):
    """tinyqwen::matmul_i4 (the prefill contraction, QwenModel::mm ->
    CPUBackend::matmul) through the reference's own dispatcher lands on the b200
    variant (it has no by-name selector; the first registration is current) and
    matches the oracle's matmul_i4_ref restatement."""
    if not os.path.exists(BIN):
        pytest.skip("drop_in_check not built (needs the reference tree at build time)")
    import numpy as np
    from conftest import max_rel
    from tqb200 import synth
    rng = np.random.default_rng(21)
    M, K, N, G = 768, 2048, 29, 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=(N, K)).astype(np.float32)
    path = str(tmp_path / "mm.bin")
    with open(path, "wb") as f:
        f.write(w.tobytes())
        f.write(x.tobytes())
    r = subprocess.run([BIN, path, "matmul", str(M), str(K), str(N), str(G)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "b200 matmul calls 1" in r.stdout
    y = np.fromfile(path + ".y", np.float32).reshape(N, M)
    assert max_rel(y, oracle.matmul_i4(w, x, M, K, N, G)) < 1e-4
