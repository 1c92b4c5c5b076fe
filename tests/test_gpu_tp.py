"""Tensor-parallel engine (tp_size 2, one process per GPU; MoE layers expert-parallel)
against the single-GPU oracle: identical greedy tokens and logits within 1e-4 on every
rank, with the activations all-gathered over NCCL and with the peer exchange (the
all-gathers fused into the producing kernels over NVLink; i4 models).  Needs two visible
GPUs (skipped otherwise)."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200.model import SynthModel

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
# "moe": attention sharded as in the dense cases, experts split across the ranks (expert
# parallelism: 8 of the 16 experts per rank, a cross-rank sum of the chosen experts' slots)
TP_CASES = [c for c in gc.MODEL_CASES if c[0] in ("qwen2_bias", "qwen3_f16kv", "vq2_rot", "moe")]


MODES = [(c, m) for c in TP_CASES for m in ("nccl", "p2p") if not (m == "p2p" and c[0] == "vq2_rot")]


def _run_ranks(tq, tmp_path, name, mode, extra=()):
    world = 2
    nid = tq.nccl_unique_id().hex()
    outs = [str(tmp_path / f"r{r}.npz") for r in range(world)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), str(r),
                               str(world), nid, name, outs[r], mode, str(tmp_path), *extra],
                              env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=240)[0])
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail("tensor-parallel ranks did not finish")
    assert all(p.returncode == 0 for p in procs), logs
    return [np.load(o) for o in outs]


@pytest.mark.parametrize("mode", ["nccl", "p2p"])
def test_tp2_moe_batched_prefill_matches_oracle(tq, oracle, tmp_path, mode):
    """Expert-parallel MoE (attention whole on every rank, 8 of the 16 experts per rank):
    a 45-token prompt as one batched prefill (grouped tensor-core GEMM over the rank's
    experts, a cross-rank sum of the expert rows), then 8 greedy steps, against the oracle
    fed token by token."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import tp_worker
    name, spec, kv16, seed = tp_worker.PF_CASE
    outs = _run_ranks(tq, tmp_path, name, mode, ("prefill",))
    om = oracle.model(SynthModel(spec, seed=seed), 64, kv16)
    nxt = None
    for t in tp_worker.prefill_prompt(spec.vocab):
        nxt = om.step(t)
    otoks, ologits = [nxt], [om.logits()]
    for _ in range(8):
        nxt = om.step(nxt)
        otoks.append(nxt)
        ologits.append(om.logits())
    for r, d in enumerate(outs):
        assert list(d["tokens"]) == otoks, (r, list(d["tokens"]), otoks)
        for a, b in zip(d["logits"], ologits):
            assert max_rel(a, b) < 1e-4


@pytest.mark.parametrize("case,mode", MODES, ids=[f"{c[0]}-{m}" for c, m in MODES])
def test_tp2_engine_matches_oracle(tq, oracle, tmp_path, case, mode):
    import torch
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    name, spec, kv16, seed = case
    nid = tq.nccl_unique_id().hex()
    outs = [str(tmp_path / f"r{r}.npz") for r in range(world)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), str(r),
                               str(world), nid, name, outs[r], mode, str(tmp_path)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=240)[0])
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail("tensor-parallel ranks did not finish")
    assert all(p.returncode == 0 for p in procs), logs
    om = oracle.model(SynthModel(spec, seed=seed), 64, kv16)
    otoks, ologits = gc.model_tokens(om, steps=10)
    for r in range(world):
        d = np.load(outs[r])
        assert list(d["tokens"]) == otoks, (r, list(d["tokens"]), otoks)
        for a, b in zip(d["logits"], ologits):
            assert max_rel(a, b) < 1e-4
