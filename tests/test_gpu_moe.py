"""MoE decode (Qwen3-MoE family, BASELINE config 5 decode) on the GPU engine vs the
reference's golden tokens and the oracle's forward_token restatement
(runtime/qwen_forward_token.cpp:478-631: router over the post-attention RMSNorm, top-k
softmax, each chosen expert's gate/up -> SwiGLU -> down, weighted sum in router order,
residual).  Bars: greedy tokens identical, logits within max relative error 1e-4."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200 import abi
from tqb200.model import QWEN3_30B_A3B, ModelSpec, SynthModel

pytestmark = pytest.mark.gpu
TOL = 1e-4
MOE = [c for c in gc.MODEL_CASES if c[0] == "moe"][0]


@pytest.mark.parametrize("graph", [True, False])
def test_moe_engine_matches_reference_golden(tq, oracle, golden, graph):
    name, spec, kv16, seed = MOE
    sm = SynthModel(spec, seed=seed)
    eng = tq.Engine(sm, max_seq_len=64, kv_fp16=kv16, use_graph=graph)
    om = oracle.model(sm, 64, kv16)
    toks, logits = gc.model_tokens(eng, steps=10)
    otoks, ologits = gc.model_tokens(om, steps=10)
    assert toks == list(golden[f"model_{name}_tokens"]) == otoks
    for a, b in zip(logits, ologits):
        assert max_rel(a, b) < TOL
    eng.close()


def test_moe_engine_i4_router(tq, oracle):
    """A quantised (i4) router takes the i4 matvec + top-k path instead of the f32 one."""
    spec = replace(MOE[1], router_dtype="i4", n_experts=32, experts_per_tok=8, moe_inter=128)
    sm = SynthModel(spec, seed=21)
    eng = tq.Engine(sm, max_seq_len=32)
    om = oracle.model(sm, 32, False)
    toks, logits = gc.model_tokens(eng, steps=8)
    otoks, ologits = gc.model_tokens(om, steps=8)
    assert toks == otoks
    for a, b in zip(logits, ologits):
        assert max_rel(a, b) < TOL
    eng.close()


def test_moe_engine_config5_shape(tq, oracle):
    """BASELINE config 5 layer shapes (hidden 2048, 128 experts, top-8, expert inter 768,
    32/4 heads of 128, vocab 151936) over 2 layers: every expert matrix of a layer is
    resident and the device picks 8 of them per token."""
    spec = replace(QWEN3_30B_A3B, n_layers=2, max_seq_len=64, weights="codes")
    sm = SynthModel(spec, seed=5)
    eng = tq.Engine(sm, max_seq_len=64)
    om = oracle.model(sm, 64, False)
    prompt = [3, 1999, 77, 151000]
    worst, toks, otoks = 0.0, [], []
    nxt = onxt = None
    for i in range(len(prompt) + 4):
        t = prompt[i] if i < len(prompt) else nxt
        ot = prompt[i] if i < len(prompt) else onxt
        nxt, onxt = eng.step(t), om.step(ot)
        worst = max(worst, max_rel(eng.logits(), om.logits()))
        toks.append(nxt)
        otoks.append(onxt)
    eng.close()
    om.close()
    assert toks == otoks
    assert worst < TOL


def test_moe_engine_profile_kinds(tq):
    sm = SynthModel(MOE[1], seed=MOE[3])
    eng = tq.Engine(sm, max_seq_len=16)
    eng.step(1)
    _, prof = eng.profile_step(2)
    assert prof["router"] > 0 and prof["moe_combine"] > 0 and prof["gate_up"] > 0
    eng.close()


def test_moe_engine_multi_pass_expert_blocks(tq, oracle):
    """Expert blocks larger than one pass: top-2 of 8 experts with intermediate 4096, so
    a CTA's share of the paired gate/up rows exceeds 100 KB and its passes (of a row
    count dividing the 4096-row block) must not straddle two experts' blocks."""
    spec = ModelSpec(name="moe-wide", model_type=abi.MODEL_QWEN3_MOE, n_layers=2, hidden=2048,
                     inter=4096, n_heads=16, n_kv_heads=4, head_dim=128, vocab=4096,
                     qk_norm=True, n_experts=8, experts_per_tok=2, moe_inter=4096, tied=False,
                     weights="codes")
    sm = SynthModel(spec, seed=13)
    eng = tq.Engine(sm, max_seq_len=32)
    om = oracle.model(sm, 32, False)
    toks, logits = gc.model_tokens(eng, steps=8)
    otoks, ologits = gc.model_tokens(om, steps=8)
    assert toks == otoks
    for a, b in zip(logits, ologits):
        assert max_rel(a, b) < TOL
    eng.close()
    om.close()
