"""The decode engine on the GPU vs the oracle and the reference's golden decode.

Bars: greedy tokens identical, logits within max
relative error 1e-4 at every step.  The oracle is the C restatement pinned to
the reference's QwenModel::forward_token (tests/test_oracle.py)."""
from __future__ import annotations

import numpy as np
import pytest

import golden_cases as gc
from conftest import max_rel
from tqb200.model import QWEN25_05B, QWEN3_06B_VQ2, QWEN3_4B, ModelSpec, SynthModel
from dataclasses import replace

pytestmark = pytest.mark.gpu
TOL = 1e-4
ENGINE_CASES = [c for c in gc.MODEL_CASES
                if c[0] in ("qwen2_bias", "qwen3_f16kv", "untied_f32embed", "vq2_rot")]


@pytest.mark.parametrize("case", ENGINE_CASES, ids=[c[0] for c in ENGINE_CASES])
@pytest.mark.parametrize("graph", [True, False])
def test_engine_matches_reference_golden(tq, oracle, golden, case, graph):
    name, spec, kv16, seed = case
    sm = SynthModel(spec, seed=seed)
    eng = tq.Engine(sm, max_seq_len=64, kv_fp16=kv16, use_graph=graph)
    om = oracle.model(sm, 64, kv16)
    toks, logits = gc.model_tokens(eng, steps=10)
    otoks, ologits = gc.model_tokens(om, steps=10)
    assert toks == list(golden[f"model_{name}_tokens"]) == otoks
    for a, b in zip(logits, ologits):
        assert max_rel(a, b) < TOL
    eng.close()


def test_engine_reset_replays_identically(tq):
    sm = SynthModel(gc.MODEL_CASES[0][1], seed=11)
    eng = tq.Engine(sm, max_seq_len=32)
    a, _ = gc.model_tokens(eng, steps=8)
    eng.reset()
    b, _ = gc.model_tokens(eng, steps=8)
    assert a == b and eng.position == 8


def test_engine_rejects_bad_input(tq):
    sm = SynthModel(gc.MODEL_CASES[0][1], seed=11)
    eng = tq.Engine(sm, max_seq_len=4)
    with pytest.raises(tq.TQB200Error):
        eng.step(sm.spec.vocab)          # token out of range (qwen_forward_token.cpp:95-98)
    for t in range(4):
        eng.step(t)
    with pytest.raises(tq.TQB200Error):
        eng.step(0)                      # position beyond max_seq_len (:99-102)


def _decode_compare(tq, oracle, sm, prompt, n_new, max_seq, kv16):
    eng = tq.Engine(sm, max_seq_len=max_seq, kv_fp16=kv16)
    om = oracle.model(sm, max_seq, kv16)
    worst, toks, otoks = 0.0, [], []
    nxt = onxt = None
    for i in range(len(prompt) + n_new):
        t = prompt[i] if i < len(prompt) else nxt
        ot = prompt[i] if i < len(prompt) else onxt
        nxt, onxt = eng.step(t), om.step(ot)
        worst = max(worst, max_rel(eng.logits(), om.logits()))
        if i >= len(prompt) - 1:
            toks.append(nxt)
            otoks.append(onxt)
    eng.close()
    om.close()
    return toks, otoks, worst


def test_config2_qwen25_05b_64_steps(tq, oracle):
    """32 random prompt ids, fp32 KV (512), 64 greedy steps."""
    sm = SynthModel(QWEN25_05B, seed=0)
    prompt = list(np.random.default_rng(0).integers(0, QWEN25_05B.vocab, 32))
    toks, otoks, worst = _decode_compare(tq, oracle, sm, prompt, 64, 512, False)
    assert toks == otoks, (toks, otoks)
    assert worst < TOL


def test_config4_qwen3_4b_f32kv(tq, oracle):
    """BASELINE config 4 shape (36 layers, hidden 2560, 32/8 heads) with an fp32 cache,
    short run; the fp16-cache configuration as benchmarked is covered at length in
    test_gpu_config4.py."""
    spec = replace(QWEN3_4B, weights="codes")
    sm = SynthModel(spec, seed=0)
    prompt = list(np.random.default_rng(1).integers(0, spec.vocab, 4))
    toks, otoks, worst = _decode_compare(tq, oracle, sm, prompt, 4, 4096, False)
    assert toks == otoks
    assert worst < TOL, worst


def test_config3_qwen3_06b_vq2_step(tq, oracle):
    """BASELINE config 3 full step: 28-layer Qwen3-0.6B-shaped VQ2 model with a BiIP
    rotation on every projection input (7 per layer), tied i4 embed / lm_head."""
    sm = SynthModel(QWEN3_06B_VQ2, seed=0)
    prompt = list(np.random.default_rng(3).integers(0, QWEN3_06B_VQ2.vocab, 8))
    toks, otoks, worst = _decode_compare(tq, oracle, sm, prompt, 8, 64, False)
    assert toks == otoks
    assert worst < TOL, worst


def test_engine_outlier_channels(tq, oracle):
    """Heavy-tailed activations through every fused prologue: RMSNorm weights of 1e3 and
    1e4 on a few channels make the q/k/v and gate/up inputs span 4+ decades, and the
    SwiGLU products feeding down (with its residual) heavier still.  Tokens identical,
    logits within 1e-4 of the oracle."""
    spec = ModelSpec(name="outliers", qk_norm=True, n_layers=4, hidden=1024, inter=3072,
                     n_heads=8, n_kv_heads=2, head_dim=128, vocab=4096)
    sm = SynthModel(spec, seed=7)
    rng = np.random.default_rng(70)
    for li in range(spec.n_layers):
        for nm in ("input_layernorm", "post_attention_layernorm"):
            w = sm.tensors[f"model.layers.{li}.{nm}.weight"].data
            idx = rng.choice(spec.hidden, 6, replace=False)
            w[idx[:3]] = 1e3
            w[idx[3:]] = 1e4
    prompt = [int(t) for t in rng.integers(0, spec.vocab, 6)]
    toks, otoks, worst = _decode_compare(tq, oracle, sm, prompt, 6, 64, False)
    assert toks == otoks
    assert worst < TOL, worst
