"""Batched prompt prefill on the GPU engine (QwenModel::forward_prefill,
runtime/qwen_forward_prefill.cpp:74; for MoE the expert grouping of
forward_prefill_moe_batch, runtime/qwen_forward_prefill.cpp:425-753) vs the same prompt
fed token by token through the oracle's forward_token restatement.

The prefill runs every projection and expert on the tensor-core matmul (fp32 results,
~1e-5 relative) and attention as one causal pass over the cache, so it is held to the
path's floating-point bar: the greedy next token identical, logits within max relative
error 1e-4, and the KV cache it leaves must give the oracle's greedy continuation."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

from conftest import max_rel
from tqb200.model import QWEN3_30B_A3B, ModelSpec, SynthModel

pytestmark = pytest.mark.gpu
TOL = 1e-4

CASES = [
    ("qwen2_bias_hd64", ModelSpec(name="p_qwen2", qkv_bias=True, norm_noise=0.1, hidden=256,
                                  inter=512, n_heads=4, n_kv_heads=2, head_dim=64), False),
    ("qwen3_f16kv_hd128", ModelSpec(name="p_qwen3", qk_norm=True, norm_noise=0.1, hidden=256,
                                    inter=512, n_heads=8, n_kv_heads=2, head_dim=128), True),
    ("qwen3_mha_hd64", ModelSpec(name="p_mha", qk_norm=True, hidden=256, inter=768, n_heads=4,
                                 n_kv_heads=4, head_dim=64, tied=False, embed_dtype="f32"), False),
    ("moe", ModelSpec(name="p_moe", model_type=3, qk_norm=True, n_experts=16, experts_per_tok=4,
                      moe_inter=64, tied=False, hidden=256, n_heads=4, n_kv_heads=2,
                      head_dim=64), False),
    ("moe_i4_router", ModelSpec(name="p_moe_i4", model_type=3, qk_norm=True, n_experts=32,
                                experts_per_tok=8, moe_inter=128, tied=False, hidden=256,
                                n_heads=8, n_kv_heads=2, head_dim=64, router_dtype="i4"), False),
]


def _read_in_place(spec):
    """Whether the prefill's matmul reads every matrix in place through a tensor map:
    only matrices whose in_dim / group_size is a multiple of 4 have one (their rows are a
    multiple of 16 bytes long); the others get a repacked copy."""
    ffn = spec.moe_inter if spec.model_type == 3 else spec.inter
    dims = (spec.hidden, spec.n_heads * spec.head_dim, ffn)
    return all((k // spec.group_size) % 4 == 0 for k in dims)


def _prompt(n, vocab, seed):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32).tolist()


def _oracle_feed(om, tokens):
    nxt = None
    for t in tokens:
        nxt = om.step(t)
    return nxt


def _continue(m, tok, steps):
    toks, logits = [], []
    for _ in range(steps):
        tok = m.step(tok)
        toks.append(tok)
        logits.append(m.logits())
    return toks, logits


@pytest.mark.parametrize("name,spec,kv16", CASES, ids=[c[0] for c in CASES])
def test_prefill_matches_token_by_token(tq, oracle, name, spec, kv16):
    sm = SynthModel(spec, seed=31)
    eng = tq.Engine(sm, max_seq_len=128, kv_fp16=kv16)
    om = oracle.model(sm, 128, kv16)
    prompt = _prompt(45, spec.vocab, 7)
    nxt = eng.prefill(prompt)
    onxt = _oracle_feed(om, prompt)
    assert eng.position == len(prompt)
    assert max_rel(eng.logits(), om.logits()) < TOL
    assert nxt == onxt
    assert (eng.prefill_copy_bytes() == 0) == _read_in_place(spec)
    toks, logits = _continue(eng, nxt, 8)
    otoks, ologits = _continue(om, onxt, 8)
    assert toks == otoks
    for a, b in zip(logits, ologits):
        assert max_rel(a, b) < TOL
    eng.close()
    om.close()


def test_prefill_after_decode_and_in_chunks(tq, oracle):
    """A prompt that starts after decoded positions (p0 > 0) and spans two chunks
    (512 + 100 tokens): the second chunk attends to the first chunk's cache."""
    spec = replace(CASES[1][1], max_seq_len=1024)
    sm = SynthModel(spec, seed=32)
    eng = tq.Engine(sm, max_seq_len=640)
    om = oracle.model(sm, 640, False)
    head = _prompt(3, spec.vocab, 8)
    for t in head:
        eng.step(t)
        om.step(t)
    prompt = _prompt(612, spec.vocab, 9)
    nxt = eng.prefill(prompt)
    onxt = _oracle_feed(om, prompt)
    assert eng.position == 615
    assert max_rel(eng.logits(), om.logits()) < TOL
    assert nxt == onxt
    toks, _ = _continue(eng, nxt, 4)
    otoks, _ = _continue(om, onxt, 4)
    assert toks == otoks
    eng.close()
    om.close()


def test_prefill_fallback_paths(tq, oracle):
    """Shapes the batched path does not take (head_dim 32) and a one-token prompt run
    as decode steps, with the same results."""
    spec = ModelSpec(name="p_hd32", qk_norm=True)
    sm = SynthModel(spec, seed=33)
    eng = tq.Engine(sm, max_seq_len=64)
    om = oracle.model(sm, 64, False)
    prompt = _prompt(12, spec.vocab, 10)
    assert eng.prefill(prompt) == _oracle_feed(om, prompt)
    assert max_rel(eng.logits(), om.logits()) < TOL
    assert eng.prefill([5]) == om.step(5)
    eng.close()
    om.close()


def test_prefill_config5_shape(tq, oracle):
    """BASELINE config 5 layer shapes (hidden 2048, 128 experts, top-8, expert inter 768,
    32/4 heads of 128, vocab 151936) over 2 layers: a 24-token prompt through the grouped
    expert GEMMs vs the oracle fed token by token."""
    spec = replace(QWEN3_30B_A3B, n_layers=2, max_seq_len=64, weights="codes")
    sm = SynthModel(spec, seed=5)
    eng = tq.Engine(sm, max_seq_len=64)
    om = oracle.model(sm, 64, False)
    prompt = _prompt(24, spec.vocab, 11)
    nxt = eng.prefill(prompt)
    onxt = _oracle_feed(om, prompt)
    assert max_rel(eng.logits(), om.logits()) < TOL
    assert nxt == onxt
    assert eng.prefill_copy_bytes() == 0  # every matrix read in place: i4 bytes held once
    toks, _ = _continue(eng, nxt, 3)
    otoks, _ = _continue(om, onxt, 3)
    assert toks == otoks
    eng.close()
    om.close()


def test_prefill_rejects_bad_input(tq):
    sm = SynthModel(CASES[0][1], seed=34)
    eng = tq.Engine(sm, max_seq_len=32)
    with pytest.raises(Exception):
        eng.prefill([1, 2, 10**6])
    with pytest.raises(Exception):
        eng.prefill(list(range(40)))  # beyond max_seq_len
    assert eng.position == 0
    eng.close()
