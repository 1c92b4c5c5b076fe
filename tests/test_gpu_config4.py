"""BASELINE config 4 (Qwen3-4B shape: 36 layers, hidden 2560, 32 query / 8 KV heads of
128, intermediate 9728, tied i4 embed / lm_head, fp16 KV) against the oracle's
forward_token (runtime/qwen_forward_token.cpp:83-742, the cache of
runtime/kv_cache.cpp:120-135).

With an fp16 cache, an fp32 K or V value that lies within a few ulp of a half-precision
rounding boundary can round the other way when the engine's float sums differ in their
last bits from the oracle's double sums: one cached element one half ulp apart (a
"flip", up to 9.8e-4 relative).  That happens even within the first step (the current
token's V is its own attention output there), and every later layer and step reads the
flipped element, so two independent runs drift apart by more than 1e-4 over 36 layers.
The tests therefore measure two things:

* Guided oracle: after each engine step the oracle runs the same step with the engine's
  cache as a guide (tqo_model_set_kv_guide): it writes the engine's K/V rows, so both
  continue from the same cache, and measures how far each element is from its own
  rounding.  Asserted: every cached element within one binary16 ulp plus 3e-5 of its
  head row's largest magnitude (the rounding of an fp32-sized difference, measured up
  to ~1e-5 after 36 layers, nothing more), logits within 1e-4 at every step, greedy
  tokens identical; the number of elements that rounded the other way is reported.
* Free-running oracle (no guide): greedy tokens identical for a 32-token prompt and 64
  steps, logits within 5e-4 at every step (the flips' drift), the worst reported.

A second case runs at the benchmarked context: seeded fp16 N(0,1) K/V written into both
caches for positions 0..4094, then 4 guided steps from position 4095.
"""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

from conftest import max_rel
from devmem import d2h, h2d
from tqb200.model import QWEN3_4B, SynthModel

pytestmark = pytest.mark.gpu
TOL = 1e-4
TOL_FREE_RUNNING = 5e-4
KV_DEV = 3e-5  # cached element vs the oracle's own rounding: one ulp + KV_DEV x head row max
SPEC = replace(QWEN3_4B, weights="codes", max_seq_len=8192)


@pytest.fixture(scope="module")
def model():
    return SynthModel(SPEC, seed=0)


def _engine_kv(eng) -> np.ndarray:
    ptr, nbytes = eng.kv_cache()
    return d2h(ptr, nbytes).view(np.uint16)


def test_config4_prompt32_then_64_steps_f16kv(tq, oracle, model):
    max_seq = 128
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, SPEC.vocab, 32)]
    eng = tq.Engine(model, max_seq_len=max_seq, kv_fp16=True)
    guided = oracle.model(model, max_seq, True)
    free = oracle.model(model, max_seq, True)
    toks, gtoks, ftoks = [], [], []
    worst_guided = worst_free = 0.0
    nxt = fnxt = None
    for i in range(len(prompt) + 64):
        t = prompt[i] if i < len(prompt) else nxt
        ft = prompt[i] if i < len(prompt) else fnxt
        nxt = eng.step(t)
        el = eng.logits()
        ekv = _engine_kv(eng)
        guided.set_kv_guide(ekv, KV_DEV)
        gnxt = guided.step(t)
        flips, mism, dev = guided.kv_guide_counts()
        assert mism == 0, f"step {i}: {mism} cached elements beyond rounding (worst {dev:.2e})"
        err = max_rel(el, guided.logits())
        assert err < TOL, f"step {i}: logits max_rel {err:.3e} against the guided oracle"
        worst_guided = max(worst_guided, err)
        fnxt = free.step(ft)
        ferr = max_rel(el, free.logits())
        assert ferr < TOL_FREE_RUNNING, f"step {i}: logits max_rel {ferr:.3e} (free-running)"
        worst_free = max(worst_free, ferr)
        if i >= len(prompt) - 1:
            toks.append(nxt)
            gtoks.append(gnxt)
            ftoks.append(fnxt)
    assert toks == gtoks == ftoks, (toks, gtoks, ftoks)
    flips, _, dev = guided.kv_guide_counts()
    n = 2 * SPEC.n_layers * SPEC.n_kv_heads * (len(prompt) + 64) * SPEC.head_dim
    print(f"config 4, 32 + 64 steps: tokens identical; {flips} of {n} cached elements rounded "
          f"the other way, at most {dev:.2e} of the head row's max beyond one ulp; logits "
          f"max_rel {worst_guided:.2e} (guided), {worst_free:.2e} (free-running)")
    eng.close()
    guided.close()
    free.close()


def test_config4_context_4096_f16kv(tq, oracle, model):
    ctx, steps = 4095, 4
    max_seq = ctx + steps + 1
    eng = tq.Engine(model, max_seq_len=max_seq, kv_fp16=True)
    om = oracle.model(model, max_seq, True)
    okv = om.kv().reshape(2, SPEC.n_layers, SPEC.n_kv_heads, max_seq, SPEC.head_dim)
    rng = np.random.default_rng(4096)
    for kv in range(2):
        for layer in range(SPEC.n_layers):
            okv[kv, layer, :, :ctx, :] = rng.standard_normal(
                (SPEC.n_kv_heads, ctx, SPEC.head_dim), dtype=np.float32).astype(np.float16).view(np.uint16)
    ptr, _ = eng.kv_cache()
    h2d(ptr, om.kv())
    eng.set_position(ctx)
    om.set_position(ctx)
    tok = int(rng.integers(0, SPEC.vocab))
    for s in range(steps):
        nxt = eng.step(tok)
        ekv = _engine_kv(eng)
        om.set_kv_guide(ekv, KV_DEV)
        onxt = om.step(tok)
        _, mism, dev = om.kv_guide_counts()
        assert mism == 0, f"step {s}: {mism} cached elements beyond rounding (worst {dev:.2e})"
        err = max_rel(eng.logits(), om.logits())
        assert nxt == onxt, f"step {s}: token {nxt} != oracle {onxt}"
        assert err < TOL, f"step {s} at position {ctx + s}: logits max_rel {err:.3e}"
        tok = nxt
    eng.close()
    om.close()
