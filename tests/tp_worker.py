"""One rank of the tensor-parallel engine test (launched by test_gpu_tp.py, one process
per GPU): builds the seeded model of a golden case, runs the engine with
tp_size = world on GPU `rank`, and saves the greedy tokens and full logits.  With the
exchange mode "p2p" the ranks share their arena handles through files in a directory
and open the peer exchange before the first step (the all-gathers then run inside the
producing kernels); "nccl" keeps the NCCL all-gathers.  With "prefill" as the eighth
argument the engine first takes a 45-token prompt as one batched prefill (MoE models:
attention whole on every rank, the experts sharded), then decodes 8 tokens."""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))
sys.path.insert(0, os.path.join(HERE, "golden"))

import golden_cases as gc  # noqa: E402
from tqb200 import exchange, lib  # noqa: E402
from tqb200.model import ModelSpec, SynthModel  # noqa: E402

# a MoE model whose shape takes the batched prefill (head_dim 64)
PF_CASE = ("moe_pf", ModelSpec(name="p_moe", model_type=3, qk_norm=True, n_experts=16,
                               experts_per_tok=4, moe_inter=64, tied=False, hidden=256,
                               n_heads=4, n_kv_heads=2, head_dim=64), False, 31)


def prefill_prompt(vocab):
    return np.random.default_rng(7).integers(0, vocab, 45).astype(np.int32).tolist()


def main():
    rank, world, nid_hex, case_name, out = sys.argv[1:6]
    mode = sys.argv[6] if len(sys.argv) > 6 else "nccl"
    rank, world = int(rank), int(world)
    _, spec, kv16, seed = [c for c in gc.MODEL_CASES + [PF_CASE] if c[0] == case_name][0]
    sm = SynthModel(spec, seed=seed)
    eng = lib.Engine(sm, max_seq_len=64, kv_fp16=kv16, device=rank, tp_size=world,
                     tp_rank=rank, nccl_id=bytes.fromhex(nid_hex))
    if mode == "p2p":
        handles = exchange.gather_over_dir(eng.exchange_handle(), rank, world, sys.argv[7])
        exchange.open_exchange(eng, handles)
    if len(sys.argv) > 8 and sys.argv[8] == "prefill":
        prompt = prefill_prompt(spec.vocab)
        nxt = eng.prefill(prompt)
        toks, logits = [nxt], [eng.logits()]
        for _ in range(8):
            nxt = eng.step(nxt)
            toks.append(nxt)
            logits.append(eng.logits())
    else:
        toks, logits = gc.model_tokens(eng, steps=10)
    np.savez(out, tokens=np.array(toks), logits=np.stack(logits))
    eng.close()


if __name__ == "__main__":
    main()
