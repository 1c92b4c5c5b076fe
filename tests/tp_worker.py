"""One rank of the tensor-parallel engine test (launched by test_gpu_tp.py, one process
per GPU): builds the seeded model of a golden case, runs the engine with
tp_size = world on GPU `rank`, and saves the greedy tokens and full logits.  With the
exchange mode "p2p" the ranks share their arena handles through files in a directory
and open the peer exchange before the first step (the all-gathers then run inside the
producing kernels); "nccl" keeps the NCCL all-gathers."""
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
from tqb200.model import SynthModel  # noqa: E402


def main():
    rank, world, nid_hex, case_name, out = sys.argv[1:6]
    mode = sys.argv[6] if len(sys.argv) > 6 else "nccl"
    rank, world = int(rank), int(world)
    _, spec, kv16, seed = [c for c in gc.MODEL_CASES if c[0] == case_name][0]
    sm = SynthModel(spec, seed=seed)
    eng = lib.Engine(sm, max_seq_len=64, kv_fp16=kv16, device=rank, tp_size=world,
                     tp_rank=rank, nccl_id=bytes.fromhex(nid_hex))
    if mode == "p2p":
        handles = exchange.gather_over_dir(eng.exchange_handle(), rank, world, sys.argv[7])
        exchange.open_exchange(eng, handles)
    toks, logits = gc.model_tokens(eng, steps=10)
    np.savez(out, tokens=np.array(toks), logits=np.stack(logits))
    eng.close()


if __name__ == "__main__":
    main()
