"""Host-side logic of the tensor-parallel path on CPU, world_size 2 over gloo.

The engine shards every projection by output rows (rank r owns rows
[r*n/G, (r+1)*n/G), one contiguous byte range of the i4 or VQ2 layout, the VQ2
codebook copied to every rank), all-gathers each rank's slice in place, and picks
the greedy token from every rank's (max, first index) pair.  These tests run that
decomposition with the oracle's matvecs on each rank and torch.distributed gloo for
the exchanges, and check that it reproduces the unsharded result bit for bit, and
that the NCCL id broadcast reaches every rank unchanged."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        q.put((rank, fn(rank)))
    except Exception as e:  # report instead of hanging the other rank
        q.put((rank, f"error: {e!r}"))
    finally:
        dist.destroy_process_group()


def _run(fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, fn, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def _sharded_matvecs(rank):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tiny-llm_b200")]
    from oracle.oracle import Oracle
    from tqb200 import synth
    orc = Oracle()
    rng = np.random.default_rng(7)
    M, K, G = 256, 512, 64
    w = synth.random_i4(rng, M, K, G)
    x = rng.normal(size=K).astype(np.float32)
    rb = synth.i4_row_bytes(K, G)
    n = M // WORLD
    mine = w.reshape(M, rb)[rank * n:(rank + 1) * n].reshape(-1)
    y = torch.from_numpy(orc.matvec_i4(mine, x, n, K, G).astype(np.float32))
    parts = [torch.empty_like(y) for _ in range(WORLD)]
    dist.all_gather(parts, y)
    full_i4 = torch.cat(parts).numpy()
    # VQ2: codebook on every rank + the rank's rows of indices
    wv = synth.random_vq2(rng, M, K)
    idx = wv[2048:].reshape(M, K // 4)
    mine_v = np.concatenate([wv[:2048], idx[rank * n:(rank + 1) * n].reshape(-1)])
    yv = torch.from_numpy(orc.matvec_vq2(mine_v, x, n, K).astype(np.float32))
    parts_v = [torch.empty_like(yv) for _ in range(WORLD)]
    dist.all_gather(parts_v, yv)
    full_v = torch.cat(parts_v).numpy()
    ref_i4 = orc.matvec_i4(w, x, M, K, G).astype(np.float32)
    ref_v = orc.matvec_vq2(wv, x, M, K).astype(np.float32)
    return bool(np.array_equal(full_i4, ref_i4) and np.array_equal(full_v, ref_v))


def _sharded_argmax(rank):
    # vocabulary shards with a tie across the shard boundary: the first index wins
    V = 1000
    logits = np.random.default_rng(3).normal(size=V).astype(np.float32)
    logits[[10, 600]] = logits.max() + 1.0
    n = V // WORLD
    mine = logits[rank * n:(rank + 1) * n]
    local = int(np.argmax(mine))  # numpy's argmax keeps the first maximum
    pair = torch.tensor([float(mine[local]), float(rank * n + local)], dtype=torch.float64)
    parts = [torch.empty_like(pair) for _ in range(WORLD)]
    dist.all_gather(parts, pair)
    best_v, best_i = -np.inf, None
    for p in parts:  # (value, index) rule of the engine's argmax over pairs
        v, i = float(p[0]), int(p[1])
        if v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    return best_i == int(np.argmax(logits)) == 10


def _nccl_id_broadcast(rank):
    nid = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        nid.copy_(torch.arange(128, dtype=torch.uint8) * 3)
    dist.broadcast(nid, src=0)
    return bytes(nid.numpy().tobytes()) == bytes((np.arange(128) * 3 % 256).astype(np.uint8))


def _handle(rank):
    return ((np.arange(64) * (rank + 3) + rank) % 256).astype(np.uint8).tobytes()


def _exchange_path():
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "tiny-llm_b200"))


def _exchange_handles_pg(rank):
    """The peer exchange's handle sharing over a process group: every rank gets every
    rank's 64-byte arena handle in rank order."""
    _exchange_path()
    from tqb200 import exchange
    got = exchange.gather_over_pg(_handle(rank), dist)
    return got == [_handle(r) for r in range(WORLD)]


def _exchange_handles_dir(directory, rank):
    """The same through files in a shared directory (the test workers' rendezvous)."""
    _exchange_path()
    from tqb200 import exchange
    got = exchange.gather_over_dir(_handle(rank), rank, WORLD, directory, timeout_s=60)
    return got == [_handle(r) for r in range(WORLD)]


@pytest.mark.parametrize("fn", [_sharded_matvecs, _sharded_argmax, _nccl_id_broadcast,
                                _exchange_handles_pg],
                         ids=["row_shards_allgather", "vocab_shard_argmax", "nccl_id_broadcast",
                              "exchange_handles_pg"])
def test_tp_host_logic_world2_gloo(fn):
    out = _run(fn)
    assert out == {0: True, 1: True}, out


def test_exchange_handles_dir_world2(tmp_path):
    import functools
    out = _run(functools.partial(_exchange_handles_dir, str(tmp_path)))
    assert out == {0: True, 1: True}, out


def test_exchange_handles_dir_times_out_without_peer(tmp_path):
    _exchange_path()
    from tqb200 import exchange
    with pytest.raises(TimeoutError, match=r"ranks \[1\]"):
        exchange.gather_over_dir(_handle(0), 0, 2, str(tmp_path), timeout_s=0.2)
    with pytest.raises(AssertionError):
        exchange.gather_over_dir(b"short", 0, 2, str(tmp_path), timeout_s=0.2)
