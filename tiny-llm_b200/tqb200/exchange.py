"""Host side of the engine's peer exchange: every rank's 64-byte arena handle shared with
every other rank, then opened by each (Engine.exchange_handle / Engine.open_exchange).

Two rendezvous forms: a torch.distributed process group (any backend; the handles travel
as Python objects), or a directory that all ranks can see (each rank writes its handle
to a file of its own, renamed into place when complete, and reads the others' once all
are there, within a time limit)."""
from __future__ import annotations

import os
import time
from typing import Callable, List

HANDLE_BYTES = 64


def gather_over_pg(handle: bytes, pg) -> List[bytes]:
    """All ranks' handles in rank order, over the process group module `pg`
    (torch.distributed or a group-bound equivalent)."""
    assert len(handle) == HANDLE_BYTES
    out: list = [None] * pg.get_world_size()
    pg.all_gather_object(out, handle)
    assert all(isinstance(h, bytes) and len(h) == HANDLE_BYTES for h in out), "bad handle"
    return out


def gather_over_dir(handle: bytes, rank: int, world: int, directory: str,
                    timeout_s: float = 60.0, sleep: Callable[[float], None] = time.sleep) -> List[bytes]:
    """All ranks' handles in rank order through files in `directory`."""
    assert len(handle) == HANDLE_BYTES and 0 <= rank < world
    path = os.path.join(directory, f"xchg_{rank}.bin")
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(handle)
    os.replace(tmp, path)
    deadline = time.monotonic() + timeout_s
    paths = [os.path.join(directory, f"xchg_{r}.bin") for r in range(world)]
    while not all(os.path.exists(p) for p in paths):
        if time.monotonic() > deadline:
            missing = [r for r, p in enumerate(paths) if not os.path.exists(p)]
            raise TimeoutError(f"peer exchange: ranks {missing} wrote no handle in {timeout_s} s")
        sleep(0.01)
    out = []
    for p in paths:
        with open(p, "rb") as f:
            h = f.read()
        if len(h) != HANDLE_BYTES:
            raise ValueError(f"peer exchange: {p} holds {len(h)} bytes")
        out.append(h)
    return out


def open_exchange(engine, handles: List[bytes]) -> None:
    """Opens the peers' arenas in `engine` (its own handle included at its rank)."""
    engine.open_exchange(handles)
