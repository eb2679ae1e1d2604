"""Host logic of the multi-GPU path with world-size-2 gloo ranks on CPU: contiguous balanced shards and the
variable-size gather that restores request order."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from opendecider_b200.distributed import gather_rows, shard


def test_shard_contiguous_balanced():
    w = [5, 1, 1, 1, 1, 1, 5, 5]
    b = shard(w, 2)
    assert b[0][0] == 0 and b[-1][1] == len(w) and b[0][1] == b[1][0]
    tot = [sum(w[s:e]) for s, e in b]
    assert abs(tot[0] - tot[1]) <= max(w)
    assert shard([1] * 8, 4) == [(0, 2), (2, 4), (4, 6), (6, 8)]
    b = shard([1, 1], 4)                       # more ranks than items: empty blocks at the end
    assert sum(e - s for s, e in b) == 2 and len(b) == 4


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = torch.full((rank + 2, 3 + rank), float(rank), dtype=torch.float64)
        parts = gather_rows(x)
        ok = [p.shape == (r + 2, 3 + r) and bool((p == r).all()) for r, p in enumerate(parts)]
        q.put((rank, all(ok)))
    finally:
        dist.destroy_process_group()


def test_gather_rows_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _failing_worker(rank, world, port, q):
    """Rank 1 dies before the gather; rank 0's gather must end with an error (a short process-group timeout or the
    closed connection), never wait for good."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        q.put((rank, "died"))
        q.close()
        q.join_thread()                                      # the message is out before the process ends
        os._exit(3)                                          # leaves without joining the collective
    try:
        gather_rows(torch.zeros(2, 3))
        q.put((rank, "no error"))
    except Exception as e:                                   # noqa: BLE001 - any error is the expected outcome
        q.put((rank, "error: " + type(e).__name__))


def test_gather_fails_cleanly_when_a_rank_dies():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 500) % 1000
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "died"
    assert res[0].startswith("error"), res[0]
