"""The N>1 host logic of bench.py on CPU ranks (gloo, world size 2): contiguous sequence
shards with no data-path collective, barrier, and the max-over-ranks timing reduction.  A
rank that fails is reported by the others through a short process-group timeout."""
from __future__ import annotations

import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        lo, hi = bench.shard_range(65536, world, rank)
        bench.barrier(world)
        t = bench.max_over_ranks(10.0 * (rank + 1), world)
        q.put((rank, lo, hi, t))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_max_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(world))
    assert [(lo, hi) for _, lo, hi, _ in res] == [(0, 32768), (32768, 65536)]
    assert all(t == 20.0 for *_, t in res)  # every rank sees the slowest rank's time


def _failing_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(3)  # a rank that dies between steps
    try:
        bench.max_over_ranks(1.0, world)
        q.put("no-error")
    except Exception as e:  # the survivor learns of it from the collective's timeout/error
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_error():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    assert procs[1].exitcode == 3
    assert q.get(timeout=5) != "no-error"


@pytest.mark.parametrize("n,world", [(10, 3), (8192, 8), (7, 8), (0, 2)])
def test_shard_range_covers_exactly(n, world):
    spans = [bench.shard_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1
