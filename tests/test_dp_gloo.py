"""The data-parallel exchange (r97training_b200/dp.py) on CPU: world-size-2 gloo ranks all-reduce a flat
gradient in per-layer buckets issued in reverse layer order, a bucket the walk never reports is issued at
the join, and a rank that dies before the exchange ends its peer's collective
with an error inside the process group's timeout instead of a hang. CPU only."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


RANGES = [(0, 7), (7, 300), (300, 301), (301, 1000), (1000, 4096)]


def _exchange(rank, world, port, results, skip, overlap):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from r97training_b200.dp import GradBuckets
        g = torch.arange(4096, dtype=torch.float32) * (rank + 1) + rank
        buckets = GradBuckets(g, RANGES, overlap=overlap)
        for li in reversed(range(len(RANGES))):
            if skip and li == 2:
                continue  # the walk never reported bucket 2 (on every rank alike)
            buckets.ready(li)
        order = buckets.join()
        ref = torch.arange(4096, dtype=torch.float32) * sum(r + 1 for r in range(world)) / world + \
            sum(range(world)) / world
        results[rank] = (bool(torch.allclose(g, ref)), order)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("skip,overlap", [(False, True), (True, True), (True, False)])
def test_bucketed_allreduce_two_ranks(skip, overlap):
    """overlap=False: the reports are recorded and the join exchanges the whole buffer at once."""
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        mp.start_processes(_exchange, args=(2, _port(), results, skip, overlap), nprocs=2, join=True,
                           start_method="spawn")
        assert results[0][0] and results[1][0], dict(results)
        for r in range(2):
            assert results[r][1] == ([4, 3, 1, 0, 2] if skip else [4, 3, 2, 1, 0])


def _dies(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from r97training_b200.dp import GradBuckets
    g = torch.ones(64)
    buckets = GradBuckets(g, [(0, 64)])
    if rank == 1:
        results[rank] = "left"
        os._exit(0)  # leaves between steps: nothing of its own in flight, never joins the exchange
    try:
        buckets.ready(0)
        buckets.join()
        results[rank] = "completed"
    except Exception as e:  # the process group's timeout (or the peer's closed connection) ends the wait
        results[rank] = "error: " + type(e).__name__


def test_dead_rank_ends_peer_collective_with_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _port()
        procs = [ctx.Process(target=_dies, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung past the process group's timeout"
        assert results.get(1) == "left"
        assert str(results.get(0, "")).startswith("error"), dict(results)
