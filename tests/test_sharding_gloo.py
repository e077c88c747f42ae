"""Batch sharding + output gather across ranks, on CPU `gloo` ranks (world size 2 and 3)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from whisper_blaze_b200.sharding import gather_batch, max_shard, run_sharded, shard_bounds


def test_shard_bounds_cover_and_balance():
    for total in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1 and max(sizes) <= max_shard(total, world)
    assert shard_bounds(64, 8, 3) == (24, 32)
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        full = torch.arange(total * 6, dtype=torch.float32).view(total, 2, 3)
        # each rank transforms only its own slice; the gather restores global order
        out = run_sharded(lambda x: x * 2 + rank * 0, full)
        ok = torch.equal(out, full * 2)
        s, e = shard_bounds(total, world, rank)
        local = full[s:e] + 1
        gathered = gather_batch(local, total)
        ok = ok and torch.equal(gathered, full + 1)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 64), (3, 8), (2, 5)])
def test_gather_restores_global_batch_order(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(results[r] for r in range(world))
