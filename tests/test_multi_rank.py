"""Multi-rank host logic on the CPU with the gloo backend (world_size 2 and 3):
batch shard ranges and the final ordered gather of per-rank outputs, plus a
rank that fails before the gather being reported to the others instead of
hanging them."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, load_package


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, fail_rank, results):
    import datetime
    import sys

    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        sharding = load_package().sharding
        start, stop = sharding.shard_range(total, world, rank)
        # Stand-in for this rank's forward output: rows tagged by global index.
        local = torch.arange(start, stop, dtype=torch.float32)[:, None].repeat(1, 3)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        out = sharding.gather_shards(local, total, dst=0)
        if rank == 0:
            results.put(("ok", out.tolist()))
    except Exception as e:  # report, then leave the group
        results.put(("err", f"rank {rank}: {type(e).__name__}"))
    finally:
        dist.destroy_process_group()


def _run(world, total, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_shard_range_covers_batch():
    sharding = load_package().sharding
    for total in (0, 1, 4, 5, 10000):
        for world in (1, 2, 3, 8):
            ranges = [sharding.shard_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    assert load_package().sharding.shard_range(4, 8, 7) == (4, 4)  # idle rank
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


@pytest.mark.parametrize("world,total", [(2, 5), (3, 7), (2, 1)])
def test_gather_is_ordered_and_complete(world, total):
    res = _run(world, total)
    oks = [r for r in res if r[0] == "ok"]
    assert len(oks) == 1, res
    rows = oks[0][1]
    assert [row[0] for row in rows] == list(range(total))


def test_failing_rank_does_not_hang_the_others():
    res = _run(2, 6, fail_rank=1)
    assert any(kind == "err" and "rank 1" in msg for kind, msg in res), res
