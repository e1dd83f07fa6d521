"""Multi-rank host logic of easyfhe.shard on CPU: two gloo ranks partition the
units, agree on the max step time and all-gather limb buffers exactly."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, total: int, queue) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "easyfhe-llama3-8b_b200"))
    import datetime

    import torch.distributed as dist

    from easyfhe import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        mine = shard.shard_range(total, world, rank)
        local = torch.stack([torch.full((3, 5), u, dtype=torch.int64) for u in mine])
        full = shard.gather_units(local, total)
        mx = shard.max_over_ranks(float(rank + 1))
        queue.put((rank, list(mine), full.tolist(), mx))
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions():
    from easyfhe import shard

    for total in (0, 1, 7, 16, 17):
        for world in (1, 2, 3, 8):
            got = [u for r in range(world) for u in shard.shard_range(total, world, r)]
            assert got == list(range(total))
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)


@pytest.mark.parametrize("total", [16, 7])
def test_two_gloo_ranks_gather_and_max(total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, total, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    assert results[0][1] + results[1][1] == list(range(total))
    expect = [[[u] * 5 for _ in range(3)] for u in range(total)]
    for _, _, full, mx in results:
        assert full == expect
        assert mx == 2.0


def _dropping_worker(rank: int, port: int, queue) -> None:
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "easyfhe-llama3-8b_b200"))
    import torch.distributed as dist

    from easyfhe import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=10))
    shard.max_over_ranks(1.0)  # one step together
    if rank == 1:
        os._exit(0)  # this rank leaves between steps, with nothing in flight
    try:
        shard.max_over_ranks(2.0)
        queue.put("no error")
    except Exception as exc:  # the survivor learns of it at its next collective
        queue.put(type(exc).__name__)


def test_dropped_rank_surfaces_as_an_error_on_the_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropping_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    result = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert result != "no error"
