"""Request sharding over ranks (``omniasr_b200.shard``): the host side of the multi-GPU path, run here as two
``gloo`` processes on the CPU. Every rank decodes its own contiguous shard; rank 0 gets the results back in request
order and the slowest rank's time."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from omniasr_b200 import shard


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("total", [0, 1, 5, 8, 64, 67])
def test_shards_cover_requests_once(world, total):
    bounds = [shard.shard_bounds(total, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == total
    for (a0, b0), (a1, _) in zip(bounds, bounds[1:]):
        assert b0 == a1  # contiguous, no overlap
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1
    assert [x for r in range(world) for x in shard.shard(list(range(total)), world, r)] == list(range(total))


def test_bad_rank_is_refused():
    with pytest.raises(ValueError):
        shard.shard_bounds(8, 2, 2)
    with pytest.raises(ValueError):
        shard.shard_bounds(8, 0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(x: int) -> list[int]:  # stands in for one request's token sequence
    return [x, x * x % 7, (3 * x + 1) % 11]


def _rank(rank: int, world: int, port: int, total: int, out_dir: str):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        mine = shard.shard(list(range(total)), world, rank)
        results = [_decode(x) for x in mine]
        dist.barrier()
        slowest = shard.max_over_ranks(1.5 + rank)
        gathered = shard.gather_in_order(results, total)
        bad_len = False
        try:
            shard.gather_in_order(results + [[0]], total)
        except ValueError:
            bad_len = True  # refused on the host before any collective
        torch.save({"slowest": slowest, "gathered": gathered, "bad_len": bad_len}, os.path.join(out_dir, f"{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [7, 8])
def test_two_ranks_gather_in_request_order(total):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, _free_port(), total, d), nprocs=world, join=True, start_method="spawn")
        r0 = torch.load(os.path.join(d, "0.pt"))
        r1 = torch.load(os.path.join(d, "1.pt"))
    assert r0["gathered"] == [_decode(x) for x in range(total)]
    assert r1["gathered"] is None
    assert r0["slowest"] == r1["slowest"] == 2.5
    assert r0["bad_len"] and r1["bad_len"]
