"""The multi-process side of bench.py on CPU: two gloo ranks, as torchrun would start them.

Replicas are independent (requests are sharded by rank, no data collective); the only
cross-rank steps are the barrier around the timed region and the max-over-ranks of the
device time, which these tests drive with host-side values. The reference arm runs on
rank 0 alone.
"""

from __future__ import annotations

import json
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist

    import bench

    r, w, local = bench.dist_setup(world)
    assert (r, w, local) == (rank, world, rank)
    assert dist.get_backend() == "gloo"
    bench.barrier(w)
    job = bench.max_over_ranks(1.5 + rank, w)  # each rank reports its own time; the job takes the slowest
    ctx, tables = bench.workload(seed=rank)  # rank r serves its own shard of requests
    bench.barrier(w)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump({"job": job, "ctx": ctx[:8], "blocks": [t[:2] for t in tables[:4]]}, f)
    dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_share_the_slowest_time_and_keep_their_own_shards(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    assert [x["job"] for x in res] == [2.5, 2.5]
    assert res[0]["ctx"] != res[1]["ctx"]  # different requests per replica (weak scaling)
    for x in res:
        assert all(128 <= c <= 2048 for c in x["ctx"])


def _reference_rank(rank: int, world: int, out_dir: str) -> None:
    import contextlib
    import io
    import sys

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world))
    import bench

    sys.argv = ["bench.py", "--impl", "reference", "--steps", "3", "--warmup", "1"]
    buf = io.StringIO()
    if rank != 0:  # the other ranks exit at once, without work or output
        with contextlib.redirect_stdout(buf):
            bench.main()
    with open(os.path.join(out_dir, f"ref{rank}.txt"), "w") as f:
        f.write(buf.getvalue())


@pytest.mark.timeout(60)
def test_reference_arm_is_silent_off_rank_zero(tmp_path):
    mp.start_processes(_reference_rank, args=(2, str(tmp_path)), nprocs=2, start_method="spawn")
    assert (tmp_path / "ref1.txt").read_text() == ""


def _serving_rank(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist

    import bench

    r, w, _ = bench.dist_setup(world)
    requests = bench.serving_workload(seed=0, vocab=1000)
    mine = [i for i in range(len(requests)) if i % w == r]  # the serving legs' sharding
    tokens = bench.sum_over_ranks(sum(requests[i][1] for i in mine), w)
    gathered = bench.gather_to_rank0((mine, [r] * len(mine)), w)
    with open(os.path.join(out_dir, f"serve{rank}.json"), "w") as f:
        json.dump({"tokens": tokens, "ids": gathered[0], "owners": gathered[1]}, f)
    dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_serving_shards_cover_every_request_once_and_totals_add_up(tmp_path):
    """Config 3's 200 requests split i mod N: every request is served by exactly one rank, the
    job's output-token total is the sum over ranks, and rank 0 gathers every rank's records."""
    import bench

    world = 2
    mp.start_processes(_serving_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    res = [json.loads((tmp_path / f"serve{r}.json").read_text()) for r in range(world)]
    requests = bench.serving_workload(seed=0, vocab=1000)
    assert res[0]["tokens"] == res[1]["tokens"] == sum(m for _, m in requests)
    ids = sorted(i for per_rank in res[0]["ids"] for i in per_rank)
    assert ids == list(range(len(requests)))
    assert [set(o) for o in res[0]["owners"]] == [{0}, {1}]
