"""The benchmark's multi-rank host logic on CPU: two gloo ranks shard the
batched workload's sequences with no overlap and reduce the whole-job
figures (slowest rank's time, all ranks' tokens) the way the GPU run does."""
import json
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    mine = bench.shard(256, rank, world)
    # rank r pretends to take 1 + r seconds for 100 * (r + 1) tokens
    t, g = bench.aggregate(dist, 1.0 + rank, 100.0 * (rank + 1), device="cpu")
    with open(os.path.join(out, f"r{rank}.json"), "w") as f:
        json.dump({"mine": mine, "t": t, "g": g}, f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shard_and_aggregate_over_gloo_ranks(tmp_path, world):
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [json.load(open(tmp_path / f"r{r}.json")) for r in range(world)]
    seen = sorted(i for r in res for i in r["mine"])
    assert seen == list(range(256))                           # every sequence on exactly one rank
    for r in res:
        assert r["t"] == 1.0 + (world - 1)                    # the slowest rank's time
        assert r["g"] == sum(100.0 * (k + 1) for k in range(world))


def test_single_rank_aggregate_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.aggregate(None, 2.5, 7.0, device="cpu") == (2.5, 7.0)
    assert bench.shard(5, 0, 1) == [0, 1, 2, 3, 4]
