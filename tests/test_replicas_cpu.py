"""The --gpus N replica path of bench.py on CPU: two gloo ranks each report their own
device times; the whole-job line takes the slowest rank's time (MAX over the process
group) and the tokens of both ranks.  Qwen3-0.6B at batch 1 does not shard, so the
replicas share nothing but this reduction."""

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _rank(rank, world, port, out):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        t_ms, e2e_ms = (100.0, 130.0) if rank == 0 else (125.0, 120.0)  # rank 1 is the slower decoder
        out[rank] = bench.aggregate_replicas(t_ms, e2e_ms, 50, world, "cpu")
    finally:
        dist.destroy_process_group()


def test_replica_aggregate_takes_slowest_rank_and_all_tokens():
    port = 29500 + os.getpid() % 1000
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank, args=(2, port, out), nprocs=2, join=True)
        res = dict(out)
    for rank in (0, 1):
        t_ms, e2e_ms, value, e2e = res[rank]
        assert t_ms == 125.0 and e2e_ms == 130.0
        assert value == pytest.approx(2 * 50 / 0.125)
        assert e2e == pytest.approx(2 * 50 / 0.130)


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.aggregate_replicas(10.0, 20.0, 4, 1, "cpu") == (10.0, 20.0, 400.0, 200.0)
