"""The multi-process path of bench.py on CPU: two gloo ranks.

The benchmark runs one process per GPU with no collective in the data path;
its only cross-rank steps are the barrier around the timed region, the
maximum of the elapsed times (the job's time is the slowest rank's) and the
sum of the kernel-launch counts. These run here on two gloo ranks, with the
per-rank input shards the benchmark generates (seeded by rank).
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert bench._env_rank() == (rank, rank, world)
        dist.barrier()
        elapsed = 1.0 + rank  # rank 1 is the slow one
        job = bench.max_over_ranks(elapsed, dist, "cpu")
        launches = bench.sum_over_ranks(10 * (rank + 1), dist, "cpu")
        cfg = dict(bench.CONFIGS["raft_cpu_case"])
        host, _ = bench.make_inputs(cfg, rank, "cpu")
        sig = float(host["f1"].float().sum())
        sigs = [None] * world
        dist.all_gather_object(sigs, sig)
        out[rank] = (job, launches, sigs)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_time_max_launch_sum_and_shards():
    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        job, launches, sigs = res[rank]
        assert job == pytest.approx(2.0)          # the slowest rank's time
        assert launches == pytest.approx(30.0)    # 10 + 20
        assert sigs[0] != sigs[1]                 # each rank draws its own shard


def test_single_process_helpers_are_identity():
    assert bench.max_over_ranks(3.5, None, "cpu") == 3.5
    assert bench.sum_over_ranks(7, None, "cpu") == 7


def test_split_workload_ranks_take_slices_of_one_global_batch():
    # The default workload splits one global batch over the ranks (strong
    # scaling): rank k's inputs are images [k*B/N, (k+1)*B/N) of the batch a
    # single process would generate.
    base = dict(bench.CONFIGS["raft_cpu_case"], B=4, split=True, backward=True)
    whole = dict(base)
    host1, dev1 = bench.make_inputs(whole, 0, "cpu")
    world = 2
    for rank in range(world):
        cfg = dict(base, global_B=4, B=4 // world)
        host, dev = bench.make_inputs(cfg, rank, "cpu")
        lo, hi = rank * 2, rank * 2 + 2
        assert torch.equal(host["f1"], host1["f1"][lo:hi])
        assert torch.equal(host["f2"], host1["f2"][lo:hi])
        assert all(torch.equal(a, b[lo:hi]) for a, b in zip(host["coords"], host1["coords"]))
        assert all(torch.equal(a, b[lo:hi]) for a, b in zip(dev["grads"], dev1["grads"]))
    assert bench.CONFIGS[bench.DEFAULT].get("split")
