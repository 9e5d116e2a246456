"""The multi-GPU bench's host logic on CPU ranks (gloo, world size 2): every rank a distinct shard, timings reduced
as the max over ranks and bytes as the sum -- the same calls bench.py makes under torchrun with NCCL."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = bench.WORKLOADS["config3"]
        sch = bench.Schedule(wl, 12, bench.shard_seed(rank), start=3)
        nbytes = sum(sch.step_bytes(s) for s in range(3, 8))
        elapsed = 10.0 + rank  # rank 1 is the slow one
        t, b = bench.combine_ranks(elapsed, nbytes, dist, torch.device("cpu"))
        out.put((rank, t, b, nbytes, sch.pos[3].tolist()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_reduce_max_time_and_sum_bytes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, t0, b0, n0, pos0), (r1, t1, b1, n1, pos1) = res
    assert t0 == t1 == 11.0  # the max over ranks
    assert b0 == b1 == float(n0 + n1)  # the whole job's bytes
    assert pos0 != pos1  # independent shards (different windows)


def test_single_process_passthrough():
    assert bench.combine_ranks(3.5, 100, None, None) == (3.5, 100.0)


@pytest.mark.parametrize("rank", [0, 1, 7])
def test_shard_seeds_distinct(rank):
    assert len({bench.shard_seed(r) for r in range(8)}) == 8
    assert bench.shard_seed(rank) == 1234 + 7919 * rank
