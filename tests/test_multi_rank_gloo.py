"""The multi-GPU bookkeeping of bench.py on CPU ranks (gloo, world size 2).

Ranks process independent batches; the only cross-rank steps are the max of
the step times and the sum of the work.  A rank that never joins must make the
others fail with an error instead of waiting forever."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    import bench
    from ops_b200 import workloads as W
    step_ms = 10.0 + rank          # rank 1 is the slowest
    e2e_ms = 20.0 + 3 * rank
    flops = 1e12 * (rank + 1)
    res = bench.reduce_over_ranks(step_ms, e2e_ms, flops, torch.device("cpu"))
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hq=16, Hk=1, S=4)
    idx = W.make_indices(cfg, "cpu", bench.rank_seed(rank))
    out[rank] = (res, int(idx.sum()))
    dist.destroy_process_group()


def test_reduce_over_two_gloo_ranks():
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for r in range(2):
        (step, e2e, fl), _ = out[r]
        assert step == 11.0 and e2e == 23.0 and fl == 3e12
    assert out[0][1] != out[1][1], "ranks draw different batches"


def _lonely(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        return  # never joins
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as ex:  # the rendezvous times out with an error
        q.put(type(ex).__name__)


def test_missing_rank_fails_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_lonely, args=(2, _free_port(), q), nprocs=2, join=True)
    assert q.get(timeout=60) != "joined"
