"""The multi-GPU bookkeeping of bench.py on CPU ranks (gloo, world size 2).

By default the ranks split the configuration's (batch, kv head) units; the
only cross-rank steps are the max of the step times and the sum of the work.
A rank that never joins must make the others fail with an error instead of
waiting forever."""
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


def _unit_worker(rank, world, port, out):
    # every rank takes its units of one shared c2-shaped batch (scaled), runs
    # the CPU restatement on views of them, and the ranks' outputs tile the
    # single-process result
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench
    from oracle import sfa_oracle as O
    from ops_b200 import workloads as W
    cfg = W.scaled(W.CONFIGS["c2"], B=2, T=256, Hq=8, Hk=2, S=4)
    d = W.make_inputs(cfg, "cpu", bench.rank_seed(0))
    b0, b1, h0, h1 = bench.unit_range(cfg, world, rank)
    G = cfg.Hq // cfg.Hk
    q = d["q"][b0:b1, :, h0 * G:h1 * G].float()
    k, v = d["k"][b0:b1, :, h0:h1].float(), d["v"][b0:b1, :, h0:h1].float()
    idx = d["idx"][b0:b1, :, h0:h1]
    o, _ = O.sfa_forward(q, k, v, idx, cfg.bs, cfg.scale)
    pairs = W.count_pairs(idx, cfg.bs, cfg.T, cfg.T) * G
    _, _, total = bench.reduce_over_ranks(1.0, 1.0, pairs, torch.device("cpu"))
    out[rank] = ((b0, b1, h0, h1), o, total)
    dist.destroy_process_group()


def test_units_split_over_two_gloo_ranks():
    from oracle import sfa_oracle as O
    from ops_b200 import workloads as W
    import bench
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_unit_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    cfg = W.scaled(W.CONFIGS["c2"], B=2, T=256, Hq=8, Hk=2, S=4)
    d = W.make_inputs(cfg, "cpu", bench.rank_seed(0))
    o, _ = O.sfa_forward(d["q"].float(), d["k"].float(), d["v"].float(), d["idx"], cfg.bs, cfg.scale)
    G = cfg.Hq // cfg.Hk
    for r in range(2):
        (b0, b1, h0, h1), orank, total = out[r]
        assert torch.equal(orank, o[b0:b1, :, h0 * G:h1 * G])
        assert total == W.count_pairs(d["idx"], cfg.bs, cfg.T, cfg.T) * G


def test_unit_range_deals_every_unit_once():
    import bench
    from ops_b200 import workloads as W
    c2, c3 = W.CONFIGS["c2"], W.CONFIGS["c3"]
    for cfg, worlds in ((c2, (1, 2, 4, 8, 16)), (c3, (1, 2, 4))):
        for n in worlds:
            seen = []
            for r in range(n):
                b0, b1, h0, h1 = bench.unit_range(cfg, n, r)
                seen += [(b, h) for b in range(b0, b1) for h in range(h0, h1)]
            assert sorted(seen) == [(b, h) for b in range(cfg.B) for h in range(cfg.Hk)], (cfg.name, n)
    # c3 has 4 units: 8 ranks fall back to the query-row split
    assert bench.unit_range(c3, 8, 0) is None

    class A:
        split = "auto"
    assert bench.resolve_split(A, c2, 8) == "units" and bench.resolve_split(A, c3, 8) == "query"
    assert bench.resolve_split(A, c2, 1) == "none"


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
