"""Query-range sharding on two GPUs (NCCL): each rank runs its rows through the
CUDA op, dK/dV partials meet in one reduce-scatter, and the assembled result
equals the single-GPU one (o / lse bitwise: rows are independent; dq, dk, dv to
bf16 rounding of the per-rank partials).  Also for one latent kv tensor (v a
leading-dims view of k: one gradient per key).  Needs two GPUs; skipped
otherwise."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(name):
    from ops_b200 import workloads as W
    if name == "latent":       # c4's layout: one latent kv tensor, v = kv[..., :512]
        cfg = W.scaled(W.CONFIGS["c4"], T=1024, S=256)
    else:
        cfg = W.scaled(W.CONFIGS["c3"], T=4096, S=16)
    return cfg, W.make_inputs(cfg, "cpu", 21)


def _v(name, cfg, t):
    return t["k"][..., :cfg.Dv] if name == "latent" else t["v"]


def _worker(rank, world, port, out, name):
    import torch.distributed as dist
    from ops_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    cfg, d = _case(name)
    t = {n: d[n].to(dev) for n in ("q", "k", "v", "idx", "do")}
    ranges = shard.query_ranges(shard.row_work(t["idx"], cfg.bs, cfg.T), world)
    r = shard.shard_step(t["q"], t["k"], _v(name, cfg, t), t["idx"], t["do"], rank, world, ranges,
                         block_size=cfg.bs)
    torch.cuda.synchronize()
    out[rank] = {key: (val.cpu() if torch.is_tensor(val) else val) for key, val in r.items()}
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["c3", "latent"])
def test_query_range_split_on_two_gpus_matches_one_gpu(name):
    from ops_b200 import shard
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out, name), nprocs=world, join=True)
    cfg, d = _case(name)
    dev = torch.device("cuda", 0)
    t = {n: d[n].to(dev) for n in ("q", "k", "v", "idx", "do")}
    o, lse, dq, dk, dv = shard.op_fwd_bwd(t["q"], t["k"], _v(name, cfg, t), t["idx"], t["do"], cfg.bs, cfg.scale,
                                          True)
    o, lse, dq, dk = (x.cpu() for x in (o, lse, dq, dk))
    pairs = [("dk", dk)] + ([] if dv is None else [("dv", dv.cpu())])
    for r in range(world):
        res = out[r]
        r0, r1 = res["rows"]
        k0, k1 = res["keys"]
        assert torch.equal(res["o"], o[:, r0:r1]) and torch.equal(res["lse"], lse[:, r0:r1])
        assert (res["dv"] is None) == (dv is None)
        for got, ref in [(res["dq"], dq[:, r0:r1])] + [(res[n], g[:, k0:k1]) for n, g in pairs]:
            err = float((got.float() - ref.float()).abs().max())
            assert err < 2e-2 * max(1.0, float(ref.float().abs().max())), (r, err)
