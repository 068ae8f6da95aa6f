"""Query-range sharding (ops_b200.shard) on CPU ranks: gloo, world size 2 and 3.

Each rank runs the CPU restatement on its rows (the CUDA op needs a GPU), and
the reduce-scatter of the dK/dV partials is the same call the GPU ranks make.
The assembled rows and key shares must equal the single-process result."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sfa_oracle as O
from ops_b200 import shard
from ops_b200 import workloads as W


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_fwd_bwd(q, k, v, idx, do, bs, scale, causal):
    o, lse = O.sfa_forward(q.float(), k.float(), v.float(), idx, bs, scale, None, causal)
    dq, dk, dv, _ = O.sfa_backward(q.float(), k.float(), v.float(), idx, o, lse, do.float(), bs, scale, None, causal)
    return o, lse, dq, dk, dv


def _case():
    cfg = W.scaled(W.CONFIGS["c3"], B=1, T=384, Hq=8, Hk=2, Dqk=32, Dv=32, bs=16, S=6)
    d = W.make_inputs(cfg, "cpu", 5, dtype=torch.float32)
    return cfg, d


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    cfg, d = _case()
    work = shard.row_work(d["idx"], cfg.bs, cfg.T)
    ranges = shard.query_ranges(work, world)
    r = shard.shard_step(d["q"], d["k"], d["v"], d["idx"], d["do"], rank, world, ranges, block_size=cfg.bs,
                         fwd_bwd=_oracle_fwd_bwd)
    rec = {key: (val.clone() if torch.is_tensor(val) else val) for key, val in r.items()}
    rec["work"] = [int(work[a:b].sum()) for a, b in ranges]
    out[rank] = rec
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_query_range_shards_assemble_to_the_full_result(world):
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    cfg, d = _case()
    o, lse, dq, dk, dv = _oracle_fwd_bwd(d["q"], d["k"], d["v"], d["idx"], d["do"], cfg.bs, None, True)
    rows, keys = [], []
    for r in range(world):
        res = out[r]
        r0, r1 = res["rows"]
        rows.append((r0, r1))
        if r1 > r0:
            assert torch.allclose(res["o"], o[:, r0:r1], atol=1e-5, rtol=1e-5)
            assert torch.allclose(res["lse"], lse[:, r0:r1], atol=1e-5, rtol=1e-5)
            assert torch.allclose(res["dq"], dq[:, r0:r1], atol=1e-5, rtol=1e-5)
        k0, k1 = res["keys"]
        keys.append((k0, k1))
        assert torch.allclose(res["dk"], dk[:, k0:k1], atol=1e-4, rtol=1e-4)
        assert torch.allclose(res["dv"], dv[:, k0:k1], atol=1e-4, rtol=1e-4)
    # the ranges tile the rows and the key shares tile the keys
    assert rows[0][0] == 0 and rows[-1][1] == cfg.T and all(rows[i][1] == rows[i + 1][0] for i in range(world - 1))
    assert keys[0][0] == 0 and keys[-1][1] == cfg.T and all(keys[i][1] == keys[i + 1][0] for i in range(world - 1))
    # balanced: no rank carries more than its share plus one row's work
    work = out[0]["work"]
    assert max(work) - sum(work) / world <= int(shard.row_work(d["idx"], cfg.bs, cfg.T).max())


def test_query_ranges_balance_and_edge_cases():
    w = torch.tensor([0, 0, 5, 5, 5, 5, 0, 0, 10, 0], dtype=torch.int64)
    rg = shard.query_ranges(w, 2)
    assert rg[0][0] == 0 and rg[-1][1] == 10 and rg[0][1] == rg[1][0]
    assert abs(int(w[rg[0][0]:rg[0][1]].sum()) - 15) <= 10
    assert shard.query_ranges(torch.zeros(4, dtype=torch.int64), 3)[-1] == (0, 4)
    assert shard.query_ranges(w, 1) == [(0, 10)]
    assert [shard.key_share(10, 3, r) for r in range(3)] == [(0, 4), (4, 8), (8, 10)]


def test_row_cost_conserves_pairs_batches_and_jobs():
    # every (batch, kv head, 2048-row range, block) list with n queries is one
    # job of ceil(n / 8) batches; the per-row costs must add up to exactly
    # per_pair * pairs + per_batch * batches + per_job * jobs
    cfg = W.scaled(W.CONFIGS["c3"], B=2, T=5000, Hq=8, Hk=2, S=8)
    idx = W.make_indices(cfg, "cpu", 4)
    pairs = int(shard.row_work(idx, cfg.bs, cfg.T).sum())
    lists = {}
    for b in range(cfg.B):
        for t in range(cfg.T):
            for h in range(cfg.Hk):
                for e in idx[b, t, h].tolist():
                    if 0 <= e and e * cfg.bs <= t:     # causal, self-attention: the block has a key <= t
                        key = (b, h, t // 2048, e)
                        lists[key] = lists.get(key, 0) + 1
    jobs = len(lists)
    batches = sum((n + 7) // 8 for n in lists.values())
    c = shard.row_cost(idx, cfg.bs, cfg.T, per_pair=1.0, per_batch=1000.0, per_job=1e6)
    assert abs(float(c.sum()) - (pairs + 1000.0 * batches + 1e6 * jobs)) < 1e-3 * float(c.sum())
    only_pairs = shard.row_cost(idx, cfg.bs, cfg.T, per_pair=1.0, per_batch=0.0, per_job=0.0)
    assert torch.equal(only_pairs, shard.row_work(idx, cfg.bs, cfg.T).to(torch.float64))


def test_default_cost_weights_come_from_the_recorded_split():
    # per-rank stage times of a two-GPU split of the c3 shape balanced by pairs
    # (bench --config c3 --split query --balance pairs, stages_ms_per_rank):
    # forward 9.3779 / 9.2859 ms, dK/dV 9.2304 / 10.5881 ms; refitting them
    # from the rows' counted pairs, batches and jobs gives row_cost's defaults
    import inspect
    cfg = W.CONFIGS["c3"]
    idx = W.make_indices(cfg, "cpu", 1000)
    ranges = shard.query_ranges(shard.row_work(idx, cfg.bs, cfg.T), 2)
    units = shard.range_units(idx, cfg.bs, ranges)
    fit = shard.fit_cost(units, [9.3779, 9.2859], [9.2304, 10.5881])
    defaults = {k: v.default for k, v in inspect.signature(shard.row_cost).parameters.items()
                if k in ("per_pair", "per_batch", "per_job")}
    for k, v in defaults.items():
        assert abs(fit[k] - v) <= 0.02 * v, (k, fit[k], v)
    # two ranks: an exact solve, flagged as such
    assert fit["exact"] and fit["rank"] == 2 and fit["residual"] < 1e-9


def test_fit_cost_rejects_models_that_do_not_fit():
    # a negative per-job time (more jobs, less time) is refused
    with pytest.raises(ValueError):
        shard.fit_cost([(100, 10, 5), (100, 10, 50)], [1.0, 1.0], [2.0, 1.0])
    # dependent counts (one rank a multiple of the other) are refused
    with pytest.raises(ValueError):
        shard.fit_cost([(100, 10, 5), (200, 20, 10)], [1.0, 2.0], [1.0, 2.0])
    # three ranks over-determine the fit: a residual is reported
    f = shard.fit_cost([(100, 10, 5), (100, 12, 9), (100, 20, 6)], [1.0, 1.0, 1.0], [1.0, 1.5, 1.6])
    assert f["rank"] == 2 and not f["exact"] and f["residual"] >= 0.0


def _oracle_fwd_bwd_latent(q, k, v, idx, do, bs, scale, causal):
    # the op's contract for v a leading-dims view of k: one gradient dk + dv in k's shape
    o, lse, dq, dk, dv = _oracle_fwd_bwd(q, k, v, idx, do, bs, scale, causal)
    dk = dk.clone()
    dk[..., :v.shape[-1]] += dv
    return o, lse, dq, dk, None


def _latent_case():
    cfg = W.scaled(W.CONFIGS["c4"], B=1, T=200, Hq=8, Hk=1, Dqk=48, Dv=32, bs=1, S=40)
    d = W.make_inputs(cfg, "cpu", 6, dtype=torch.float32)
    return cfg, d


def _latent_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    cfg, d = _latent_case()
    ranges = shard.query_ranges(shard.row_work(d["idx"], cfg.bs, cfg.T), world)
    k = d["k"]
    r = shard.shard_step(d["q"], k, k[..., :cfg.Dv], d["idx"], d["do"], rank, world, ranges, block_size=cfg.bs,
                         fwd_bwd=_oracle_fwd_bwd_latent)
    out[rank] = {key: (val.clone() if torch.is_tensor(val) else val) for key, val in r.items()}
    dist.destroy_process_group()


def test_query_range_shards_with_one_latent_kv_tensor():
    # v = k[..., :Dv] (the MLA layout): the ranks reduce one gradient per key
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_latent_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    cfg, d = _latent_case()
    k = d["k"]
    _, _, _, dk, _ = _oracle_fwd_bwd_latent(d["q"], k, k[..., :cfg.Dv], d["idx"], d["do"], cfg.bs, None, True)
    for r in range(world):
        res = out[r]
        k0, k1 = res["keys"]
        assert res["dv"] is None
        assert torch.allclose(res["dk"], dk[:, k0:k1], atol=1e-4, rtol=1e-4)
