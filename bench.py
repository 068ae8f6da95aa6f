#!/usr/bin/env python
"""SFA forward+backward throughput on B200 — prints one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A step is one forward + backward of the sparse attention op over one batch of
the configuration's synthetic inputs (default c2: B=4, T=8192, Hq=64, Hk=4,
D=128, block_size=64, 16 selected blocks per (query, kv head)).  Under torchrun
every rank processes its own batch of that shape (weak scaling: the global
batch is 4*N; no collective on the data path — ranks share nothing).  With
--split query (for configurations with fewer (batch, kv head) units than
ranks, e.g. c3) the ranks instead split one batch's query rows, balanced by
selected pairs (ops_b200/shard.py), and the step includes the one
reduce-scatter that sums the dK/dV partials (strong scaling).

value      selected-token TFLOP/s of the whole job (all ranks), inputs resident
           in HBM, timed with CUDA events per step (L2 flushed between steps),
           max over ranks.  FLOPs: fwd 2P(Dqk+Dv) + bwd 2P(3Dqk+2Dv) over the
           P valid (query-head, key) pairs counted from the indices.
e2e        the same metric through the public API (ops_b200.sparse_flash_attention
           + autograd) with the step's inputs copied from pinned host memory and
           its outputs (o, dq, dk, dv) copied back inside the timed region.
roofline   the dominant kernel: its algorithmic FLOPs per launch / its CUDA-event
           duration, against the measured bf16 peak.
cpu_baseline  the CPU restatement (oracle/sfa_oracle.py, fp32 PyTorch, all host
           threads) on a bounded sample of the same workload (rank 0, N=1).
--impl reference  times that CPU restatement alone on the same config/metric
           (the reference's own kernels are Triton-Ascend and have no CPU or CUDA
           implementation to run here).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SFA fwd+bwd TFLOP/s (selected tokens) & % bf16 tensor peak, 1/2/4/8 B200"
# DRAM bytes (read + write) per launch from ncu captures of the c2 shape at B=1
# (the kernel summaries kept with the profiles), scaled x4 to the bench's B=4
# launch: each unit's q/dO/o/dq rows are read or written once and its K/V stay
# in L2.
NCU_TRAFFIC = {"c2": {"fwd": 4 * (0.153979e9 + 0.102984e9),
                      "bwd_dq": 4 * (0.296924e9 + 0.112170e9),        # SFA_DQ_SEPARATE
                      "bwd_dkdv": 4 * (1.294898e9 + 0.735617e9)}}     # with the fused dQ
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi SM clocks / throttle reasons sampled every 50 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.samples = []
        self.proc = None
        self.gpu = gpu_index
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0, t1):
        sel = [p for (t, p) in self.samples if t0 <= t <= t1] or [p for (_, p) in self.samples]
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(p[1]) for p in sel if num(p[1]) is not None]
        mx = [num(p[2]) for p in sel if num(p[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for p in sel for n, v in zip(names, p[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sel)}


# ---------------------------------------------------------------------------
# CPU restatement (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def cpu_sample_run(cfg, n_tok, seed=0):
    """fwd+bwd of the CPU restatement over the last n_tok queries of one (batch,
    kv head) unit of the configuration; returns (seconds, flops)."""
    import torch
    from oracle import sfa_oracle as O
    from ops_b200 import workloads as W
    G = cfg.Hq // cfg.Hk
    one = W.scaled(cfg, B=1, Hq=G, Hk=1)
    d = W.make_inputs(one, "cpu", seed, dtype=torch.bfloat16)
    t0 = cfg.T - n_tok
    q = d["q"][:, t0:].float()
    k, v = d["k"].float(), d["v"].float()
    idx = d["idx"][:, t0:]
    do = d["do"][:, t0:].float()
    pairs = W.count_pairs(idx, cfg.bs, n_tok, cfg.T) * G
    flops = O.sfa_flops(pairs, cfg.Dqk, cfg.Dv).total
    s = time.perf_counter()
    o, lse = O.sfa_forward(q, k, v, idx, cfg.bs, cfg.scale, None, cfg.causal)
    O.sfa_backward(q, k, v, idx, o, lse, do, cfg.bs, cfg.scale, None, cfg.causal)
    return time.perf_counter() - s, flops


def calibrate_cpu_tokens(cfg, target_s):
    n = 32
    dt, _ = cpu_sample_run(cfg, n)
    n2 = int(max(32, min(cfg.T, n * target_s / max(dt, 1e-3))))
    return n2


def cpu_baseline(cfg, target_s=12.0):
    import torch
    n = calibrate_cpu_tokens(cfg, target_s)
    dt, fl = cpu_sample_run(cfg, n)
    G = cfg.Hq // cfg.Hk
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"last {n} queries x {G} heads of one (batch, kv head) unit of {cfg.name}, "
                      f"fwd+bwd, fp32 PyTorch ({dt:.1f} s)"}


def run_reference(args, cfg):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    n = calibrate_cpu_tokens(cfg, 4.0)
    for _ in range(args.warmup):
        cpu_sample_run(cfg, n)
    tot_t, tot_f = 0.0, 0.0
    for i in range(args.steps):
        dt, fl = cpu_sample_run(cfg, n, seed=i)
        tot_t += dt
        tot_f += fl
    v = tot_f / tot_t / 1e12
    G = cfg.Hq // cfg.Hk
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_t / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, args.gpus),
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"per step: last {n} queries x {G} heads of one (batch, kv head) unit, "
                                       "fwd+bwd of the fp32 PyTorch restatement of SFA.py"},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def reduce_over_ranks(step_ms, e2e_ms, flops, device):
    """Whole-job figures: the slowest rank's step times and the work of all
    ranks (each rank processes its own batch; nothing else is exchanged)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(step_ms), float(e2e_ms), float(flops)
    t = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    f = torch.tensor([flops], dtype=torch.float64, device=device)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(f[0])


def rank_seed(rank: int) -> int:
    """Each rank draws its own batch of the configuration."""
    return 1000 + rank


def config_dict(cfg, n, split=False):
    per = "" if split else "/rank"
    return {"workload": f"{cfg.name}: block-sparse GQA attention fwd+bwd, B={cfg.B}{per}, T={cfg.T}, "
                        f"Hq={cfg.Hq}, Hk={cfg.Hk}, Dqk={cfg.Dqk}, Dv={cfg.Dv}, block_size={cfg.bs}, "
                        f"S={cfg.S}, {cfg.mode} causal selection, q/k/v/dO ~ N(0,1)",
            "global_batch": cfg.B if split else cfg.B * n, "seq_len": cfg.T,
            "parallelism": (f"{n} query-row ranges balanced by selected pairs, dK/dV summed by one "
                            f"reduce-scatter" if split else f"dp{n} (independent batch shards)"),
            "l2": "flushed between timed steps (256 MiB memset)"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    import ops_b200
    from ops_b200 import _lib
    from ops_b200 import sfa as S
    from ops_b200 import workloads as W
    from oracle import sfa_oracle as O  # noqa: F401  (FLOP formula only)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()

    # --split query (strong scaling of one batch): every rank builds the same
    # inputs and takes its range of query rows against the keys they can see;
    # the dK/dV partials are summed by one reduce-scatter inside the step
    split = args.split == "query" and world > 1
    d = W.make_inputs(cfg, dev, seed=rank_seed(0 if split else rank))
    q, k, v, idx, do = d["q"], d["k"], d["v"], d["idx"], d["do"]
    r0, r1, ke = 0, cfg.T, cfg.T
    if split:
        from ops_b200 import shard
        work = (shard.row_cost(idx, cfg.bs, cfg.T) if args.balance == "cost"
                else shard.row_work(idx, cfg.bs, cfg.T))
        ranges = shard.query_ranges(work, world)
        r0, r1 = ranges[rank]
        ke = r1
        q, idx, do = q[:, r0:r1], idx[:, r0:r1], do[:, r0:r1]
        k, v = k[:, :ke], v[:, :ke]
    G = cfg.Hq // cfg.Hk
    pairs = W.count_pairs(idx, cfg.bs, r1 - r0, ke) * G
    fl = O.sfa_flops(pairs, cfg.Dqk, cfg.Dv)
    o = torch.empty(*q.shape[:-1], cfg.Dv, dtype=q.dtype, device=dev)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=dev)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    scfg = S._Cfg(cfg.bs, cfg.scale, True, False, r1 - r0, ke, _lib.SFA_DKV_AUTO, _lib.SFA_KERNEL_AUTO, False,
                  S._DQ[args.dq_mode])
    P = S.build_params(q, k, v, idx, o, lse, scfg, None, None, None, do, dq, dk, dv, None)
    fam_f = lib.sfa_select_kernel(ctypes.byref(P), 0)
    fam_b = lib.sfa_select_kernel(ctypes.byref(P), 1)
    dkv_mode, dq_mode = ctypes.c_int32(), ctypes.c_int32()
    _lib.check(min(0, lib.sfa_bwd_plan(ctypes.byref(P), ctypes.byref(dkv_mode), ctypes.byref(dq_mode))), "plan")
    fused_dq = dq_mode.value == _lib.SFA_DQ_FUSED
    nbytes = lib.sfa_bwd_workspace_bytes(ctypes.byref(P))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    Pp = ctypes.byref(P)
    stages = ["fwd", "bwd_preprocess", "bwd_dq", "bwd_dkdv"] + (["dkdv_reduce_scatter"] if split else [])
    if split:
        tc = (cfg.T + world - 1) // world
        rs_in = torch.zeros(world * tc, cfg.B, cfg.Hk, cfg.Dqk + cfg.Dv, dtype=torch.float32, device=dev)
        rs_out = torch.empty(tc, cfg.B, cfg.Hk, cfg.Dqk + cfg.Dv, dtype=torch.float32, device=dev)

    def step(ev=None):
        if ev:
            ev[0].record(stream)
        _lib.check(lib.sfa_fwd(Pp, None, 0, sptr), "sfa_fwd")
        if ev:
            ev[1].record(stream)
        _lib.check(lib.sfa_bwd_preprocess(Pp, ws.data_ptr(), nbytes, sptr), "preprocess")
        if ev:
            ev[2].record(stream)
        _lib.check(lib.sfa_bwd_dq(Pp, ws.data_ptr(), nbytes, sptr), "dq")
        if ev:
            ev[3].record(stream)
        _lib.check(lib.sfa_bwd_dkdv(Pp, ws.data_ptr(), nbytes, sptr), "dkdv")
        if ev:
            ev[4].record(stream)
        if split:
            rs_in[:ke, ..., :cfg.Dqk].copy_(dk.transpose(0, 1))
            rs_in[:ke, ..., cfg.Dqk:].copy_(dv.transpose(0, 1))
            dist.reduce_scatter_tensor(rs_out, rs_in)
            if ev:
                ev[5].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    nev = len(stages) + 1
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(args.steps)]
    n0 = lib.sfa_kernel_launches()
    t_wall0 = time.time()
    for i in range(args.steps):
        flush.zero_()
        step(evs[i])
    torch.cuda.synchronize()
    t_wall1 = time.time()
    n1 = lib.sfa_kernel_launches()
    if world > 1:
        dist.barrier()
    stage_ms = {s: sum(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps)) / args.steps
                for j, s in enumerate(stages)}
    step_ms = sum(evs[i][0].elapsed_time(evs[i][nev - 1]) for i in range(args.steps)) / args.steps

    # e2e through the public API, host buffers
    host = {n: t.cpu().pin_memory() for n, t in (("q", q), ("k", k), ("v", v), ("idx", idx), ("do", do))}
    outs = {n: torch.empty(tuple(t.shape), dtype=t.dtype, pin_memory=True) for n, t in
            (("o", o), ("dq", q), ("dk", k), ("dv", v))}
    if split:   # a rank gets back its rows and its key share of dk / dv
        k0, k1 = shard.key_share(cfg.T, world, rank)
        outs["dk"] = torch.empty((cfg.B, k1 - k0, cfg.Hk, cfg.Dqk), dtype=k.dtype, pin_memory=True)
        outs["dv"] = torch.empty((cfg.B, k1 - k0, cfg.Hk, cfg.Dv), dtype=v.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs.values())

    def e2e_split_step():
        qd = host["q"].to(dev, non_blocking=True)
        kd = host["k"].to(dev, non_blocking=True)
        vd = host["v"].to(dev, non_blocking=True)
        ixd = host["idx"].to(dev, non_blocking=True)
        dod = host["do"].to(dev, non_blocking=True)
        r = shard.local_step(qd, kd, vd, ixd, dod, (r0, r1), cfg.T, rank, world, cfg.bs, cfg.scale)
        outs["o"].copy_(r["o"], non_blocking=True)
        outs["dq"].copy_(r["dq"], non_blocking=True)
        outs["dk"].copy_(r["dk"], non_blocking=True)
        outs["dv"].copy_(r["dv"], non_blocking=True)

    def e2e_step():
        if split:
            return e2e_split_step()
        qd = host["q"].to(dev, non_blocking=True).requires_grad_()
        kd = host["k"].to(dev, non_blocking=True).requires_grad_()
        vd = host["v"].to(dev, non_blocking=True).requires_grad_()
        ixd = host["idx"].to(dev, non_blocking=True)
        dod = host["do"].to(dev, non_blocking=True)
        oo, _ = ops_b200.sparse_flash_attention(qd, kd, vd, ixd, cfg.bs, dq_mode=args.dq_mode)
        oo.backward(dod)
        outs["o"].copy_(oo.detach(), non_blocking=True)
        outs["dq"].copy_(qd.grad, non_blocking=True)
        outs["dk"].copy_(kd.grad, non_blocking=True)
        outs["dv"].copy_(vd.grad, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 5))
    for _ in range(max(1, min(args.warmup, 2))):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_ms = 0.0
    for _ in range(e2e_steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush.zero_()
        a.record(stream)
        e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_ms += a.elapsed_time(b)
    e_ms /= e2e_steps
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)

    per_rank = [stage_ms]
    if world > 1:   # every rank's stage times (load balance of a split)
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {k: round(v, 4) for k, v in stage_ms.items()})
    step_ms_max, e_ms_max, flops_all = reduce_over_ranks(step_ms, e_ms, fl.total, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_kind = peaks()
    # algorithmic FLOPs owned by each stage (recomputation not counted)
    two_p = 2.0 * pairs
    tc_bwd = fam_b == _lib.SFA_KERNEL_TCGEN05
    # with the fused dQ the dK/dV stage also owns dQ = dS.K (2P.Dqk) and the dQ
    # stage only clears the accumulator
    stage_flops = {"fwd": fl.fwd,
                   "bwd_preprocess": 0.0,
                   "bwd_dq": 0.0 if fused_dq else (two_p * (2 * cfg.Dqk + cfg.Dv) if tc_bwd else fl.bwd),
                   "bwd_dkdv": (two_p * (2 * cfg.Dqk + cfg.Dv) if fused_dq else two_p * (cfg.Dqk + cfg.Dv))
                   if tc_bwd else 0.0,
                   "dkdv_reduce_scatter": 0.0}
    dom = max(stages, key=lambda s: stage_ms[s])
    # K and V rows gathered per (row, kv head): selected keys x (Dqk + Dv) bf16
    kv_gather = pairs / G * (cfg.Dqk + cfg.Dv) * 2.0
    # dK/dV: each selected (block, query) gathers the query's G heads of q and dO
    qdo_gather = pairs / cfg.bs * (cfg.Dqk + cfg.Dv) * 2.0
    gather_bytes = {"fwd": kv_gather, "bwd_dkdv": qdo_gather} if tc_bwd else {}
    if tc_bwd and not fused_dq:
        gather_bytes["bwd_dq"] = kv_gather
    ach = stage_flops[dom] / (stage_ms[dom] * 1e-3) / 1e12
    value = flops_all / (step_ms_max * 1e-3) / 1e12
    e2e_v = flops_all / (e_ms_max * 1e-3) / 1e12
    fams = {1: "tcgen05", 2: "general"}
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms_max, "higher_is_better": True,
        "scaling": "strong" if split else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config_dict(cfg, world, split),
        "pct_bf16_peak": 100.0 * value / world / peak,
        "tokens_per_s": cfg.B * cfg.T * (1 if split else world) / (step_ms_max * 1e-3),
        "selected_pairs_per_rank": pairs,
        "stages_ms": stage_ms,
        **({"stages_ms_per_rank": per_rank} if world > 1 else {}),
        "kernel_family": {"fwd": fams.get(fam_f, str(fam_f)), "bwd": fams.get(fam_b, str(fam_b)),
                          "dkv": {1: "inverted", 2: "atomic"}.get(dkv_mode.value),
                          "dq": {1: "separate", 2: "fused"}.get(dq_mode.value)},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                     "frac": ach / peak, "peak_kind": f"{peak_kind} bf16 burst",
                     "traffic": NCU_TRAFFIC.get(cfg.name, {}).get(dom) if cfg.B == 4 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at B=1, "
                                       "x4 for the B=4 launch (profiles/)"},
        # gathered K/V rows per launch (L2 -> shared memory) of the dominant stage
        "gather": {"kernel": dom, "bytes_per_launch": gather_bytes.get(dom),
                   "achieved": (gather_bytes[dom] / (stage_ms[dom] * 1e-3) / 1e12) if gather_bytes.get(dom) else None,
                   "unit": "TB/s"},
        "e2e": {"value": e2e_v, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e_ms_max},
        "clocks": clocks,
        "gpu_launches": int(n1 - n0),
    }
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def run_decode(args, cfg):
    """Forward-only configurations (c5: varlen decode, one query per sequence):
    a step is one sfa_fwd over the batch; HBM-bound, so the line reports the
    gathered K/V bytes per second against the measured copy bandwidth."""
    import torch
    import torch.distributed as dist

    import ops_b200
    from ops_b200 import _lib
    from ops_b200 import sfa as S
    from ops_b200 import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()
    d = W.make_decode(cfg, dev, seed=rank_seed(rank))
    q, k, v, idx, cu_q, cu_k = d["q"], d["k"], d["v"], d["idx"], d["cu_q"], d["cu_k"]
    keys = W.count_pairs(idx, cfg.bs, 1, 0, kv_lens=d["kv_lens"])        # valid (query, kv head, key)
    G = cfg.Hq // cfg.Hk
    gathered = keys * (cfg.Dqk + cfg.Dv) * 2.0                             # K and V rows read
    flops = 2.0 * keys * G * (cfg.Dqk + cfg.Dv)
    o = torch.empty(q.shape[0], cfg.Hq, cfg.Dv, dtype=q.dtype, device=dev)
    lse = torch.empty(q.shape[0], cfg.Hq, dtype=torch.float32, device=dev)
    scfg = S._Cfg(cfg.bs, cfg.scale, True, True, 1, d["max_k"], _lib.SFA_DKV_AUTO, _lib.SFA_KERNEL_AUTO, False)
    P = S.build_params(q, k, v, idx, o, lse, scfg, None, cu_q, cu_k)
    fam = lib.sfa_select_kernel(ctypes.byref(P), 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    for _ in range(args.warmup):
        _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, sptr), "sfa_fwd")
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    n0 = lib.sfa_kernel_launches()
    t_wall0 = time.time()
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, sptr), "sfa_fwd")
        b.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    n1 = lib.sfa_kernel_launches()
    step_ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    # e2e through the public API with host buffers
    host = {n: t.cpu().pin_memory() for n, t in (("q", q), ("k", k), ("v", v), ("idx", idx))}
    o_h = torch.empty(tuple(o.shape), dtype=o.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = o_h.numel() * o_h.element_size()
    cu_qd, cu_kd = cu_q.to(dev), cu_k.to(dev)

    def e2e_step():
        qd, kd, vd, ixd = (host[n].to(dev, non_blocking=True) for n in ("q", "k", "v", "idx"))
        oo, _ = ops_b200.sparse_flash_attention(qd, kd, vd, ixd, cfg.bs, cu_seqlens=cu_qd, cu_seqlens_k=cu_kd,
                                                max_seqlen_q=1, max_seqlen_k=d["max_k"])
        o_h.copy_(oo, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_ms = 0.0
    for _ in range(max(1, min(args.steps, 3))):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_ms += a.elapsed_time(b)
    e_ms /= max(1, min(args.steps, 3))
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)
    step_ms_max, e_ms_max, bytes_all = reduce_over_ranks(step_ms, e_ms, gathered, dev)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    hbm = None
    try:
        hbm = float(json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                "MEASURED_PEAKS.json")))["hbm_gbs"])
        hbm_kind = "measured copy"
    except Exception:
        hbm, hbm_kind = 6650.0, "fallback"
    gbs = gathered / (step_ms * 1e-3) / 1e9
    line = {
        "metric": "SFA decode forward GB/s (gathered K/V rows), B200", "value": bytes_all / (step_ms_max * 1e-3) / 1e9,
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: varlen decode forward, {cfg.n_seqs} sequences/rank x 1 query, kv "
                               f"lengths U[{cfg.kv_min}, {cfg.kv_max}], Hq={cfg.Hq}, Hk={cfg.Hk}, Dqk={cfg.Dqk}, "
                               f"Dv={cfg.Dv}, block_size={cfg.bs}, S={cfg.S} uniform blocks, q/k/v ~ N(0,1)",
                   "global_batch": cfg.n_seqs * world, "parallelism": f"dp{world} (independent sequence shards)",
                   "l2": "flushed between timed steps (256 MiB memset)"},
        "tflops": flops / (step_ms * 1e-3) / 1e12,
        "kernel_family": {1: "tcgen05", 2: "general"}.get(fam, str(fam)),
        "roofline": {"bound": "hbm", "kernel": "fwd", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "peak_kind": hbm_kind, "traffic": None},
        "e2e": {"value": bytes_all / (e_ms_max * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e_ms_max},
        "clocks": clocks,
        "gpu_launches": int(n1 - n0),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c2")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--batch", type=int, default=0, help="override the per-rank batch (profiling runs)")
    ap.add_argument("--seq", type=int, default=0, help="override the sequence length (scaled secondary configs)")
    ap.add_argument("--dq-mode", choices=["auto", "separate", "fused"], default="auto",
                    help="backward dQ plan (profiling runs): its own query-centric pass or fused into dK/dV")
    ap.add_argument("--balance", choices=["pairs", "cost"], default="cost",
                    help="--split query: balance rows by selected pairs, or by a cost that also counts the "
                         "dK/dV pass's jobs and batches (ops_b200/shard.py row_cost)")
    ap.add_argument("--split", choices=["none", "query"], default="none",
                    help="with N > 1: 'query' splits one batch's query rows over the ranks (strong scaling, "
                         "for configurations with fewer (batch, kv head) units than ranks)")
    args = ap.parse_args()
    from ops_b200 import workloads as W
    cfg = W.CONFIGS[args.config]
    if args.batch:
        cfg = W.scaled(cfg, B=args.batch)
    if args.seq:
        cfg = W.scaled(cfg, T=args.seq)
    if cfg.fwd_only:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "forward-only decode config; the reference arm "
                              "times the fwd+bwd configurations"}))
            return
        run_decode(args, cfg)
        return
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
