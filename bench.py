#!/usr/bin/env python
"""SFA forward+backward throughput on B200 — prints one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A step is one forward + backward of the sparse attention op over one batch of
the configuration's synthetic inputs (default c2: B=4, T=8192, Hq=64, Hk=4,
D=128, block_size=64, 16 selected blocks per (query, kv head)).

Several GPUs (torchrun, one process per GPU).  The default split is by
(batch, kv head) units, the partition the op's independence gives: c2's 16
units are dealt out 16/N per rank (whole batches, or kv heads of one batch),
every rank runs the unchanged op on views of its units, and nothing is
exchanged (strong scaling: the global problem is the configuration's).
``--split query`` splits one batch's query rows instead (for configurations
with fewer units than ranks, e.g. c3 at 8 GPUs; ops_b200/shard.py) and adds the
one reduce-scatter that sums the dK/dV partials; ``--split batch`` gives every
rank its own batch of the configuration (weak scaling).

value      selected-token TFLOP/s of the whole job (all ranks), inputs resident
           in HBM, timed with CUDA events per step (L2 flushed between steps),
           max over ranks.  FLOPs: fwd 2P(Dqk+Dv) + bwd 2P(3Dqk+2Dv) over the
           P valid (query-head, key) pairs counted from the indices.
kernels    every kernel of the step, timed with CUDA events recorded between
           launches (the library's launch trace, sfa_launch_trace).
roofline   the kernel with the largest share of the step: its algorithmic
           FLOPs per launch / its CUDA-event duration, against the measured
           bf16 peak; traffic from an ncu capture of that kernel.
smem_port  (block-sparse forward) the forward's shared-memory traffic modelled
           from its N = G tiles (operand reads, gather and P writes) against
           the port's 128 B/clk on every SM: what bounds the N = 16 forward.
e2e        the same metric through the public API (ops_b200.sparse_flash_attention
           + autograd) with the step's inputs copied from pinned host memory and
           its outputs (o, dq, dk, dv) copied back inside the timed region; the
           rank's units go through in chunks on three streams, so one chunk's
           copies overlap another's kernels.
cpu_baseline  the CPU restatement (oracle/sfa_oracle.py, fp32 PyTorch, all host
           threads) on a fixed sample of the same workload (rank 0, N=1); the
           reference arm (--impl reference) runs that same sample per step.
configs    (N = 1, default config) the other BASELINE configurations, each
           with its value, roofline, e2e and CPU baseline.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SFA fwd+bwd TFLOP/s (selected tokens) & % bf16 tensor peak, 1/2/4/8 B200"
DECODE_METRIC = "SFA decode forward GB/s (gathered K/V rows), B200"
# DRAM bytes (read + write) per launch of each tensor-core kernel from ncu
# captures of the c2 shape at B = 1 (4 (batch, kv head) units; the summaries
# are kept with the profiles).  A launch over u units moves u/4 of that: each
# unit's q/dO/o/dq rows are read or written once and its K/V stay in L2.
NCU_TRAFFIC_C2_B1 = {"fwd_tc": 0.153979e9 + 0.102984e9,
                     "bwd_dq_tc": 0.296924e9 + 0.112170e9,
                     "bwd_dkdv_tc": 1.294898e9 + 0.735617e9}
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0


def peaks():
    """(bf16 burst TFLOP/s, HBM GB/s, kind) from MEASURED_PEAKS.json."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, FALLBACK_HBM_GBS, "fallback"


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
# CPU restatement: one sampling rule for cpu_baseline and the reference arm
# ---------------------------------------------------------------------------
# Fixed sample per configuration: fwd+bwd of the last `last` queries of the
# (batch 0, kv head 0) unit (decode: the forward of the first `seqs`
# sequences).  Up to a few seconds of fp32 work on 16 host threads each;
# cpu_baseline times it again on the same inputs until its budget is spent.
CPU_SAMPLE = {"c1": {"last": 1024}, "c2": {"last": 8192}, "c3": {"last": 1024}, "c4": {"last": 128},
              "c5": {"seqs": 16}, "tok128": {"last": 256}}


def cpu_sample_desc(cfg) -> str:
    s = CPU_SAMPLE.get(cfg.name, {"last": min(cfg.T, 1024)})
    if cfg.fwd_only:
        return (f"forward of the first {s.get('seqs', cfg.n_seqs)} sequences of {cfg.name} (all kv heads), "
                "fp32 PyTorch restatement of SFA.py")
    G = cfg.Hq // cfg.Hk
    return (f"fwd+bwd of the last {min(cfg.T, s['last'])} queries x {G} heads of the (batch 0, kv head 0) unit "
            f"of {cfg.name}, fp32 PyTorch restatement of SFA.py")


def cpu_sample_prepare(cfg, seed=0):
    """The fixed CPU sample's inputs (generated once, untimed); returns a
    function that runs the sample and returns (seconds, work), work in FLOPs
    (fwd+bwd configurations) or gathered K/V bytes (decode)."""
    import torch
    from oracle import sfa_oracle as O
    from ops_b200 import workloads as W
    s = CPU_SAMPLE.get(cfg.name, {"last": min(cfg.T, 1024)})
    if cfg.fwd_only:
        n = s.get("seqs", cfg.n_seqs)
        d = W.make_decode(W.scaled(cfg, n_seqs=n), "cpu", seed)
        keys = W.count_pairs(d["idx"], cfg.bs, 1, 0, kv_lens=d["kv_lens"])
        q, k, v = d["q"].float(), d["k"].float(), d["v"].float()

        def run_decode():
            t0 = time.perf_counter()
            O.sfa_forward(q, k, v, d["idx"], cfg.bs, cfg.scale, None, True, d["cu_q"], d["cu_k"])
            return time.perf_counter() - t0, keys * (cfg.Dqk + cfg.Dv) * 2.0
        return run_decode
    G = cfg.Hq // cfg.Hk
    one = W.scaled(cfg, B=1, Hq=G, Hk=1)
    d = W.make_inputs(one, "cpu", seed, dtype=torch.bfloat16)
    n_tok = min(cfg.T, s["last"])
    t0 = cfg.T - n_tok
    q = d["q"][:, t0:].float()
    k, v = d["k"].float(), d["v"].float()
    idx = d["idx"][:, t0:]
    do = d["do"][:, t0:].float()
    pairs = W.count_pairs(idx, cfg.bs, n_tok, cfg.T) * G
    flops = W.sfa_flops(pairs, cfg.Dqk, cfg.Dv).total

    def run():
        t1 = time.perf_counter()
        o, lse = O.sfa_forward(q, k, v, idx, cfg.bs, cfg.scale, None, cfg.causal)
        O.sfa_backward(q, k, v, idx, o, lse, do, cfg.bs, cfg.scale, None, cfg.causal)
        return time.perf_counter() - t1, flops
    return run


def cpu_sample_run(cfg, seed=0):
    """One CPU sample (inputs of `seed`); returns (seconds, work)."""
    return cpu_sample_prepare(cfg, seed)()


def cpu_unit(cfg):
    return ("GB/s", 1e9) if cfg.fwd_only else ("TFLOP/s", 1e12)


def cpu_baseline(cfg, min_s=10.0, max_reps=8):
    """The fixed sample (seed 0), run again until `min_s` seconds of CPU work
    (or `max_reps` runs) are timed: total work / total time.  The inputs are
    generated once, outside the timed runs."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    run = cpu_sample_prepare(cfg, seed=0)
    tt, ww, reps = 0.0, 0.0, 0
    while reps < max_reps and (reps == 0 or tt < min_s):
        dt, w = run()
        tt += dt
        ww += w
        reps += 1
    unit, div = cpu_unit(cfg)
    return {"value": ww / tt / div, "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{cpu_sample_desc(cfg)}; seed 0, {reps} timed runs, {tt:.1f} s"}


def run_reference(args, cfg):
    """The reference arm: the CPU restatement on the same sample rule as
    cpu_baseline, one sample per step (seed = step index)."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    for i in range(args.warmup):
        cpu_sample_run(cfg, seed=i)
    tot_t, tot_w = 0.0, 0.0
    for i in range(args.steps):
        dt, w = cpu_sample_run(cfg, seed=i)
        tot_t += dt
        tot_w += w
    unit, div = cpu_unit(cfg)
    v = tot_w / tot_t / div
    split = resolve_split(args, cfg, args.gpus)
    line = {"impl": "reference", "metric": DECODE_METRIC if cfg.fwd_only else METRIC, "value": v, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * tot_t / args.steps, "higher_is_better": True,
            "scaling": scaling_kind(split), "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": config_dict(cfg, args.gpus, split, args.balance),
            "cpu_baseline": {"value": v, "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"per step: {cpu_sample_desc(cfg)}"},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# splits
# ---------------------------------------------------------------------------
def unit_range(cfg, world, rank):
    """(b0, b1, h0, h1) of rank's (batch, kv head) units, or None when the
    units do not deal out evenly as whole batches or kv-head groups."""
    units = cfg.B * cfg.Hk
    if units % world:
        return None
    per = units // world
    u0 = rank * per
    if per % cfg.Hk == 0:
        b0 = u0 // cfg.Hk
        return b0, b0 + per // cfg.Hk, 0, cfg.Hk
    if cfg.Hk % per == 0:
        b0, h0 = divmod(u0, cfg.Hk)
        return b0, b0 + 1, h0, h0 + per
    return None


def resolve_split(args, cfg, world):
    if world == 1:
        return "none"
    if args.split != "auto":
        return args.split
    if cfg.fwd_only:
        return "units"
    return "units" if unit_range(cfg, world, 0) is not None else "query"


def rank_seed(rank: int) -> int:
    """Seed of a rank's inputs under --split batch (each rank its own batch);
    the other splits give every rank the inputs of rank 0."""
    return 1000 + rank


def reduce_over_ranks(step_ms, e2e_ms, work, device):
    """Whole-job figures: the slowest rank's step and e2e times, the work of
    all ranks.  One MAX and one SUM all-reduce, the same on every rank."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(step_ms), float(e2e_ms), float(work)
    t = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    f = torch.tensor([work], dtype=torch.float64, device=device)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(f[0])


def scaling_kind(split):
    return "weak" if split == "batch" else "strong"


def config_dict(cfg, n, split, balance="cost", paged=False):
    if cfg.fwd_only:
        return {"workload": f"{cfg.name}: varlen decode forward, {cfg.n_seqs} sequences x 1 query, kv "
                            f"lengths U[{cfg.kv_min}, {cfg.kv_max}], Hq={cfg.Hq}, Hk={cfg.Hk}, Dqk={cfg.Dqk}, "
                            f"Dv={cfg.Dv}, block_size={cfg.bs}, S={cfg.S} uniform blocks, q/k/v ~ N(0,1)"
                            + (f", paged kv cache ({cfg.bs}-row pages at shuffled pool places, block table)"
                               if paged else ""),
                "global_batch": cfg.n_seqs,
                "parallelism": "single GPU" if n == 1 else f"{n} ranks x {cfg.n_seqs // n} sequences",
                "l2": "flushed between timed steps (256 MiB memset)"}
    per = "/rank" if split == "batch" else ""
    par = {"none": "single GPU",
           "units": f"{n} ranks x {cfg.B * cfg.Hk // max(n, 1)} (batch, kv head) units each, no collective",
           "batch": f"dp{n} (every rank its own batch)",
           "query": (f"{n} query-row ranges balanced by "
                     + ("the job-aware cost (shard.row_cost)" if balance == "cost" else "selected pairs")
                     + ", dK/dV summed by one reduce-scatter")}[split]
    sel = {"uniform": "uniform causal", "recent": "recent-biased causal", "token": "token-level causal top-k",
           "decode": "uniform"}[cfg.mode]
    return {"workload": f"{cfg.name}: sparse attention fwd+bwd, B={cfg.B}{per}, T={cfg.T}, Hq={cfg.Hq}, "
                        f"Hk={cfg.Hk}, Dqk={cfg.Dqk}, Dv={cfg.Dv}, block_size={cfg.bs}, S={cfg.S}, {sel} "
                        "selection, q/k/v/dO ~ N(0,1)",
            "global_batch": cfg.B * n if split == "batch" else cfg.B, "seq_len": cfg.T,
            "parallelism": par, "l2": "flushed between timed steps (256 MiB memset)"}


# ---------------------------------------------------------------------------
# GPU arm: one fwd+bwd configuration
# ---------------------------------------------------------------------------
def kernel_flops(name, P, cfg, fl, fused_dq):
    """Algorithmic FLOPs a kernel owns (recomputation not counted).  With the
    fused dQ the key-centric pass performs every backward product (S, dP, dQ,
    dK, dV); the separate dQ pass owns S, dP and dQ, leaving dK and dV; the
    two-pass token-level backward's first pass owns S and dP, its gradient
    half dQ, dK and dV."""
    two_p = 2.0 * P
    if name.startswith("fwd_"):
        return fl.fwd
    if name == "bwd_dq_tc":
        return two_p * (2 * cfg.Dqk + cfg.Dv)
    if name == "bwd_dkdv_tc":
        return fl.bwd if fused_dq else two_p * (cfg.Dqk + cfg.Dv)
    if name in ("bwd_general", "bwd_tok"):
        return fl.bwd
    # the two-pass token-level backward: S and dP in the first pass, dQ, dK and
    # dV in the gradient half
    if name == "bwd_mla_sdp":
        return two_p * (cfg.Dqk + cfg.Dv)
    if name in ("bwd_tok_grad", "bwd_mla_grad"):
        return two_p * (2 * cfg.Dqk + cfg.Dv)
    return 0.0


def smem_port(cfg, pairs, ms, clocks):
    """The query-centric block-sparse forward's shared-memory traffic, modelled
    from its tiles: per (row, kv head, selected key) the N = G MMAs read the K
    and V rows as A operands (2·Dqk + 2·Dv bytes) and G·(Dqk + Dv)·2/128 bytes
    of Q^T / P^T as B, the gathers write the K and V rows (2·(Dqk + Dv)) and the
    softmax writes 2·G bytes of P.  Against the port's 128 B/clk on every SM."""
    G = cfg.Hq // cfg.Hk
    per_key = 4 * (cfg.Dqk + cfg.Dv) + 2 * G * (cfg.Dqk + cfg.Dv) / 128 + 2 * G
    nbytes = pairs / G * per_key
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    import torch
    peak = 128 * torch.cuda.get_device_properties(0).multi_processor_count * mhz * 1e6 / 1e12
    ach = nbytes / (ms * 1e-3) / 1e12
    return {"kernel": "fwd_tc", "bytes_per_launch": nbytes, "bytes_per_row_key": per_key, "achieved_tbs": ach,
            "peak_tbs": peak, "frac": ach / peak, "source": "modelled from the kernel's tiles (128 B/clk/SM)"}


def measure_config(args, cfg, world, rank, dev, split, steps, warmup, primary):
    import torch
    import torch.distributed as dist

    from ops_b200 import _lib
    from ops_b200 import sfa as S
    from ops_b200 import workloads as W

    lib = _lib.load()
    d = W.make_inputs(cfg, dev, seed=rank_seed(rank if split == "batch" else 0))
    q, k, v, idx, do = d["q"], d["k"], d["v"], d["idx"], d["do"]
    if getattr(args, "as_tokens", False) and cfg.bs > 1:
        # the same selected keys as token-level indices: runs the token-level
        # kernels (query-centric dK/dV with fp32 reductions) on this workload
        idx = W.blocks_to_tokens(idx, cfg.bs)
        cfg = W.scaled(cfg, bs=1, S=cfg.S * cfg.bs, name=cfg.name + "-as-tokens")
    v_view = v.data_ptr() == k.data_ptr()            # v = kv[..., :Dv] (MLA latent)
    T = cfg.T
    r0, r1, ke = 0, T, T
    b0, b1, h0, h1 = 0, cfg.B, 0, cfg.Hk
    G = cfg.Hq // cfg.Hk
    if split == "units":
        b0, b1, h0, h1 = unit_range(cfg, world, rank)
        q, do = q[b0:b1, :, h0 * G:h1 * G], do[b0:b1, :, h0 * G:h1 * G]
        k, v, idx = k[b0:b1, :, h0:h1], v[b0:b1, :, h0:h1], idx[b0:b1, :, h0:h1]
    elif split == "query":
        from ops_b200 import shard
        work = (shard.row_cost(idx, cfg.bs, T) if args.balance == "cost" else shard.row_work(idx, cfg.bs, T))
        r0, r1 = shard.query_ranges(work, world)[rank]
        ke = r1
        q, idx, do = q[:, r0:r1], idx[:, r0:r1], do[:, r0:r1]
        k, v = k[:, :ke], v[:, :ke]
    units = (b1 - b0) * (h1 - h0)
    pairs = W.count_pairs(idx, cfg.bs, r1 - r0, ke) * G
    fl = W.sfa_flops(pairs, cfg.Dqk, cfg.Dv)
    o = torch.empty(*q.shape[:-1], cfg.Dv, dtype=q.dtype, device=dev)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=dev)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    # v = kv[..., :Dv] (c4, tok128): one kv tensor, one gradient dk + dv (the
    # library sums them in fp32 when dk and dv alias)
    dv = dk if v_view else torch.empty_like(v)
    scfg = S._Cfg(cfg.bs, cfg.scale, cfg.causal, False, r1 - r0, ke, _lib.SFA_DKV_AUTO, _lib.SFA_KERNEL_AUTO,
                  False, S._DQ[args.dq_mode])
    P = S.build_params(q, k, v, idx, o, lse, scfg, None, None, None, do, dq, dk, dv, None)
    Pp = ctypes.byref(P)
    fam_f = lib.sfa_select_kernel(Pp, 0)
    fam_b = lib.sfa_select_kernel(Pp, 1)
    _lib.check(min(0, fam_f), "select fwd")
    _lib.check(min(0, fam_b), "select bwd")
    dkv_mode, dq_mode = ctypes.c_int32(), ctypes.c_int32()
    _lib.check(min(0, lib.sfa_bwd_plan(Pp, ctypes.byref(dkv_mode), ctypes.byref(dq_mode))), "plan")
    fused_dq = dq_mode.value == _lib.SFA_DQ_FUSED
    nbytes = lib.sfa_bwd_workspace_bytes(Pp)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    if split == "query":
        tc = (T + world - 1) // world
        # fp32 dK | dV per key (one dK + dV of the latent's dims when v is k's view)
        width = cfg.Dqk if v_view else cfg.Dqk + cfg.Dv
        rs_in = torch.zeros(world * tc, cfg.B, cfg.Hk, width, dtype=torch.float32, device=dev)
        rs_out = torch.empty(tc, cfg.B, cfg.Hk, width, dtype=torch.float32, device=dev)

    def step():
        _lib.check(lib.sfa_fwd(Pp, None, 0, sptr), "sfa_fwd")
        _lib.check(lib.sfa_bwd_preprocess(Pp, ws.data_ptr(), nbytes, sptr), "preprocess")
        _lib.check(lib.sfa_bwd_dq(Pp, ws.data_ptr(), nbytes, sptr), "dq")
        _lib.check(lib.sfa_bwd_dkdv(Pp, ws.data_ptr(), nbytes, sptr), "dkdv")
        if split == "query":
            rs_in[:ke, ..., :cfg.Dqk].copy_(dk.transpose(0, 1))
            if not v_view:
                rs_in[:ke, ..., cfg.Dqk:].copy_(dv.transpose(0, 1))
            dist.reduce_scatter_tensor(rs_out, rs_in)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # events: one before the step, then one after each library operation (trace)
    NEV = 48
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    tr = [[torch.cuda.Event(enable_timing=True) for _ in range(NEV)] for _ in range(steps)]
    for e in starts + ends + [x for row in tr for x in row]:
        e.record(stream)                      # creates the handles
    torch.cuda.synchronize()
    handles = [(ctypes.c_void_p * NEV)(*[e.cuda_event for e in row]) for row in tr]
    sampler = None
    if primary:
        sampler = ClockSampler(torch.cuda.current_device())
        sampler.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    counts, names = [], []
    n0 = lib.sfa_kernel_launches()
    t_wall0 = time.time()
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        lib.sfa_launch_trace(handles[i], NEV)
        step()
        counts.append(lib.sfa_launch_trace_count())
        names.append([lib.sfa_launch_trace_name(j).decode() for j in range(counts[-1])])
        lib.sfa_launch_trace(None, 0)
        ends[i].record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    n1 = lib.sfa_kernel_launches()
    if world > 1:
        dist.barrier()
    step_ms = sum(starts[i].elapsed_time(ends[i]) for i in range(steps)) / steps
    kern_ms = {}
    for i in range(steps):
        prev = starts[i]
        for j in range(counts[i]):
            kern_ms[names[i][j]] = kern_ms.get(names[i][j], 0.0) + prev.elapsed_time(tr[i][j]) / steps
            prev = tr[i][j]
        if split == "query":
            kern_ms["dkdv_reduce_scatter"] = kern_ms.get("dkdv_reduce_scatter", 0.0) + \
                prev.elapsed_time(ends[i]) / steps

    e2e_ms, h2d, d2h = e2e_pipeline(args, cfg, d, split, (b0, b1, h0, h1), (r0, r1, ke), world, rank, dev,
                                    stream, flush, v_view, steps=max(1, min(steps, 5)))
    clocks = None
    if sampler is not None:
        sampler.stop()
        clocks = sampler.summary(t_wall0, t_wall1)

    per_rank = None
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {kk: round(vv, 4) for kk, vv in kern_ms.items()})
    step_max, e2e_max, flops_all = reduce_over_ranks(step_ms, e2e_ms, fl.total, dev)
    if rank != 0:
        return None

    peak, _, peak_kind = peaks()
    fams = {1: "tcgen05", 2: "general"}
    kernels = {}
    for name, ms in sorted(kern_ms.items(), key=lambda x: -x[1]):
        f = kernel_flops(name, pairs, cfg, fl, fused_dq)
        ent = {"ms": round(ms, 4), "share": round(ms / step_ms, 4)}
        if f:
            ach_k = f / (ms * 1e-3) / 1e12
            ent.update(tflops=round(ach_k, 2), frac=round(ach_k / peak, 4))
        kernels[name] = ent
    dom = max((n for n in kern_ms if not n.startswith("memset") and n != "dkdv_reduce_scatter"),
              key=lambda n: kern_ms[n])
    dom_f = kernel_flops(dom, pairs, cfg, fl, fused_dq)
    ach = dom_f / (kern_ms[dom] * 1e-3) / 1e12 if dom_f else 0.0
    traffic = tsrc = None
    if cfg.name == "c2" and dom in NCU_TRAFFIC_C2_B1 and cfg.T == 8192 and split in ("none", "units", "batch"):
        traffic = NCU_TRAFFIC_C2_B1[dom] * units / 4.0
        tsrc = (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one {dom} launch at c2 B=1 (4 units), "
                f"x{units}/4 for this launch's {units} units (profiles/)")
    fwd_name = next((n for n in kern_ms if n.startswith("fwd_")), None)
    # K/V rows the query-centric forward gathers: selected keys x (Dqk + Dv) bf16 per (row, kv head)
    gather = pairs / G * (cfg.Dqk + cfg.Dv) * 2.0
    value = flops_all / (step_max * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": step_max, "higher_is_better": True,
        "scaling": scaling_kind(split), "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(cfg, world, split, args.balance),
        "pct_bf16_peak": 100.0 * value / world / peak,
        "tokens_per_s": cfg.B * cfg.T * (world if split == "batch" else 1) / (step_max * 1e-3),
        "selected_pairs_rank0": pairs,
        "kernels": kernels,
        **({"kernels_ms_per_rank": per_rank} if per_rank else {}),
        "kernel_family": {"fwd": fams.get(fam_f, str(fam_f)), "bwd": fams.get(fam_b, str(fam_b)),
                          "dkv": {1: "inverted", 2: "atomic"}.get(dkv_mode.value),
                          "dq": {1: "separate", 2: "fused"}.get(dq_mode.value)},
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                     "frac": ach / peak, "peak_kind": f"{peak_kind} bf16 burst (kernels timed alone, a few ms)",
                     "traffic": traffic, "traffic_source": tsrc,
                     "algorithmic": f"{dom_f:.4g} FLOP per launch"},
        "gather": {"kernel": fwd_name, "bytes_per_launch": gather,
                   "achieved_tbs": gather / (kern_ms[fwd_name] * 1e-3) / 1e12 if fwd_name else None},
        **({"smem_port": smem_port(cfg, pairs, kern_ms["fwd_tc"], clocks)} if "fwd_tc" in kern_ms else {}),
        "e2e": {"value": flops_all / (e2e_max * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_max},
        "gpu_launches": int(n1 - n0),
    }
    if clocks is not None:
        line["clocks"] = clocks
    return line


def e2e_chunks(cfg, split, units):
    """The e2e pipeline's chunks: (batch, kv head, row0, row1, first, last)
    per chunk, or [None] for the query split (one chunk: the rank's rows).
    A configuration with fewer than 8 units (c3: 4, c4: 1) also cuts each
    unit's query rows into ranges, so the copies of one range overlap the
    kernels of another; ``first`` / ``last`` mark a unit's first and last
    range (its k / v go in with the first, its dk / dv come back after the
    last)."""
    if split == "query":
        return [None]
    b0, b1, h0, h1 = units
    n_units = (b1 - b0) * (h1 - h0)
    n_r = -(-8 // n_units) if n_units < 8 and cfg.T >= 8192 else 1
    return [(b, h, cfg.T * i // n_r, cfg.T * (i + 1) // n_r, i == 0, i == n_r - 1)
            for b in range(b0, b1) for h in range(h0, h1) for i in range(n_r)]


def e2e_pipeline(args, cfg, d, split, units, rows, world, rank, dev, stream, flush, v_view, steps):
    """Public-API step with host-resident inputs/outputs; returns (ms, h2d, d2h).

    The rank's share is cut into chunks (``e2e_chunks``: one (batch, kv
    head) unit each, or row ranges of a unit when units are few); chunk i's
    H2D copies run on one stream, its forward + backward on a second, its D2H
    copies on a third, so the PCIe traffic of neighbouring chunks overlaps the
    kernels (and H2D overlaps D2H).  Within a chunk the forward starts once
    q/k/v/idx are in (dO is still crossing) and o goes back while the backward
    runs, which shortens the last chunk's tail.  A row range takes keys
    [0, row1) (causal: every row keeps its position) and its dk / dv partial is
    added into the unit's fp32 sum, rounded to bf16 after the unit's last
    range."""
    import torch

    import ops_b200
    from ops_b200 import shard
    r0, r1, ke = rows
    G = cfg.Hq // cfg.Hk
    q, k, v, idx, do = d["q"], d["k"], d["v"], d["idx"], d["do"]
    chunks = e2e_chunks(cfg, split, units)

    def pin(t):
        return t.contiguous().cpu().pin_memory()

    host, dbuf, outs, unit_of = [], [], [], []
    unit_dev, unit_acc = {}, {}
    for c in chunks:
        if c is None:   # query split: this rank's rows and visible keys
            hs = dict(q=pin(q[:, r0:r1]), k=pin(k[:, :ke]), idx=pin(idx[:, r0:r1]), do=pin(do[:, r0:r1]))
            if not v_view:
                hs["v"] = pin(v[:, :ke])
            db = {n: torch.empty(t.shape, dtype=t.dtype, device=dev) for n, t in hs.items()}
            k0, k1 = shard.key_share(cfg.T, world, rank)
            kv_sh = (cfg.B, k1 - k0, cfg.Hk)
            o_sh = tuple(hs["q"].shape[:-1]) + (cfg.Dv,)
            od = dict(o=torch.empty(o_sh, dtype=q.dtype, pin_memory=True),
                      dq=torch.empty(tuple(hs["q"].shape), dtype=q.dtype, pin_memory=True),
                      dk=torch.empty(kv_sh + (cfg.Dqk,), dtype=k.dtype, pin_memory=True))
            if not v_view:
                od["dv"] = torch.empty(kv_sh + (cfg.Dv,), dtype=v.dtype, pin_memory=True)
            unit_of.append(None)
        else:
            b, h, c0, c1, first, last = c
            hs = dict(q=pin(q[b:b + 1, c0:c1, h * G:(h + 1) * G]), idx=pin(idx[b:b + 1, c0:c1, h:h + 1]),
                      do=pin(do[b:b + 1, c0:c1, h * G:(h + 1) * G]))
            if first:   # the unit's keys go in once, with its first range
                hs["k"] = pin(k[b:b + 1, :, h:h + 1])
                if not v_view:
                    hs["v"] = pin(v[b:b + 1, :, h:h + 1])
            db = {n: torch.empty(t.shape, dtype=t.dtype, device=dev) for n, t in hs.items()}
            if first:
                unit_dev[(b, h)] = db
                if not last:   # ranges: fp32 sums of the dk / dv partials
                    unit_acc[(b, h)] = {n: torch.empty(db[n].shape, dtype=torch.float32, device=dev)
                                        for n in (("k",) if v_view else ("k", "v"))}
            od = dict(o=torch.empty(tuple(hs["q"].shape[:-1]) + (cfg.Dv,), dtype=q.dtype, pin_memory=True),
                      dq=torch.empty(tuple(hs["q"].shape), dtype=q.dtype, pin_memory=True))
            if last:
                kdev = unit_dev[(b, h)]
                od["dk"] = torch.empty(tuple(kdev["k"].shape), dtype=k.dtype, pin_memory=True)
                if not v_view:
                    od["dv"] = torch.empty(tuple(kdev["v"].shape), dtype=v.dtype, pin_memory=True)
            unit_of.append((b, h))
        host.append(hs)
        dbuf.append(db)
        outs.append(od)
    h2d = sum(t.numel() * t.element_size() for hs in host for t in hs.values())
    d2h = sum(t.numel() * t.element_size() for od in outs for t in od.values())
    s_in, s_c, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def one_step():
        keep = []
        start = torch.cuda.Event()
        start.record(stream)
        for s in (s_in, s_c, s_out):
            s.wait_event(start)
        fwd_ev, bwd_ev = [], []   # per chunk: forward inputs in / dO in
        for hs, db in zip(host, dbuf):
            with torch.cuda.stream(s_in):
                for n in hs:
                    if n != "do":
                        db[n].copy_(hs[n], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                fwd_ev.append(e)
                db["do"].copy_(hs["do"], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                bwd_ev.append(e)
        for i, (c, db, od) in enumerate(zip(chunks, dbuf, outs)):
            res = []
            with torch.cuda.stream(s_c):
                s_c.wait_event(fwd_ev[i])
                if c is None:
                    s_c.wait_event(bwd_ev[i])
                    r = shard.local_step(db["q"], db["k"], db["k"][..., :cfg.Dv] if v_view else db["v"], db["idx"],
                                         db["do"], (r0, r1), cfg.T, rank, world, cfg.bs, cfg.scale)
                    res = [("o", r["o"]), ("dq", r["dq"]), ("dk", r["dk"])] + \
                        ([] if v_view else [("dv", r["dv"])])
                else:
                    _, _, c0, c1, first, last = c
                    kd = unit_dev[unit_of[i]]
                    acc = unit_acc.get(unit_of[i])
                    ke_c = c1 if cfg.causal else cfg.T   # causal: rows < c1 see no key past c1
                    qg = db["q"].detach().requires_grad_()
                    kg = kd["k"][:, :ke_c].detach().requires_grad_()
                    vg = kg[..., :cfg.Dv] if v_view else kd["v"][:, :ke_c].detach().requires_grad_()
                    oo, _ = ops_b200.sparse_flash_attention(qg, kg, vg, db["idx"], cfg.bs, cfg.scale,
                                                            causal=cfg.causal, dq_mode=args.dq_mode)
                    e_fwd = torch.cuda.Event()
                    e_fwd.record(s_c)
                    with torch.cuda.stream(s_out):   # o leaves while the backward runs
                        s_out.wait_event(e_fwd)
                        od["o"].copy_(oo.detach(), non_blocking=True)
                    s_c.wait_event(bwd_ev[i])
                    oo.backward(db["do"])
                    res = [("o", oo.detach()), ("dq", qg.grad)]
                    grads = [("k", kg.grad)] + ([] if v_view else [("v", vg.grad)])
                    if acc is not None:   # a row range: add this partial to the unit's fp32 sum
                        for n, g in grads:
                            if first:
                                acc[n].zero_()
                            acc[n][:, :ke_c] += g
                        if last:
                            grads = [(n, acc[n].to(k.dtype)) for n, _ in grads]
                    if last:
                        res += [("d" + n, g) for n, g in grads]
                    else:
                        res += [("_" + n, g) for n, g in grads]   # kept alive until the step ends
                e = torch.cuda.Event()
                e.record(s_c)
            keep.append(res)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e)
                for n, t in res:
                    if n in od and (c is None or n != "o"):
                        od[n].copy_(t, non_blocking=True)
        end = torch.cuda.Event()
        end.record(s_out)
        stream.wait_event(end)
        return keep

    one_step()
    torch.cuda.synchronize()
    ms = 0.0
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        keep = one_step()
        b.record(stream)
        torch.cuda.synchronize()
        del keep
        ms += a.elapsed_time(b)
    return ms / steps, h2d, d2h


# ---------------------------------------------------------------------------
# GPU arm: decode (forward-only, HBM-bound)
# ---------------------------------------------------------------------------
def measure_decode(args, cfg, world, rank, dev, steps, warmup, primary):
    import torch
    import torch.distributed as dist

    import ops_b200
    from ops_b200 import _lib
    from ops_b200 import sfa as S
    from ops_b200 import workloads as W

    lib = _lib.load()
    # the sequences are dealt out evenly: every rank draws its own share
    n_local = cfg.n_seqs // world if cfg.n_seqs % world == 0 else cfg.n_seqs
    local_cfg = W.scaled(cfg, n_seqs=n_local)
    d = W.make_decode(local_cfg, dev, seed=rank_seed(rank))
    q, k, v, idx, cu_q, cu_k = d["q"], d["k"], d["v"], d["idx"], d["cu_q"], d["cu_k"]
    keys = W.count_pairs(idx, cfg.bs, 1, 0, kv_lens=d["kv_lens"])
    G = cfg.Hq // cfg.Hk
    gathered = keys * (cfg.Dqk + cfg.Dv) * 2.0
    o = torch.empty(q.shape[0], cfg.Hq, cfg.Dv, dtype=q.dtype, device=dev)
    lse = torch.empty(q.shape[0], cfg.Hq, dtype=torch.float32, device=dev)
    scfg = S._Cfg(cfg.bs, cfg.scale, True, True, 1, d["max_k"], _lib.SFA_DKV_AUTO, _lib.SFA_KERNEL_AUTO, False)
    paged = getattr(args, "paged", False)
    if paged:
        # the same cache as 64-row pages at shuffled places of one pool, reached
        # through a block table (the serving layout)
        kp, vp, table = W.page_kv(k, v, cu_k, cfg.bs, seed=rank_seed(rank) + 1)
        del d["k"], d["v"], k, v
        torch.cuda.empty_cache()
        k = kp.view(-1, *kp.shape[2:])
        v = vp.view(-1, *vp.shape[2:])
    P = S.build_params(q, k, v, idx, o, lse, scfg, None, cu_q, cu_k)
    if paged:
        P.block_table, P.bt_stride, P.page_size = table.data_ptr(), table.stride(0), cfg.bs
    fam = lib.sfa_select_kernel(ctypes.byref(P), 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    for _ in range(warmup):
        _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, sptr), "sfa_fwd")
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = None
    if primary:
        sampler = ClockSampler(torch.cuda.current_device())
        sampler.start()
        time.sleep(0.3)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
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
    step_ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    # decode e2e: the KV cache is state that stays resident in HBM (as in
    # serving); a step's inputs from the host are the new queries and their
    # selected block ids, its output the attention rows
    host = {n: t.cpu().pin_memory() for n, t in (("q", q), ("idx", idx))}
    o_h = torch.empty(tuple(o.shape), dtype=o.dtype, pin_memory=True)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = o_h.numel() * o_h.element_size()
    cu_qd, cu_kd = cu_q.to(dev), cu_k.to(dev)

    def e2e_step():
        qd, ixd = (host[n].to(dev, non_blocking=True) for n in ("q", "idx"))
        if paged:
            oo, _ = ops_b200.sparse_flash_attention_paged(qd, kp, vp, ixd, table, d["kv_lens"], cfg.bs,
                                                          max_seqlen_q=1, max_seqlen_k=d["max_k"])
        else:
            oo, _ = ops_b200.sparse_flash_attention(qd, k, v, ixd, cfg.bs, cu_seqlens=cu_qd, cu_seqlens_k=cu_kd,
                                                    max_seqlen_q=1, max_seqlen_k=d["max_k"])
        o_h.copy_(oo, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e_ms = 0.0
    ne = max(1, min(steps, 3))
    for _ in range(ne):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        e_ms += a.elapsed_time(b)
    e_ms /= ne
    clocks = None
    if sampler is not None:
        sampler.stop()
        clocks = sampler.summary(t_wall0, t_wall1)
    step_max, e_max, bytes_all = reduce_over_ranks(step_ms, e_ms, gathered, dev)
    if rank != 0:
        return None
    _, hbm, kind = peaks()
    gbs = gathered / (step_ms * 1e-3) / 1e9
    line = {
        "metric": DECODE_METRIC, "value": bytes_all / (step_max * 1e-3) / 1e9,
        "unit": "GB/s", "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": step_max,
        "higher_is_better": True, "scaling": "strong" if n_local != cfg.n_seqs else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": config_dict(cfg, world, "units", paged=paged),
        "tflops": 2.0 * keys * G * (cfg.Dqk + cfg.Dv) / (step_ms * 1e-3) / 1e12,
        "kernel_family": {1: "tcgen05", 2: "general"}.get(fam, str(fam)),
        "roofline": {"bound": "hbm", "kernel": "fwd", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "peak_kind": f"{kind} copy", "traffic": None,
                     "algorithmic": "gathered K/V rows (selected keys x (Dqk + Dv) x 2 B) per launch"},
        "e2e": {"value": bytes_all / (e_max * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e_max, "kv_cache": "resident in HBM"},
        "gpu_launches": int(n1 - n0),
    }
    if clocks is not None:
        line["clocks"] = clocks
    return line


def families(cfg, dev):
    """Kernel families (fwd, bwd) the library picks for cfg's shape (asked on
    a short copy of it: the choice depends on head dims, group size,
    block_size and alignment, not on the length)."""
    import torch
    from ops_b200 import _lib
    from ops_b200 import sfa as S
    from ops_b200 import workloads as W
    small = W.scaled(cfg, B=1, T=256)
    d = W.make_inputs(small, dev, seed=0)
    o = torch.empty(*d["q"].shape[:-1], cfg.Dv, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(d["q"].shape[:-1], dtype=torch.float32, device=dev)
    c = S._Cfg(cfg.bs, cfg.scale, cfg.causal, False, small.T, small.T, _lib.SFA_DKV_AUTO, _lib.SFA_KERNEL_AUTO,
               False)
    P = S.build_params(d["q"], d["k"], d["v"], d["idx"], o, lse, c, None, None, None, d["do"],
                       torch.empty_like(d["q"]), torch.empty_like(d["k"]), torch.empty_like(d["v"]), None)
    lib = _lib.load()
    names = {_lib.SFA_KERNEL_TCGEN05: "tcgen05", _lib.SFA_KERNEL_GENERAL: "general"}
    return tuple(names.get(lib.sfa_select_kernel(ctypes.byref(P), b), "unsupported") for b in (0, 1))


def compact(line, cpu):
    """A secondary configuration's entry in the primary line."""
    keys = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "config", "kernel_family", "roofline",
            "e2e", "kernels", "pct_bf16_peak", "tflops", "gpu_launches")
    out = {k: line[k] for k in keys if k in line}
    out["cpu_baseline"] = cpu
    return out


def measure_indexer(dev, T=32768, H=64, D=128, topk=2048, steps=5, warmup=3):
    """The top-k token indexer on config 4's sequence (T = 32768, causal) with
    DeepSeek-V3.2's indexer shape (64 heads x 128 dims, top-2048): scoring
    FLOPs 2 * H * D per (query, key) pair, per-kernel CUDA-event times."""
    import torch

    from ops_b200 import _lib
    from ops_b200.indexer import lightning_indexer_topk

    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn(1, T, H, D, generator=g, device=dev).bfloat16()
    k = torch.randn(1, T, D, generator=g, device=dev).bfloat16()
    w = torch.rand(1, T, H, generator=g, device=dev) / H
    for _ in range(warmup):
        lightning_indexer_topk(q, k, w, topk)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    NEV = 32
    kern = {}
    tot = 0.0
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tr = [torch.cuda.Event(enable_timing=True) for _ in range(NEV)]
        for e in tr:
            e.record(stream)
        torch.cuda.synchronize()
        hs = (ctypes.c_void_p * NEV)(*[e.cuda_event for e in tr])
        a.record(stream)
        lib.sfa_launch_trace(hs, NEV)
        lightning_indexer_topk(q, k, w, topk)
        n = lib.sfa_launch_trace_count()
        names = [lib.sfa_launch_trace_name(j).decode() for j in range(n)]
        lib.sfa_launch_trace(None, 0)
        b.record(stream)
        torch.cuda.synchronize()
        tot += a.elapsed_time(b) / steps
        prev = a
        for j in range(n):
            kern[names[j]] = kern.get(names[j], 0.0) + prev.elapsed_time(tr[j]) / steps
            prev = tr[j]
    pairs = T * (T + 1) // 2
    flops = 2.0 * H * D * pairs
    peak, _, kind = peaks()
    sc = kern.get("indexer_score", 0.0)
    return {"workload": f"top-{topk} token indexer, B=1, T={T} causal, {H} heads x {D} dims (config 4's "
                        "sequence, DeepSeek-V3.2 indexer shape), q/k ~ N(0,1)",
            "ms_per_call": tot, "tflops": flops / (tot * 1e-3) / 1e12,
            "kernels": {n: round(m, 4) for n, m in kern.items()},
            "roofline": {"bound": "tensor", "kernel": "indexer_score", "achieved": flops / (sc * 1e-3) / 1e12,
                         "peak": peak, "unit": "TFLOP/s", "frac": flops / (sc * 1e-3) / 1e12 / peak,
                         "peak_kind": f"{kind} bf16 burst", "algorithmic": f"2*H*D per causal pair: {flops:.3e} FLOP"}}


def measure_fp8kv(dev, steps=5, warmup=3):
    """Config 4's forward (T = 32768, MLA) over the e4m3 latent cache against
    the bf16 cache, same indices; CUDA events per call, L2 flushed between."""
    import torch

    import ops_b200
    from ops_b200 import workloads as W

    cfg = W.CONFIGS["c4"]
    d = W.make_inputs(cfg, dev, seed=0, with_do=False)
    q, k, idx = d["q"], d["k"], d["idx"]
    kv8, sc = ops_b200.quantize_kv_fp8(k)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(warmup):
            fn()
        tot = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            tot += a.elapsed_time(b) / steps
        return tot

    bf = timed(lambda: ops_b200.sparse_flash_attention(q, k, k[..., :cfg.Dv], idx, 1))
    f8 = timed(lambda: ops_b200.sparse_flash_attention_fp8kv(q, kv8, sc, idx, cfg.Dv))
    pairs = W.count_pairs(idx, 1, cfg.T, cfg.T) * cfg.Hq
    fl = 2.0 * pairs * (cfg.Dqk + cfg.Dv)
    return {"workload": "c4 forward (T=32768, Hq=128 on one latent kv head, Dqk 576 / Dv 512, top-2048) over "
                        "an e4m3 cache with power-of-two row scales vs the bf16 cache",
            "bf16_ms": bf, "fp8_ms": f8, "bf16_tflops": fl / (bf * 1e-3) / 1e12, "fp8_tflops": fl / (f8 * 1e-3) / 1e12,
            "kv_cache_bytes": {"bf16": k.numel() * 2, "fp8": kv8.numel() + sc.numel() * 4}}


def run_ours(args, cfg):
    import datetime

    import torch
    import torch.distributed as dist
    from ops_b200 import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    split = resolve_split(args, cfg, world)
    if cfg.fwd_only:
        line = measure_decode(args, cfg, world, rank, dev, args.steps, args.warmup, True)
    else:
        line = measure_config(args, cfg, world, rank, dev, split, args.steps, args.warmup, True)
    others = []
    if world == 1 and args.configs != "none":
        others = [c for c in args.configs.split(",") if c and c != cfg.name]
    extra = {}
    for name in others:
        sub_cfg = W.CONFIGS[name]
        torch.cuda.empty_cache()
        if not sub_cfg.fwd_only and sub_cfg.T > 4096 and "general" in families(sub_cfg, dev):
            # the CUDA-core family would take minutes per step at full size
            sub_cfg = W.scaled(sub_cfg, T=2048)
        if sub_cfg.fwd_only:
            sub = measure_decode(args, sub_cfg, 1, 0, dev, 5, 3, False)
        else:
            sub = measure_config(args, sub_cfg, 1, 0, dev, "none", 3, 3, False)
        extra[name] = (sub, None if args.no_cpu else cpu_baseline(sub_cfg, min_s=2.0))
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg)
    if world == 1 and args.configs != "none":
        # the step before the op: the top-k indexer that produces token-level indices
        line["indexer"] = measure_indexer(torch.device("cuda", local))
        torch.cuda.empty_cache()
        # config 4's forward over an e4m3 latent kv cache
        line["fp8_kv"] = measure_fp8kv(torch.device("cuda", local))
    if extra:
        line["configs"] = {n: compact(s, c) for n, (s, c) in extra.items()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c2")
    ap.add_argument("--configs", default="c1,c3,c4,c5",
                    help="secondary configurations measured after the primary one at N=1 ('none' to skip)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline samples")
    ap.add_argument("--batch", type=int, default=0, help="override the batch (profiling runs)")
    ap.add_argument("--seq", type=int, default=0, help="override the sequence length (scaled secondary configs)")
    ap.add_argument("--dq-mode", choices=["auto", "separate", "fused"], default="auto",
                    help="backward dQ plan (profiling runs): its own query-centric pass or fused into dK/dV")
    ap.add_argument("--balance", choices=["pairs", "cost"], default="cost",
                    help="--split query: balance rows by selected pairs, or by a cost that also counts the "
                         "dK/dV pass's jobs and batches (ops_b200/shard.py row_cost)")
    ap.add_argument("--indexer", action="store_true",
                    help="measure only the top-k token indexer (config 4's sequence) and print its line")
    ap.add_argument("--fp8-kv", action="store_true",
                    help="measure only config 4's forward over an e4m3 latent kv cache against the bf16 cache")
    ap.add_argument("--paged", action="store_true",
                    help="decode configurations (c5): the kv cache as 64-row pages of a shuffled pool, reached "
                         "through a block table (sparse_flash_attention_paged)")
    ap.add_argument("--as-tokens", action="store_true",
                    help="expand a block-level configuration's indices to token level (the same selected keys), "
                         "so the token-level kernels and their query-centric dK/dV run on it")
    ap.add_argument("--split", choices=["auto", "units", "batch", "query"], default="auto",
                    help="with N > 1: 'units' deals (batch, kv head) units out to the ranks (strong scaling; "
                         "the default when they divide evenly), 'query' splits one batch's query rows "
                         "(strong scaling with one reduce-scatter; the default otherwise), 'batch' gives each "
                         "rank its own batch (weak scaling)")
    args = ap.parse_args()
    from ops_b200 import workloads as W
    cfg = W.CONFIGS[args.config]
    if args.batch:
        cfg = W.scaled(cfg, B=args.batch)
    if args.seq:
        cfg = W.scaled(cfg, T=args.seq)
    if args.batch or args.seq:
        args.configs = "none"
    if args.indexer or args.fp8_kv:
        import torch
        torch.cuda.set_device(0)
        out = measure_indexer(torch.device("cuda", 0)) if args.indexer else measure_fp8kv(torch.device("cuda", 0))
        print(json.dumps(out), flush=True)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
