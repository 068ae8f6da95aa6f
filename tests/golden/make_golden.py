"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that holds the reference source (read-only) at ``--ref``:

    python tests/golden/make_golden.py --ref <path to lilac-me/ops checkout>

Every case feeds seeded bf16 inputs through the reference's own
``SparseFlashAttentionTriton`` (forward + backward, executed under Triton's CPU
interpreter by ``ref_interp.py``) and stores inputs and outputs as ``.npz``.
Values are stored as float32 (bf16 inputs are exact in float32).

Cases:
* ``tok_*`` — the reference's native surface: SBHD, one shared kv head,
  token-level indices left-packed with a -1 tail, attention sink.  They cover the
  three tiling buckets (topk <= 128, <= 160, > 160; ``SFA.py:51-59``), a head
  count that is not a multiple of BLOCK_H = 32, and B > 1.
* ``gqa_block_causal`` — the generalised surface mapped onto the reference: per
  kv head g the reference runs on q heads [g*G, (g+1)*G) with kv = k = v of head g,
  block ids expanded to token ids, keys past the query position dropped, and
  valid entries left-packed (the reference reads only the first max-valid-count
  slots).  The stored inputs are the block-level ones; outputs are reassembled.
* ``mla_dv_lt_dqk`` — D_v < D_qk with v = kv[..., :D_v]: the reference runs on the
  full kv with dO zero-padded past D_v, which leaves o[..., :D_v], dq, and
  dk + pad(dv) unchanged.
* ``empty_row`` — one query with no valid entry: the reference returns o = 0 and
  lse = +inf (``SFA.py:381``, ``SFA.py:472``); recorded as a known divergence.
"""
from __future__ import annotations

import argparse
import math
import os
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16(shape, gen):
    return torch.randn(*shape, generator=gen).bfloat16()


def _packed_tok(S, B, K, S_kv, gen, lo=1):
    idx = torch.full((S, B, K), -1, dtype=torch.int32)
    for s in range(S):
        for b in range(B):
            n = int(torch.randint(lo, K + 1, (), generator=gen))
            idx[s, b, :n] = torch.randperm(S_kv, generator=gen)[:n].int()
    return idx


def _f32(t):
    return t.detach().float().numpy()


def case_tok(SFA, run, name, S, B, H, D, S_kv, K, seed, lo=1, full=False):
    gen = torch.Generator().manual_seed(seed)
    q = _bf16((S, B, H, D), gen)
    kv = _bf16((S_kv, B, D), gen)
    sink = torch.randn(H, generator=gen)
    if full:
        idx = torch.stack([torch.stack([torch.randperm(S_kv, generator=gen)[:K] for _ in range(B)])
                           for _ in range(S)]).int()
    else:
        idx = _packed_tok(S, B, K, S_kv, gen, lo)
    do = _bf16((S, B, H, D), gen)
    scale = 1.0 / math.sqrt(D)
    out, lse2, dq, dkv, dsink = run(SFA, q, kv, sink, idx, scale, do)
    return dict(kind="tok", q=_f32(q), kv=_f32(kv), sink=_f32(sink), idx=idx.numpy(), do=_f32(do),
                scale=np.float32(scale), out=_f32(out), lse2=_f32(lse2), dq=_f32(dq), dkv=_f32(dkv),
                dsink=_f32(dsink))


def case_gqa(SFA, run, seed=5, B=1, T=96, Hq=32, Hk=2, D=64, bs=16, S=3):
    gen = torch.Generator().manual_seed(seed)
    G = Hq // Hk
    q = _bf16((B, T, Hq, D), gen)
    kv = _bf16((B, T, Hk, D), gen)
    sink = torch.randn(Hq, generator=gen)
    do = _bf16((B, T, Hq, D), gen)
    bidx = torch.full((B, T, Hk, S), -1, dtype=torch.int32)
    for b in range(B):
        for t in range(T):
            cur = t // bs
            for h in range(Hk):
                others = torch.randperm(cur, generator=gen)[: S - 1] if cur > 0 else torch.empty(0, dtype=torch.int64)
                sel = torch.cat([torch.tensor([cur]), others]).int()
                perm = torch.randperm(len(sel), generator=gen)
                bidx[b, t, h, : len(sel)] = sel[perm]
    scale = 1.0 / math.sqrt(D)
    out = torch.zeros(B, T, Hq, D)
    lse2 = torch.zeros(B, T, Hq)
    dq = torch.zeros(B, T, Hq, D)
    dkv = torch.zeros(B, T, Hk, D)
    dsink = torch.zeros(Hq)
    for b in range(B):
        for g in range(Hk):
            hs = slice(g * G, (g + 1) * G)
            keys = bidx[b, :, g, :].long()[..., None] * bs + torch.arange(bs)          # [T,S,bs]
            ok = (bidx[b, :, g, :, None] >= 0) & (keys <= torch.arange(T)[:, None, None])
            keys, ok = keys.flatten(1), ok.flatten(1)
            tok = torch.full((T, 1, keys.shape[1]), -1, dtype=torch.int32)
            for t in range(T):
                sel = keys[t][ok[t]]
                tok[t, 0, : len(sel)] = sel.int()
            r = run(SFA, q[b, :, hs][:, None].contiguous(), kv[b, :, g][:, None].contiguous(),
                    sink[hs].contiguous(), tok, scale, do[b, :, hs][:, None].contiguous())
            out[b, :, hs] = r[0][:, 0].float()
            lse2[b, :, hs] = r[1][:, 0]
            dq[b, :, hs] = r[2][:, 0].float()
            dkv[b, :, g] = r[3][:, 0].float()
            dsink[hs] += r[4].float()
    return dict(kind="gqa", q=_f32(q), kv=_f32(kv), sink=_f32(sink), idx=bidx.numpy(), do=_f32(do),
                scale=np.float32(scale), block_size=np.int32(bs), out=_f32(out), lse2=_f32(lse2),
                dq=_f32(dq), dkv=_f32(dkv), dsink=_f32(dsink))


def case_mla(SFA, run, seed=7, S=4, B=1, H=16, Dqk=96, Dv=64, S_kv=64, K=16):
    gen = torch.Generator().manual_seed(seed)
    q = _bf16((S, B, H, Dqk), gen)
    kv = _bf16((S_kv, B, Dqk), gen)
    sink = torch.randn(H, generator=gen)
    idx = _packed_tok(S, B, K, S_kv, gen, lo=K // 2)
    do = _bf16((S, B, H, Dv), gen)
    do_pad = torch.cat([do, torch.zeros(S, B, H, Dqk - Dv, dtype=do.dtype)], -1)
    scale = 1.0 / math.sqrt(Dqk)
    out, lse2, dq, dkv, dsink = run(SFA, q, kv, sink, idx, scale, do_pad)
    return dict(kind="mla", q=_f32(q), kv=_f32(kv), sink=_f32(sink), idx=idx.numpy(), do=_f32(do),
                scale=np.float32(scale), d_v=np.int32(Dv), out=_f32(out[..., :Dv]), lse2=_f32(lse2),
                dq=_f32(dq), dkv=_f32(dkv), dsink=_f32(dsink))


def case_empty(SFA, run, seed=9, S=3, B=1, H=16, D=64, S_kv=48, K=8):
    gen = torch.Generator().manual_seed(seed)
    q = _bf16((S, B, H, D), gen)
    kv = _bf16((S_kv, B, D), gen)
    sink = torch.randn(H, generator=gen)
    idx = _packed_tok(S, B, K, S_kv, gen)
    idx[0] = -1
    do = _bf16((S, B, H, D), gen)
    scale = 1.0 / math.sqrt(D)
    out, lse2, dq, dkv, dsink = run(SFA, q, kv, sink, idx, scale, do)
    return dict(kind="tok", q=_f32(q), kv=_f32(kv), sink=_f32(sink), idx=idx.numpy(), do=_f32(do),
                scale=np.float32(scale), out=_f32(out), lse2=_f32(lse2), dq=_f32(dq), dkv=_f32(dkv),
                dsink=_f32(dsink))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="directory holding the reference SFA.py")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    import ref_interp
    SFA = ref_interp.load_reference(args.ref)
    run = ref_interp.run_reference
    cases = {
        "tok_bucket128": lambda: case_tok(SFA, run, "tok_bucket128", 6, 1, 16, 64, 96, 8, seed=1),
        "tok_bucket160": lambda: case_tok(SFA, run, "tok_bucket160", 3, 1, 32, 64, 200, 150, seed=2, full=True),
        "tok_bucket640": lambda: case_tok(SFA, run, "tok_bucket640", 4, 2, 20, 64, 300, 200, seed=3),
        "gqa_block_causal": lambda: case_gqa(SFA, run),
        "mla_dv_lt_dqk": lambda: case_mla(SFA, run),
        "empty_row": lambda: case_empty(SFA, run),
    }
    for name, fn in cases.items():
        if args.only and name != args.only:
            continue
        t0 = time.time()
        d = fn()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print(f"{name}: {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
