"""Seeded synthetic inputs for the benchmark configurations of the SFA op.

No public dataset is involved: every configuration is q/k/v/dO ~ N(0, 1) with
index tensors drawn as the configuration describes.  Generation runs on any
torch device (chunked, so the 32k x 32k token-level draw of the MLA config does
not materialise at once).

Configurations (same numbering as the benchmark):
  c1  B1  T1024  Hq16 Hk1 D64       bs64 S8   causal, uniform w/o replacement
  c2  B4  T8192  Hq64 Hk4 D128      bs64 S16  causal, current block always in
  c3  B1  T65536 Hq64 Hk4 D128      bs64 S32  half the mass on the last 8 blocks
  c4  B1  T32768 Hq128 Hk1 Dqk576 Dv512 bs1 k2048 token-level, causal; one
      latent kv tensor (k), v = k[..., :512] (a view)
  c5  128 seqs, kv U[4096,131072], 1 query each, Hq64 Hk8 D128 bs64 S32 (forward only)
  tok128  B1 T8192 Hq128 Hk1 D128 bs1 k2048, one shared kv tensor (the reference
      op's own mode; not a BASELINE configuration)
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional

import torch


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    T: int
    Hq: int
    Hk: int
    Dqk: int
    Dv: int
    bs: int
    S: int
    mode: str            # "uniform" | "recent" | "token" | "decode"
    causal: bool = True
    n_seqs: int = 0      # decode: number of sequences
    kv_min: int = 0
    kv_max: int = 0
    fwd_only: bool = False

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.Dqk)


CONFIGS = {
    "c1": Config("c1", 1, 1024, 16, 1, 64, 64, 64, 8, "uniform"),
    "c2": Config("c2", 4, 8192, 64, 4, 128, 128, 64, 16, "uniform"),
    "c3": Config("c3", 1, 65536, 64, 4, 128, 128, 64, 32, "recent"),
    "c4": Config("c4", 1, 32768, 128, 1, 576, 512, 1, 2048, "token"),
    "c5": Config("c5", 128, 1, 64, 8, 128, 128, 64, 32, "decode", n_seqs=128, kv_min=4096, kv_max=131072,
                 fwd_only=True),
    # not a BASELINE configuration: the reference op's own operating mode
    # (SparseFlashAttentionTriton: one kv tensor whose rows are keys and values,
    # token-level top-k) at D = 128, for the token-level kernels' measurements
    "tok128": Config("tok128", 1, 8192, 128, 1, 128, 128, 1, 2048, "token"),
}


def scaled(cfg: Config, **kw) -> Config:
    """A smaller copy of a configuration with the same index distribution."""
    return replace(cfg, **kw)


def _causal_blocks(gen, device, T, nb_total, S, bs, mode, t0, t1):
    """Block ids [t1-t0, S] for queries t0..t1-1 of one (batch, kv head)."""
    t = torch.arange(t0, t1, device=device)
    cur = t // bs                                             # current block
    j = torch.arange(nb_total, device=device)
    u = torch.rand(t1 - t0, nb_total, generator=gen, device=device).clamp_min(1e-12)
    if mode == "recent":
        # weighted sampling without replacement (exponential race): the last 8
        # blocks carry half the weight, the older blocks the other half
        recent = (j[None, :] > cur[:, None] - 8) & (j[None, :] <= cur[:, None])
        n_old = (cur - 7).clamp_min(0).to(torch.float32)
        w = torch.where(recent, torch.full_like(u, 0.5 / 8),
                        0.5 / n_old.clamp_min(1.0)[:, None].expand_as(u))
        key = -torch.log(u) / w
    else:
        key = u
    valid = j[None, :] <= cur[:, None]
    key = torch.where(valid, key, torch.full_like(key, float("inf")))
    key = torch.where(j[None, :] == cur[:, None], torch.full_like(key, -1.0), key)   # current block always in
    k = min(S, nb_total)
    val, sel = torch.topk(key, k, dim=1, largest=False)
    sel = torch.where(torch.isfinite(val), sel, torch.full_like(sel, -1))
    if k < S:
        sel = torch.cat([sel, torch.full((sel.shape[0], S - k), -1, dtype=sel.dtype, device=device)], 1)
    return sel.to(torch.int32)


def _token_topk(gen, device, T, K, t0, t1):
    t = torch.arange(t0, t1, device=device)
    j = torch.arange(T, device=device)
    u = torch.rand(t1 - t0, T, generator=gen, device=device)
    u = torch.where(j[None, :] <= t[:, None], u, torch.full_like(u, float("inf")))
    k = min(K, T)
    val, sel = torch.topk(u, k, dim=1, largest=False)
    sel = torch.where(torch.isfinite(val), sel, torch.full_like(sel, -1))
    if k < K:
        sel = torch.cat([sel, torch.full((sel.shape[0], K - k), -1, dtype=sel.dtype, device=device)], 1)
    return sel.to(torch.int32)


def make_indices(cfg: Config, device="cpu", seed=0, chunk=1024):
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    if cfg.mode == "token":
        idx = torch.empty(cfg.B, cfg.T, cfg.Hk, cfg.S, dtype=torch.int32, device=device)
        ch = max(1, (1 << 24) // max(cfg.T, 1))
        for b in range(cfg.B):
            for h in range(cfg.Hk):
                for t0 in range(0, cfg.T, ch):
                    idx[b, t0:t0 + ch, h] = _token_topk(gen, device, cfg.T, cfg.S, t0, min(cfg.T, t0 + ch))
        return idx
    nb = (cfg.T + cfg.bs - 1) // cfg.bs
    idx = torch.empty(cfg.B, cfg.T, cfg.Hk, cfg.S, dtype=torch.int32, device=device)
    ch = max(1, min(chunk, (1 << 24) // max(nb, 1)))
    for b in range(cfg.B):
        for h in range(cfg.Hk):
            for t0 in range(0, cfg.T, ch):
                idx[b, t0:t0 + ch, h] = _causal_blocks(gen, device, cfg.T, nb, cfg.S, cfg.bs, cfg.mode, t0,
                                                       min(cfg.T, t0 + ch))
    return idx


def make_decode(cfg: Config, device="cpu", seed=0, dtype=torch.bfloat16):
    """Varlen decode batch: one query per sequence at position kv_len - 1."""
    gen = torch.Generator(device=device).manual_seed(seed)
    n = cfg.n_seqs
    kv_lens = torch.randint(cfg.kv_min, cfg.kv_max + 1, (n,), generator=gen, device=device)
    cu_k = torch.zeros(n + 1, dtype=torch.int32, device=device)
    cu_k[1:] = torch.cumsum(kv_lens, 0).to(torch.int32)
    cu_q = torch.arange(n + 1, dtype=torch.int32, device=device)
    total_kv = int(cu_k[-1])
    q = torch.randn(n, cfg.Hq, cfg.Dqk, generator=gen, device=device).to(dtype)
    k = torch.randn(total_kv, cfg.Hk, cfg.Dqk, generator=gen, device=device).to(dtype)
    v = torch.randn(total_kv, cfg.Hk, cfg.Dv, generator=gen, device=device).to(dtype)
    nblk = (kv_lens + cfg.bs - 1) // cfg.bs
    u = torch.rand(n, cfg.Hk, int(nblk.max()), generator=gen, device=device)
    j = torch.arange(u.shape[-1], device=device)
    u = torch.where(j[None, None, :] < nblk[:, None, None], u, torch.full_like(u, float("inf")))
    k_ = min(cfg.S, u.shape[-1])
    val, sel = torch.topk(u, k_, dim=-1, largest=False)
    idx = torch.where(torch.isfinite(val), sel, torch.full_like(sel, -1)).to(torch.int32)
    return dict(q=q, k=k, v=v, idx=idx, cu_q=cu_q, cu_k=cu_k, max_q=1, max_k=int(kv_lens.max()),
                kv_lens=kv_lens)


def page_kv(k: torch.Tensor, v: torch.Tensor, cu_k: torch.Tensor, page_size: int, seed: int = 0):
    """A varlen kv cache ([total_kv, Hk, D] rows, sequence s at rows cu_k[s]..)
    laid out as a paged cache: every sequence's rows cut into pages of
    page_size rows, the pages placed at shuffled positions of one pool.
    Returns (k_pool, v_pool, block_table) with pools [num_pages, page_size,
    Hk, D] (rows past a sequence's end zero) and block_table [n, max_pages]
    int32 (-1 past a sequence's pages).  Vectorised, on k's device."""
    dev = k.device
    cu = cu_k.to(device=dev, dtype=torch.int64)
    lens = cu[1:] - cu[:-1]
    n = lens.numel()
    npg = (lens + page_size - 1) // page_size
    total = int(npg.sum())
    gen = torch.Generator(device=dev).manual_seed(seed)
    perm = torch.randperm(total, generator=gen, device=dev)
    seq = torch.repeat_interleave(torch.arange(n, device=dev), npg)          # sequence of each page
    first = torch.cumsum(npg, 0) - npg
    j = torch.arange(total, device=dev) - first[seq]                          # page index within its sequence
    table = torch.full((n, int(npg.max()) if n else 0), -1, dtype=torch.int32, device=dev)
    table[seq, j] = perm.to(torch.int32)
    r = torch.arange(page_size, device=dev)
    pos = j[:, None] * page_size + r[None, :]                                 # kv position of each pool row
    ok = pos < lens[seq][:, None]
    src = (cu[:-1][seq][:, None] + pos)[ok]
    dst = (perm[:, None] * page_size + r[None, :])[ok]
    pools = []
    for t in (k, v):
        pool = torch.zeros(total * page_size, *t.shape[1:], dtype=t.dtype, device=dev)
        pool[dst] = t[src]
        pools.append(pool.view(total, page_size, *t.shape[1:]))
    return pools[0], pools[1], table


def make_inputs(cfg: Config, device="cpu", seed=0, dtype=torch.bfloat16, with_do=True):
    """Dense configs: dict(q, k, v, idx, do).  Decode: see make_decode."""
    if cfg.mode == "decode":
        d = make_decode(cfg, device, seed, dtype)
        if with_do:
            gen = torch.Generator(device=device).manual_seed(seed + 7)
            d["do"] = torch.randn(d["q"].shape[0], cfg.Hq, cfg.Dv, generator=gen, device=device).to(dtype)
        return d
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(cfg.B, cfg.T, cfg.Hq, cfg.Dqk, generator=gen, device=device).to(dtype)
    k = torch.randn(cfg.B, cfg.T, cfg.Hk, cfg.Dqk, generator=gen, device=device).to(dtype)
    if cfg.mode == "token" and cfg.Dv <= cfg.Dqk:
        # MLA-style: one latent kv tensor; v is its first Dv dims (a view of k)
        v = k[..., :cfg.Dv]
    else:
        v = torch.randn(cfg.B, cfg.T, cfg.Hk, cfg.Dv, generator=gen, device=device).to(dtype)
    d = dict(q=q, k=k, v=v, idx=make_indices(cfg, device, seed))
    if with_do:
        d["do"] = torch.randn(cfg.B, cfg.T, cfg.Hq, cfg.Dv, generator=gen, device=device).to(dtype)
    return d


@dataclass(frozen=True)
class Flops:
    """Algorithmic FLOPs of one fwd+bwd step (recomputation not counted)."""
    fwd: float
    bwd: float

    @property
    def total(self) -> float:
        return self.fwd + self.bwd


def sfa_flops(pairs_qhead: int, d_qk: int, d_v: int) -> Flops:
    """FLOPs over P selected (query-head, key) pairs: fwd = 2P(Dqk+Dv) (QK^T and
    PV, SFA.py:425, 456); bwd = 2P(3Dqk+2Dv) (S, dP, dQ, dK, dV: SFA.py:678-679,
    708, 831, 841)."""
    return Flops(2.0 * pairs_qhead * (d_qk + d_v), 2.0 * pairs_qhead * (3 * d_qk + 2 * d_v))


def blocks_to_tokens(idx: torch.Tensor, bs: int) -> torch.Tensor:
    """Token-level indices that select the same keys as block indices: slot
    s*bs + j holds e*bs + j for the block e in slot s (-1 stays -1).  Keys past
    kv_len or the causal limit are dropped by the op's own validity rule, so
    the selected (query, key) pairs are the same."""
    j = torch.arange(bs, device=idx.device, dtype=idx.dtype)
    e = idx.unsqueeze(-1)
    t = torch.where(e >= 0, e * bs + j, torch.full_like(e * bs + j, -1))
    return t.flatten(-2)


def count_pairs(idx: torch.Tensor, bs: int, q_len: int, kv_len: int, causal: bool = True,
                q_pos: Optional[torch.Tensor] = None, kv_lens: Optional[torch.Tensor] = None) -> int:
    """Valid (query, kv head, key) triples; times Hq/Hk gives (query-head, key) pairs.

    Dense idx [B,T,Hk,S]; decode idx [n,Hk,S] with per-sequence kv_lens (query at
    the last position).  Same validity rules as the kernels."""
    if kv_lens is not None:
        nb = (kv_lens + bs - 1) // bs
        e = idx.to(torch.int64)
        ok = (e >= 0) & (e < nb[:, None, None])
        n_keys = torch.clamp(kv_lens[:, None, None] - e * bs, 0, bs)
        return int(torch.where(ok, n_keys, torch.zeros_like(n_keys)).sum())
    T = idx.shape[1]
    pos = torch.arange(T, device=idx.device) + (kv_len - q_len) if q_pos is None else q_pos
    e = idx.to(torch.int64)
    nblk = (kv_len + bs - 1) // bs
    first = e * bs
    end = torch.clamp(first + bs, max=kv_len)
    if causal:
        end = torch.minimum(end, pos[None, :, None, None] + 1)
    n = torch.clamp(end - first, min=0)
    ok = (e >= 0) & (e < nblk)
    return int(torch.where(ok, n, torch.zeros_like(n)).sum())
