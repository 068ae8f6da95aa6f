"""Query-range sharding of one long sequence across ranks (strong scaling).

Independent (sequence, kv head) units need no coordination at all: a rank
takes whole units or whole batches.  A configuration with fewer units than
ranks (one 65536-token sequence with 4 kv heads, or a single-unit MLA shape)
splits its query rows instead.  Rank r takes rows ``[r0, r1)`` of every
sequence in the batch and attends to keys ``[0, r1 + (Tk - T))``: with the
bottom-right causal alignment the op uses (``pos(t) = t + kv_len - q_len``),
``q_len = r1 - r0`` and ``kv_len = r1 + Tk - T`` give every row the position it
has in the full problem, and no key past that range is visible to those rows.
The forward outputs and dq of those rows stay on the rank.  dK / dV receive
contributions from every rank's rows: each rank's fp32 partial (zero past its
key range) is summed with one reduce-scatter over the key axis, after which
rank r holds dk / dv of its own equal key share — the one exchange step of the
path, so the one collective.

The row ranges balance the exact work: valid (query, kv head, key) triples per
query row, counted from the indices with the op's own validity rules.
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple

import torch


def row_work(block_indices: torch.Tensor, block_size: int, kv_len: int, causal: bool = True) -> torch.Tensor:
    """Valid (kv head, key) pairs of each query row, summed over the batch.

    ``block_indices [B, T, Hk, S]``; an entry ``e`` is valid iff
    ``0 <= e < ceil(kv_len / block_size)``; block ``e`` holds keys
    ``e*block_size + j < kv_len`` and, when causal, ``<= pos(t)``."""
    B, T, Hk, S = block_indices.shape
    e = block_indices.to(torch.int64)
    nblk = (kv_len + block_size - 1) // block_size
    pos = torch.arange(T, device=e.device) + (kv_len - T)
    first = e * block_size
    end = torch.clamp(first + block_size, max=kv_len)
    if causal:
        end = torch.minimum(end, pos[None, :, None, None] + 1)
    n = torch.clamp(end - first, min=0)
    n = torch.where((e >= 0) & (e < nblk), n, torch.zeros_like(n))
    return n.sum(dim=(0, 2, 3))


def row_cost(block_indices: torch.Tensor, block_size: int, kv_len: int, causal: bool = True,
             range_rows: int = 2048, batch_rows: int = 8, per_pair: float = 3.59e-8,
             per_batch: float = 1.62e-5, per_job: float = 3.67e-5) -> torch.Tensor:
    """A per-row cost (ms) that also counts the key-centric dK/dV pass's units.

    Pairs alone balance the forward, but the dK/dV pass works in jobs (one per
    row range of ``range_rows``, kv head and block with at least one query) of
    batches of ``batch_rows`` queries, and a job costs its change-over on top
    of its batches.  Rows whose selections spread over more blocks make more,
    thinner jobs.  Each valid (row, kv head, block) entry carries 1/n of its
    job and ceil(n / batch_rows)/n of its batches (n = the job's queries).  The
    default weights are B200 times at D = 128 (ms per pair of the forward, per
    batch and per job of the pass), fitted with :func:`fit_cost` to the two
    ranks of a measured two-GPU split of one 65536-token sequence (4 kv heads,
    32 selected 64-key blocks a row).  Returns float64 per row.

    It is an approximation of what the ranks run: jobs are counted in row
    ranges from global row 0, while each rank's kernel counts its ranges from
    its own first row (``range_units`` models that), and long sequences get
    longer ranges in the kernel (at most 64 ranges a unit).  ``range_units`` on
    the chosen ranges gives the exact per-rank counts to check a split."""
    B, T, Hk, S = block_indices.shape
    e = block_indices.to(torch.int64)
    nblk = (kv_len + block_size - 1) // block_size
    pos = torch.arange(T, device=e.device) + (kv_len - T)
    first = e * block_size
    end = torch.clamp(first + block_size, max=kv_len)
    if causal:
        end = torch.minimum(end, pos[None, :, None, None] + 1)
    n = torch.clamp(end - first, min=0)
    valid = (e >= 0) & (e < nblk) & (n > 0)
    pairs = torch.where(valid, n, torch.zeros_like(n)).sum(dim=(0, 2, 3)).to(torch.float64)
    # job id of every entry: (batch, kv head, row range, block)
    rr = (torch.arange(T, device=e.device) // range_rows)[None, :, None, None]
    nr = (T + range_rows - 1) // range_rows
    bb = torch.arange(B, device=e.device)[:, None, None, None]
    hh = torch.arange(Hk, device=e.device)[None, None, :, None]
    jid = ((bb * Hk + hh) * nr + rr) * max(nblk, 1) + torch.clamp(e, 0, max(nblk - 1, 0))
    counts = torch.bincount(jid[valid], minlength=B * Hk * nr * max(nblk, 1)).to(torch.float64)
    per_entry = torch.where(counts > 0, (per_job + per_batch * torch.ceil(counts / batch_rows)) / counts.clamp(min=1),
                            torch.zeros_like(counts))
    ent = torch.where(valid, per_entry[jid.clamp(min=0)], torch.zeros(jid.shape, dtype=torch.float64, device=e.device))
    return per_pair * pairs + ent.sum(dim=(0, 2, 3))


def range_units(block_indices: torch.Tensor, block_size: int, ranges: List[Tuple[int, int]], kv_len_of=None,
                causal: bool = True, range_rows: int = 2048, batch_rows: int = 8) -> List[Tuple[int, int, int]]:
    """(pairs, batches, jobs) of each rank's rows as the rank runs them: rows
    [r0, r1) against keys [0, r1) (``kv_len_of(r0, r1)`` overrides), the
    dK/dV pass's row ranges counted from r0."""
    out = []
    for r0, r1 in ranges:
        if r1 <= r0:
            out.append((0, 0, 0))
            continue
        kv = kv_len_of(r0, r1) if kv_len_of else r1
        e = block_indices[:, r0:r1].to(torch.int64)
        B, Tq, Hk, S = e.shape
        nblk = (kv + block_size - 1) // block_size
        pos = torch.arange(Tq, device=e.device) + (kv - Tq)
        first = e * block_size
        end = torch.clamp(first + block_size, max=kv)
        if causal:
            end = torch.minimum(end, pos[None, :, None, None] + 1)
        n = torch.clamp(end - first, min=0)
        valid = (e >= 0) & (e < nblk) & (n > 0)
        nr = (Tq + range_rows - 1) // range_rows
        rr = (torch.arange(Tq, device=e.device) // range_rows)[None, :, None, None]
        jid = ((torch.arange(B, device=e.device)[:, None, None, None] * Hk +
                torch.arange(Hk, device=e.device)[None, None, :, None]) * nr + rr) * nblk + torch.clamp(e, 0, nblk - 1)
        cnt = torch.bincount(jid[valid], minlength=B * Hk * nr * nblk)
        out.append((int(n[valid].sum()), int(((cnt + batch_rows - 1) // batch_rows).sum()), int((cnt > 0).sum())))
    return out


def fit_cost(units: List[Tuple[int, int, int]], fwd_ms: List[float], dkdv_ms: List[float]) -> dict:
    """Weights for :func:`row_cost` from a measured split: per-rank (pairs,
    batches, jobs) from :func:`range_units` and the ranks' forward and dK/dV
    kernel times (the bench line's per-rank kernel times).  The forward is
    taken as proportional to pairs; the dK/dV pass as a per-batch plus a
    per-job time, solved by least squares.

    Two ranks give two equations for two unknowns: the fit is exact
    (``residual`` 0) and says nothing about how well the model predicts; more
    ranks (or several splits' ranks together) over-determine it.  Returns the
    weights plus ``residual`` (RMS, ms) and ``rank`` of the system; raises
    ``ValueError`` when the system is singular or a weight comes out negative
    (the model does not describe the measurements)."""
    pairs = torch.tensor([u[0] for u in units], dtype=torch.float64)
    A = torch.tensor([[u[1], u[2]] for u in units], dtype=torch.float64)
    y = torch.tensor(dkdv_ms, dtype=torch.float64)
    per_pair = float(sum(fwd_ms)) / float(pairs.sum())
    rank = int(torch.linalg.matrix_rank(A))
    if rank < 2:
        raise ValueError("fit_cost: the ranks' (batches, jobs) counts are linearly dependent")
    sol = torch.linalg.lstsq(A, y[:, None]).solution.flatten()
    if float(sol.min()) < 0.0 or per_pair < 0.0:
        raise ValueError(f"fit_cost: negative weight (per_batch {float(sol[0]):.3g}, per_job {float(sol[1]):.3g})")
    resid = float(((A @ sol - y) ** 2).mean().sqrt())
    return {"per_pair": per_pair, "per_batch": float(sol[0]), "per_job": float(sol[1]), "residual": resid,
            "rank": rank, "exact": len(units) == 2}


def query_ranges(work: torch.Tensor, world: int) -> List[Tuple[int, int]]:
    """Contiguous row ranges of (nearly) equal total work, one per rank.

    Cut r (r = 1 .. world-1) is the first row whose work prefix reaches
    r / world of the total; rows of zero work go with their neighbours."""
    T = int(work.numel())
    csum = torch.cumsum(work.to(torch.float64).cpu(), 0)
    total = float(csum[-1]) if T else 0.0
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        c = int(torch.searchsorted(csum, torch.tensor([target], dtype=torch.float64)).item()) + 1 if total else 0
        cuts.append(min(max(c, cuts[-1]), T))
    cuts.append(T)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def key_share(kv_len: int, world: int, rank: int) -> Tuple[int, int]:
    """Keys [k0, k1) whose dk / dv rank ``rank`` holds after the reduce-scatter."""
    tc = (kv_len + world - 1) // world
    return min(rank * tc, kv_len), min((rank + 1) * tc, kv_len)


def op_fwd_bwd(q, k, v, idx, do, block_size, scale, causal):
    """The single-device step on the CUDA op: (o, lse, dq, dk, dv)."""
    from .sfa import sparse_flash_attention
    qg = q.detach().requires_grad_(True)
    kg = k.detach().requires_grad_(True)
    vg = v.detach().requires_grad_(True)
    o, lse = sparse_flash_attention(qg, kg, vg, idx, block_size, scale, causal=causal)
    o.backward(do)
    return o.detach(), lse, qg.grad, kg.grad, vg.grad


def shard_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor, do: torch.Tensor,
               rank: int, world: int, ranges: List[Tuple[int, int]], block_size: int = 64,
               scale: Optional[float] = None, causal: bool = True, group=None,
               fwd_bwd: Callable = op_fwd_bwd) -> dict:
    """Forward + backward of this rank's query rows of a dense batch.

    ``q [B,T,Hq,Dqk]``, ``k [B,Tk,Hk,Dqk]``, ``v [B,Tk,Hk,Dv]`` (every rank holds
    the inputs), ``ranges`` from :func:`query_ranges`.  Slices this rank's rows
    and visible keys and runs :func:`local_step` on them."""
    T, Tk = q.shape[1], k.shape[1]
    r0, r1 = ranges[rank]
    ke = r1 + (Tk - T) if r1 > r0 else 0            # keys visible to rows < r1
    return local_step(q[:, r0:r1], k[:, :ke], v[:, :ke], block_indices[:, r0:r1], do[:, r0:r1], (r0, r1), Tk,
                      rank, world, block_size, scale, causal, group, fwd_bwd)


def local_step(q_rows: torch.Tensor, k_pre: torch.Tensor, v_pre: torch.Tensor, idx_rows: torch.Tensor,
               do_rows: torch.Tensor, rows: Tuple[int, int], kv_len: int, rank: int, world: int,
               block_size: int = 64, scale: Optional[float] = None, causal: bool = True, group=None,
               fwd_bwd: Callable = op_fwd_bwd) -> dict:
    """The same step from this rank's own slices: rows ``[r0, r1)`` of q /
    indices / dO and the first ``r1 + kv_len - T`` keys of k / v.  Returns the
    rows with their ``o``, ``lse`` and ``dq``, and this rank's key share
    ``(k0, k1)`` of ``[0, kv_len)`` with the summed ``dk``, ``dv`` (fp32 sums, in
    k's dtype).  ``fwd_bwd(q, k, v, idx, do, block_size, scale, causal)`` is the
    single-device step (the CUDA op by default).  When v is a leading-dims view
    of k (one latent kv tensor), the op returns one gradient ``dk + dv`` in k's
    shape: it is summed here as ``dk`` and ``dv`` is None."""
    import torch.distributed as dist
    B, _, _, Dqk = q_rows.shape
    Hk, Dv = k_pre.shape[2], v_pre.shape[3]
    dev = q_rows.device
    # decided from the inputs, so every rank (with rows or without) agrees
    shared = (v_pre.data_ptr() == k_pre.data_ptr() and v_pre.stride() == k_pre.stride()
              and v_pre.shape[:-1] == k_pre.shape[:-1])
    width = Dqk if shared else Dqk + Dv
    if scale is None:
        scale = 1.0 / math.sqrt(Dqk)
    r0, r1 = rows
    ke = k_pre.shape[1]
    o = lse = dq = None
    if r1 > r0:
        o, lse, dq, dk, dv = fwd_bwd(q_rows, k_pre, v_pre, idx_rows, do_rows, block_size, scale, causal)
    else:                                            # no rows here: nothing to add
        ke = 0
    # fp32 partials on the key axis (keys major), padded to world equal shares;
    # dk and dv travel in one buffer
    tc = (kv_len + world - 1) // world
    buf = torch.zeros(world * tc, B, Hk, width, dtype=torch.float32, device=dev)
    if ke > 0:
        buf[:ke, ..., :Dqk] = dk.float().transpose(0, 1)
        if not shared:
            buf[:ke, ..., Dqk:] = dv.float().transpose(0, 1)
    mine = torch.empty(tc, B, Hk, width, dtype=torch.float32, device=dev)
    if world > 1:
        dist.reduce_scatter_tensor(mine, buf, group=group)
    else:
        mine.copy_(buf)
    k0, k1 = key_share(kv_len, world, rank)
    n = k1 - k0
    dk_own = mine[:n, ..., :Dqk].transpose(0, 1).to(k_pre.dtype).contiguous()
    dv_own = None if shared else mine[:n, ..., Dqk:].transpose(0, 1).to(v_pre.dtype).contiguous()
    return dict(rows=(r0, r1), o=o, lse=lse, dq=dq, keys=(k0, k1), dk=dk_own, dv=dv_own)
