"""CPU oracle for sparse flash attention (SFA) — TEST INFRASTRUCTURE ONLY.

This module restates, in plain fp32 PyTorch on the CPU, the arithmetic of the
reference op ``SparseFlashAttentionTriton`` (lilac-me/ops ``SFA.py``).  It is the
checker for the CUDA kernels in ``ops_b200`` and the timed CPU baseline of
``bench.py``; nothing in the product path imports it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may use it.

Parity pin: the token-level, K-is-V, non-causal special case of every function
here is checked against outputs of the reference's own Triton kernels, executed
under Triton's CPU interpreter in the build container (fixtures and the script
that made them live in ``tests/golden``).  The generalisations (GQA, separate k
and v, block_size > 1, causal masking, varlen, D_v < D_qk, natural-log lse) are
pinned through the mapping onto that special case described in
``tests/golden/make_golden.py``.

Semantics (shared by the oracle and the CUDA kernels):

* A selected entry ``e`` of ``block_indices[..., s]`` is valid iff
  ``0 <= e < ceil(kv_len / block_size)``.  The reference treats only ``e < 0`` as
  invalid (``SFA.py:396``, ``SFA.py:404``) and reads out of bounds for
  ``e >= kv_len``; rejecting those is a superset with identical in-range
  behaviour.  Entries may appear in any slot (the reference needs left-packed
  entries, ``SFA.py:62-66``); duplicates count once per slot, as in the
  reference's sum over slots.
* Block ``e`` covers keys ``e*block_size + j`` for ``j < block_size``; a key is
  valid iff it is ``< kv_len`` and, when ``causal``, ``<= pos(t)`` where
  ``pos(t) = t + kv_len - q_len`` (bottom-right aligned).  The reference has no
  causal mask; causality there lives in the indices (``SFA.py:386-396``).
* Scores ``s = scale * q.k`` (``SFA.py:425``, ``SFA.py:432``).  The optional
  attention sink adds ``exp(sink[h])`` to the softmax denominator and is not
  scaled (``SFA.py:469-474``).
* ``lse`` is natural-log: ``lse = log(sum_k exp(s_k) + exp(sink))``.  The
  reference keeps ``lse2 = lse * log2(e)`` internally (``SFA.py:474``).
* A row with no valid key and no sink has ``o = 0`` and ``lse = -inf`` and zero
  gradients.  (The reference yields ``lse = +inf`` there because of its
  ``-1e11`` running-max seed, ``SFA.py:381`` — a documented divergence.)
* Backward: ``delta = rowsum(o * do)`` (``SFA.py:590-610``);
  ``p = exp(s - lse)``; ``ds = p * (do.v - delta)`` (``SFA.py:688-700``);
  ``dq = scale * ds.k`` (``SFA.py:708-714``); ``dk[key] += scale * ds^T q`` and
  ``dv[key] += p^T do`` (``SFA.py:831-853``, which sums both into one ``grad_kv``
  because its k is v); ``dsink[h] = -sum exp(sink - lse) * delta``
  (``SFA.py:964-970``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

LOG2E = 1.4426950408889634
NEG_INF = float("-inf")


# --------------------------------------------------------------------------
# index expansion
# --------------------------------------------------------------------------
def key_table(block_indices: torch.Tensor, block_size: int, q_pos: torch.Tensor,
              kv_len: int, causal: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """Expand selected block ids to key ids plus a validity mask.

    ``block_indices``: ``[T, S]`` integer block ids of one (sequence, kv head).
    ``q_pos``: ``[T]`` absolute query positions.  Returns ``keys [T, S*bs]``
    (int64, 0 where invalid) and ``valid [T, S*bs]`` (bool).  Follows the
    gather/mask of ``SFA.py:394-412`` generalised to ``block_size`` keys per
    entry and to the causal/out-of-range rules in the module docstring.
    """
    bi = block_indices.to(torch.int64)
    nblk = (kv_len + block_size - 1) // block_size
    blk_ok = (bi >= 0) & (bi < nblk)
    keys = bi[..., None] * block_size + torch.arange(block_size, dtype=torch.int64)
    ok = blk_ok[..., None] & (keys < kv_len)
    if causal:
        ok &= keys <= q_pos.to(torch.int64)[:, None, None]
    keys = torch.where(ok, keys, torch.zeros_like(keys))
    return keys.flatten(-2), ok.flatten(-2)


# --------------------------------------------------------------------------
# one sequence
# --------------------------------------------------------------------------
def _seq_forward(q, k, v, idx, block_size, scale, sink, causal, chunk=256, q_pos=None):
    """q [T,Hq,Dqk] k [Tk,Hk,Dqk] v [Tk,Hk,Dv] idx [T,Hk,S] -> o [T,Hq,Dv], lse [T,Hq].

    Restates the forward of ``_inner_fwd`` (``SFA.py:309-480``) with an exact
    (non-online) softmax in fp32.  ``q_pos`` gives the rows' causal positions
    when q holds a subset of a sequence's rows (default: the whole sequence,
    bottom-right aligned).
    """
    T, Hq, _ = q.shape
    Tk, Hk, Dv = v.shape
    G = Hq // Hk
    o = torch.zeros(T, Hq, Dv, dtype=torch.float32)
    lse = torch.full((T, Hq), NEG_INF, dtype=torch.float32)
    if q_pos is None:
        q_pos = torch.arange(T) + (Tk - T)
    for hk in range(Hk):
        hs = slice(hk * G, (hk + 1) * G)
        keys, ok = key_table(idx[:, hk], block_size, q_pos, Tk, causal)
        kk, vv = k[:, hk].float(), v[:, hk].float()
        sk = None if sink is None else sink[hs].float()
        for t0 in range(0, T, chunk):
            ts = slice(t0, min(T, t0 + chunk))
            kt, okt = keys[ts], ok[ts]
            ks, vs = kk[kt], vv[kt]                                    # [t,N,D]
            s = torch.einsum("tgd,tnd->tgn", q[ts, hs].float(), ks) * scale
            s = s.masked_fill(~okt[:, None, :], NEG_INF)
            if sk is not None:
                s_all = torch.cat([s, sk[None, :, None].expand(s.shape[0], G, 1)], -1)
            else:
                s_all = s
            l = torch.logsumexp(s_all, -1) if s_all.shape[-1] else torch.full(s.shape[:2], NEG_INF)
            lsafe = torch.where(torch.isfinite(l), l, torch.zeros_like(l))
            p = torch.exp(s - lsafe[..., None])
            p = torch.where(okt[:, None, :], p, torch.zeros_like(p))
            o[ts, hs] = torch.einsum("tgn,tnd->tgd", p, vs)
            lse[ts, hs] = l
    return o, lse


def _seq_backward(q, k, v, idx, block_size, scale, sink, causal, o, lse, do, chunk=256, q_pos=None):
    """Gradients of one sequence; follows ``SFA.py:590-1002`` (delta, dq, dsink)
    and ``SFA.py:719-853`` (dk/dv), with k and v kept separate.  With a subset
    of rows (``q_pos`` set), dk/dv hold those rows' contributions only."""
    T, Hq, Dqk = q.shape
    Tk, Hk, Dv = v.shape
    G = Hq // Hk
    dq = torch.zeros(T, Hq, Dqk, dtype=torch.float32)
    dk = torch.zeros(Tk, Hk, Dqk, dtype=torch.float32)
    dv = torch.zeros(Tk, Hk, Dv, dtype=torch.float32)
    dsink = torch.zeros(Hq, dtype=torch.float32)
    if q_pos is None:
        q_pos = torch.arange(T) + (Tk - T)
    delta = (o.float() * do.float()).sum(-1)                          # [T,Hq]
    lsafe_all = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    for hk in range(Hk):
        hs = slice(hk * G, (hk + 1) * G)
        keys, ok = key_table(idx[:, hk], block_size, q_pos, Tk, causal)
        kk, vv = k[:, hk].float(), v[:, hk].float()
        for t0 in range(0, T, chunk):
            ts = slice(t0, min(T, t0 + chunk))
            kt, okt = keys[ts], ok[ts]
            ks, vs = kk[kt], vv[kt]
            qt, dot = q[ts, hs].float(), do[ts, hs].float()
            s = torch.einsum("tgd,tnd->tgn", qt, ks) * scale
            p = torch.exp(s - lsafe_all[ts, hs][..., None])
            p = torch.where(okt[:, None, :] & torch.isfinite(lse[ts, hs])[..., None], p, torch.zeros_like(p))
            dp = torch.einsum("tgd,tnd->tgn", dot, vs)
            ds = p * (dp - delta[ts, hs][..., None])
            dq[ts, hs] = scale * torch.einsum("tgn,tnd->tgd", ds, ks)
            dks = scale * torch.einsum("tgn,tgd->tnd", ds, qt)           # [t,N,Dqk]
            dvs = torch.einsum("tgn,tgd->tnd", p, dot)                   # [t,N,Dv]
            m = okt.reshape(-1)
            flat = kt.reshape(-1)[m]
            dk[:, hk].index_add_(0, flat, dks.reshape(-1, Dqk)[m])
            dv[:, hk].index_add_(0, flat, dvs.reshape(-1, Dv)[m])
    if sink is not None:
        fin = torch.isfinite(lse)
        ps = torch.where(fin, torch.exp(sink.float()[None, :] - lsafe_all), torch.zeros_like(lse))
        dsink = -(ps * delta).sum(0)
    return dq, dk, dv, dsink


# --------------------------------------------------------------------------
# public oracle API (mirrors ops_b200.sparse_flash_attention's argument meaning)
# --------------------------------------------------------------------------
def _sequences(q, k, cu_seqlens_q, cu_seqlens_k):
    if cu_seqlens_q is None:
        return [(b, slice(None), slice(None)) for b in range(q.shape[0])]
    cq = [int(x) for x in cu_seqlens_q]
    ck = [int(x) for x in cu_seqlens_k]
    return [(None, slice(cq[i], cq[i + 1]), slice(ck[i], ck[i + 1])) for i in range(len(cq) - 1)]


def sfa_forward(q, k, v, block_indices, block_size=64, scale=None, attn_sink=None,
                causal=True, cu_seqlens_q=None, cu_seqlens_k=None):
    """fp32 forward.  Dense layout: q [B,T,Hq,Dqk], k [B,Tk,Hk,Dqk], v [B,Tk,Hk,Dv],
    block_indices [B,T,Hk,S].  Varlen: drop the batch axis and pass cu_seqlens.
    Returns (o fp32, lse fp32 natural log)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if cu_seqlens_q is None:
        outs = [_seq_forward(q[b], k[b], v[b], block_indices[b], block_size, scale, attn_sink, causal)
                for b in range(q.shape[0])]
        return torch.stack([x[0] for x in outs]), torch.stack([x[1] for x in outs])
    o = torch.zeros(*q.shape[:-1], v.shape[-1], dtype=torch.float32)
    lse = torch.full(q.shape[:-1], NEG_INF, dtype=torch.float32)
    for _, sq, sk in _sequences(q, k, cu_seqlens_q, cu_seqlens_k):
        o[sq], lse[sq] = _seq_forward(q[sq], k[sk], v[sk], block_indices[sq], block_size, scale,
                                      attn_sink, causal)
    return o, lse


def sfa_backward(q, k, v, block_indices, o, lse, do, block_size=64, scale=None, attn_sink=None,
                 causal=True, cu_seqlens_q=None, cu_seqlens_k=None):
    """fp32 backward given the forward's o and lse.  Returns (dq, dk, dv, dsink)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    dq = torch.zeros(q.shape, dtype=torch.float32)
    dk = torch.zeros(k.shape, dtype=torch.float32)
    dv = torch.zeros(v.shape, dtype=torch.float32)
    dsink = torch.zeros(q.shape[-2], dtype=torch.float32)
    if cu_seqlens_q is None:
        for b in range(q.shape[0]):
            r = _seq_backward(q[b], k[b], v[b], block_indices[b], block_size, scale, attn_sink, causal,
                              o[b], lse[b], do[b])
            dq[b], dk[b], dv[b] = r[0], r[1], r[2]
            dsink += r[3]
    else:
        for _, sq, sk in _sequences(q, k, cu_seqlens_q, cu_seqlens_k):
            r = _seq_backward(q[sq], k[sk], v[sk], block_indices[sq], block_size, scale, attn_sink,
                              causal, o[sq], lse[sq], do[sq])
            dq[sq], dk[sk], dv[sk] = r[0], r[1], r[2]
            dsink += r[3]
    return dq, dk, dv, (dsink if attn_sink is not None else None)


def sfa_rows_forward(q_rows, k, v, idx_rows, q_pos, block_size=64, scale=None, attn_sink=None, causal=True):
    """fp32 forward of selected query rows of one sequence: q_rows [n,Hq,Dqk],
    k [Tk,Hk,Dqk], v [Tk,Hk,Dv], idx_rows [n,Hk,S], q_pos [n] causal positions.
    Each row depends only on its own indices, so the result equals those rows
    of the full-sequence forward.  Returns (o, lse)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q_rows.shape[-1])
    return _seq_forward(q_rows, k, v, idx_rows, block_size, scale, attn_sink, causal,
                        q_pos=torch.as_tensor(q_pos, dtype=torch.int64))


def sfa_rows_backward(q_rows, k, v, idx_rows, q_pos, o_rows, lse_rows, do_rows, block_size=64, scale=None,
                      attn_sink=None, causal=True):
    """Gradients from selected query rows of one sequence: dq of those rows
    (exact), and the rows' contributions to dk/dv (exact for every key whose
    selecting rows are all among them).  Returns (dq, dk, dv, dsink_part)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q_rows.shape[-1])
    return _seq_backward(q_rows, k, v, idx_rows, block_size, scale, attn_sink, causal, o_rows, lse_rows,
                         do_rows, q_pos=torch.as_tensor(q_pos, dtype=torch.int64))


def reference_compat_forward(q, kv, attn_sink, topk_idxs, sm_scale):
    """Oracle for the reference signature ``SparseFlashAttentionTriton.apply``
    (``SFA.py:75-82``): SBHD q [S,B,H,D], shared kv [S_kv,B,D], topk [S,B,TopK],
    token-level, no causal mask.  Returns (out fp32 [S,B,H,D], lse natural log [S,B,H])."""
    qb = q.permute(1, 0, 2, 3)
    kvb = kv.permute(1, 0, 2)[:, :, None, :]
    ib = topk_idxs.permute(1, 0, 2)[:, :, None, :]
    o, lse = sfa_forward(qb, kvb, kvb, ib, 1, sm_scale, attn_sink, False)
    return o.permute(1, 0, 2, 3), lse.permute(1, 0, 2)


def reference_compat_backward(q, kv, attn_sink, topk_idxs, sm_scale, o, lse, do):
    """Gradients for the reference signature: returns (dq, dkv = dk + dv, dsink),
    matching ``SFA.py:300-306`` where k is v."""
    qb = q.permute(1, 0, 2, 3)
    kvb = kv.permute(1, 0, 2)[:, :, None, :]
    ib = topk_idxs.permute(1, 0, 2)[:, :, None, :]
    dq, dk, dv, ds = sfa_backward(qb, kvb, kvb, ib, o.permute(1, 0, 2, 3), lse.permute(1, 0, 2),
                                  do.permute(1, 0, 2, 3), 1, sm_scale, attn_sink, False)
    dkv = (dk + dv)[:, :, 0, :].permute(1, 0, 2)
    return dq.permute(1, 0, 2, 3), dkv, ds


# --------------------------------------------------------------------------
# accounting shared by tests and the bench
# --------------------------------------------------------------------------
def selected_pairs(block_indices, block_size, q_len, kv_len, causal=True):
    """P = number of valid (query, kv-head, key) triples for a dense [B,T,Hk,S] index
    tensor; multiply by G for (query-head, key) pairs."""
    B, T, Hk, S = block_indices.shape
    q_pos = torch.arange(T) + (kv_len - q_len)
    total = 0
    for b in range(B):
        for hk in range(Hk):
            _, ok = key_table(block_indices[b, :, hk], block_size, q_pos, kv_len, causal)
            total += int(ok.sum())
    return total


@dataclass
class Flops:
    fwd: float
    bwd: float

    @property
    def total(self):
        return self.fwd + self.bwd


def sfa_flops(pairs_qhead, d_qk, d_v):
    """Algorithmic FLOPs over selected (query-head, key) pairs:
    fwd = 2P(Dqk+Dv); bwd = 2P(3Dqk+2Dv) (S, dP, dQ, dK, dV; no recompute)."""
    return Flops(2.0 * pairs_qhead * (d_qk + d_v), 2.0 * pairs_qhead * (3 * d_qk + 2 * d_v))
