"""Top-k token indexer: produces the token-level indices the sparse attention
op consumes (the reference takes ``topk_idxs`` as an input and has no indexer,
SFA.py:90).

Scores follow the lightning-indexer formula of DeepSeek-V3.2's sparse
attention, ``I[t, s] = sum_h w[t, h] * ReLU(q_idx[t, h] . k_idx[s])``, over the
keys of t's sequence (causal: ``s <= t + Tk - Tq``).  Each output row holds the
indices of the ``topk`` highest scores (ties: the lower index first) in
ascending order, then -1 — directly usable as ``block_indices`` of
``sparse_flash_attention(..., block_size=1)`` (view it as ``[B, Tq, 1, topk]``)
or, permuted to ``[Tq, B, topk]``, as the reference's ``topk_idxs``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import SfaIndexerParams


def lightning_indexer_topk(q_idx: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor, topk: int,
                           causal: bool = True) -> torch.Tensor:
    """``q_idx [B, Tq, H, D]`` bf16, ``k_idx [B, Tk, D]`` bf16 (one head shared
    by every query head), ``weights [B, Tq, H]`` fp32 -> ``[B, Tq, topk]`` int32.
    H in {16, 32, 64, 128}, D in {64, 128}, topk <= 4096, Tk <= 49152."""
    for name, t in (("q_idx", q_idx), ("k_idx", k_idx)):
        if not t.is_cuda or t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be a bfloat16 CUDA tensor")
    if q_idx.dim() != 4 or k_idx.dim() != 3 or weights.dim() != 3:
        raise ValueError("expected q_idx [B, Tq, H, D], k_idx [B, Tk, D], weights [B, Tq, H]")
    B, Tq, H, D = q_idx.shape
    if k_idx.shape[0] != B or k_idx.shape[2] != D or tuple(weights.shape) != (B, Tq, H):
        raise ValueError("q_idx, k_idx and weights shapes disagree")
    q = q_idx if (q_idx.stride(-1) == 1 and q_idx.stride(-2) == D) else q_idx.contiguous()
    k = k_idx if k_idx.stride(-1) == 1 else k_idx.contiguous()
    w = weights.float()
    w = w if w.stride(-1) == 1 else w.contiguous()
    out = torch.empty(B, Tq, int(topk), dtype=torch.int32, device=q.device)
    P = SfaIndexerParams(q_idx=q.data_ptr(), k_idx=k.data_ptr(), weights=w.data_ptr(), out=out.data_ptr(),
                         q_sb=q.stride(0), q_st=q.stride(1), q_sh=q.stride(2), k_sb=k.stride(0), k_st=k.stride(1),
                         w_sb=w.stride(0), w_st=w.stride(1), o_sb=out.stride(0), o_st=out.stride(1),
                         batch=B, q_len=Tq, kv_len=k.shape[1], heads=H, dim=D, topk=int(topk),
                         causal=1 if causal else 0)
    lib = _lib.load()
    nbytes = lib.sfa_indexer_workspace_bytes(ctypes.byref(P))     # 0 also when the shape is refused
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    _lib.check(lib.sfa_indexer_topk(ctypes.byref(P), ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream),
               "sfa_indexer_topk")
    return out
