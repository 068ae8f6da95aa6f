"""CPU restatement of the top-k token indexer — TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg use this module; the product path
(ops_b200.lightning_indexer_topk -> libsfa_b200.so) never imports it.

The reference has no indexer (it consumes ``topk_idxs``, SFA.py:90), so there
is no reference output to pin this restatement to: parity unpinned.  It
follows the published lightning-indexer formula of DeepSeek-V3.2's sparse
attention, I[t, s] = sum_h w[t, h] * ReLU(q_idx[t, h] . k_idx[s]), and the
selection rule of ops_b200.indexer: the topk highest scores of the row's keys
(causal: s <= t + Tk - Tq), ties to the lower index, ascending, -1 tail.
"""
from __future__ import annotations

import numpy as np
import torch


def indexer_scores(q_idx: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """[B, Tq, Tk] float64 scores (no mask)."""
    q = q_idx.double()
    k = k_idx.double()
    dots = torch.einsum("bthd,bsd->bths", q, k)
    return torch.einsum("bth,bths->bts", weights.double(), dots.clamp_min(0.0))


def indexer_topk(q_idx, k_idx, weights, topk: int, causal: bool = True, scores=None) -> torch.Tensor:
    """[B, Tq, topk] int32, the selection rule above."""
    B, Tq = q_idx.shape[:2]
    Tk = k_idx.shape[1]
    sc = indexer_scores(q_idx, k_idx, weights) if scores is None else scores.double()
    out = np.full((B, Tq, topk), -1, dtype=np.int32)
    for b in range(B):
        for t in range(Tq):
            n = min(Tk, max(0, t + Tk - Tq + 1)) if causal else Tk
            if n == 0:
                continue
            row = sc[b, t, :n].numpy()
            # descending score, then ascending index (stable sort on -score)
            order = np.argsort(-row, kind="stable")[:topk]
            sel = np.sort(order)
            out[b, t, :sel.size] = sel
    return torch.from_numpy(out)
