"""GPU: the top-k token indexer against its CPU restatement.

With small-integer q / k and power-of-two weights every score is exact in
fp32, so the tensor-core scores equal the oracle's and the selected indices
must match exactly — ties included (frequent with integer scores), which pins
the tie rule.  With random inputs the selection is checked against fp64
scores: what it keeps scores no lower than what it drops (to fp32 rounding).
"""
import pytest
import torch

import ops_b200
from oracle import indexer_oracle as IO
from oracle import sfa_oracle as O
from sfa_check import assert_close

pytestmark = pytest.mark.gpu


def _int_inputs(B, Tq, Tk, H, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-2, 3, (B, Tq, H, D), generator=g).bfloat16()
    k = torch.randint(-2, 3, (B, Tk, D), generator=g).bfloat16()
    w = torch.tensor([0.5, 1.0, 2.0, -1.0])[torch.randint(0, 4, (B, Tq, H), generator=g)]
    return q, k, w


@pytest.mark.parametrize("B,Tq,Tk,H,D,topk,causal", [
    (2, 300, 300, 64, 128, 64, True),       # DeepSeek-V3.2's indexer shape (64 heads x 128 dims)
    (1, 257, 257, 16, 64, 100, True),       # 16 queries a group, a partial last group
    (1, 130, 130, 128, 128, 32, False),     # 2 queries a group, non-causal
    (2, 5, 700, 32, 128, 128, True),        # decode-like: few queries at the end of a long cache
])
def test_indexer_exact_on_integer_scores(B, Tq, Tk, H, D, topk, causal):
    q, k, w = _int_inputs(B, Tq, Tk, H, D, seed=Tq + H)
    dev = torch.device("cuda")
    got = ops_b200.lightning_indexer_topk(q.to(dev), k.to(dev), w.to(dev), topk, causal=causal)
    torch.cuda.synchronize()
    ref = IO.indexer_topk(q.float(), k.float(), w, topk, causal=causal)
    assert torch.equal(got.cpu(), ref)


def test_indexer_random_scores_keep_the_largest():
    B, Tq, Tk, H, D, topk = 1, 64, 6000, 64, 128, 2048
    g = torch.Generator().manual_seed(3)
    q = torch.randn(B, Tq, H, D, generator=g).bfloat16()
    k = torch.randn(B, Tk, D, generator=g).bfloat16()
    w = torch.rand(B, Tq, H, generator=g) / H
    dev = torch.device("cuda")
    got = ops_b200.lightning_indexer_topk(q.to(dev), k.to(dev), w.to(dev), topk, causal=True).cpu()
    sc = IO.indexer_scores(q.float(), k.float(), w)
    for t in range(Tq):
        n = min(Tk, t + Tk - Tq + 1)
        sel = got[0, t]
        kept = sel[sel >= 0]
        assert kept.numel() == min(topk, n)
        assert torch.equal(kept, kept.sort().values)                      # ascending
        assert kept.unique().numel() == kept.numel() and int(kept.max()) < n
        mask = torch.zeros(n, dtype=torch.bool)
        mask[kept.long()] = True
        row = sc[0, t, :n]
        if (~mask).any():
            tol = 1e-4 * float(row.abs().max())
            assert float(row[mask].min()) >= float(row[~mask].max()) - tol


def test_indexer_feeds_the_op():
    # the indexer's rows are the op's token-level block_indices as they are
    B, T, H, D = 1, 200, 64, 128
    q_idx, k_idx, w = _int_inputs(B, T, T, H, D, seed=5)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(B, T, 16, 128, generator=g).bfloat16()
    kv = torch.randn(B, T, 1, 128, generator=g).bfloat16()
    dev = torch.device("cuda")
    idx = ops_b200.lightning_indexer_topk(q_idx.to(dev), k_idx.to(dev), w.to(dev), 48)
    o, lse = ops_b200.sparse_flash_attention(q.to(dev), kv.to(dev), kv.to(dev), idx.unsqueeze(2), 1)
    torch.cuda.synchronize()
    ref_idx = IO.indexer_topk(q_idx.float(), k_idx.float(), w, 48)
    ro, _ = O.sfa_forward(q.float(), kv.float(), kv.float(), ref_idx.unsqueeze(2), 1)
    assert_close("o", o.cpu(), ro)
