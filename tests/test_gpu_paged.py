"""GPU: the forward over a paged kv cache (block table + page pool) gives the
same o and lse as the contiguous varlen forward over the same keys (bitwise:
the same kernel reads the same rows from other addresses), and matches the
oracle.  Block-level (the tensor-core decode path of config 5, pages of one
and of two blocks), token-level (pages of 16 rows), the CUDA-core family, and
several queries per sequence."""
import pytest
import torch

import ops_b200
from oracle import sfa_oracle as O
from sfa_check import assert_close, assert_lse

pytestmark = pytest.mark.gpu


def _problem(seed, n, Hq, Hk, D, bs, S, q_per_seq=1, kv_lo=100, kv_hi=900):
    g = torch.Generator().manual_seed(seed)
    kv_lens = torch.randint(kv_lo, kv_hi, (n,), generator=g)
    q_lens = torch.full((n,), q_per_seq, dtype=torch.int64)
    cu_q = torch.cat([torch.zeros(1, dtype=torch.int64), q_lens.cumsum(0)]).to(torch.int32)
    cu_k = torch.cat([torch.zeros(1, dtype=torch.int64), kv_lens.cumsum(0)]).to(torch.int32)
    tq, tk = int(cu_q[-1]), int(cu_k[-1])
    q = torch.randn(tq, Hq, D, generator=g).bfloat16()
    k = torch.randn(tk, Hk, D, generator=g).bfloat16()
    v = torch.randn(tk, Hk, D, generator=g).bfloat16()
    rows = []
    for s in range(n):
        units = (int(kv_lens[s]) + bs - 1) // bs
        for _ in range(q_per_seq):
            rows.append(torch.stack([torch.randperm(units, generator=g)[:S] for _ in range(Hk)]))
    idx = torch.full((tq, Hk, S), -1, dtype=torch.int32)
    for i, r in enumerate(rows):
        idx[i, :, :r.shape[1]] = r.to(torch.int32)
    return q, k, v, idx, cu_q, cu_k, kv_lens


def _paged(k, v, cu_k, kv_lens, page_size, seed):
    """Scatter each sequence's rows into pages of a shuffled pool; returns the
    pools [num_pages, page_size, Hk, D] and the block table."""
    g = torch.Generator().manual_seed(seed)
    n = kv_lens.numel()
    pages = [(int(l) + page_size - 1) // page_size for l in kv_lens]
    total = sum(pages) + 3                                  # a few pages nobody uses
    perm = torch.randperm(total, generator=g)
    table = torch.full((n, max(pages) + 2), -1, dtype=torch.int32)
    kp = torch.zeros(total, page_size, *k.shape[1:], dtype=k.dtype)
    vp = torch.zeros(total, page_size, *v.shape[1:], dtype=v.dtype)
    j = 0
    for s in range(n):
        k0, l = int(cu_k[s]), int(kv_lens[s])
        for p in range(pages[s]):
            pg = int(perm[j])
            j += 1
            table[s, p] = pg
            r0, r1 = p * page_size, min(l, (p + 1) * page_size)
            kp[pg, :r1 - r0] = k[k0 + r0:k0 + r1]
            vp[pg, :r1 - r0] = v[k0 + r0:k0 + r1]
    return kp, vp, table


@pytest.mark.parametrize("bs,page_size,S,q_per_seq,kernel", [
    (64, 64, 8, 1, "auto"),        # config 5's decode path: one block a page
    (64, 128, 8, 1, "auto"),       # two blocks a page
    (64, 64, 8, 3, "auto"),        # several queries per sequence (causal within the sequence)
    (1, 16, 96, 1, "auto"),        # token-level: the row gather through the table
    (64, 64, 8, 1, "general"),     # CUDA-core family
])
def test_paged_matches_contiguous_and_oracle(bs, page_size, S, q_per_seq, kernel):
    Hq, Hk, D = 16, 2, 128
    q, k, v, idx, cu_q, cu_k, kv_lens = _problem(bs + page_size + q_per_seq, 6, Hq, Hk, D, bs, S, q_per_seq)
    sink = torch.randn(Hq, generator=torch.Generator().manual_seed(3))
    dev = torch.device("cuda")
    mq, mk = q_per_seq, int(kv_lens.max())
    o1, l1 = ops_b200.sparse_flash_attention(q.to(dev), k.to(dev), v.to(dev), idx.to(dev), bs,
                                             cu_seqlens=cu_q.to(dev), cu_seqlens_k=cu_k.to(dev),
                                             attn_sink=sink.to(dev), max_seqlen_q=mq, max_seqlen_k=mk,
                                             kernel=kernel)
    kp, vp, table = _paged(k, v, cu_k, kv_lens, page_size, seed=bs + 7)
    o2, l2 = ops_b200.sparse_flash_attention_paged(q.to(dev), kp.to(dev), vp.to(dev), idx.to(dev), table.to(dev),
                                                   kv_lens.to(dev), bs, cu_seqlens=cu_q.to(dev),
                                                   attn_sink=sink.to(dev), max_seqlen_q=mq, max_seqlen_k=mk,
                                                   kernel=kernel)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.equal(l1, l2)
    ro, rl = O.sfa_forward(q.float(), k.float(), v.float(), idx, bs, None, sink, True, cu_q, cu_k)
    assert_close("o", o2.cpu(), ro)
    assert_lse(l2.cpu(), rl)


def test_paged_decode_defaults_and_shared_latent_cache():
    # one query per sequence (cu_seqlens omitted) and v the leading dims of one
    # latent cache, token-level with MLA head dims
    Hq, Hk, Dqk, Dv, S = 64, 1, 576, 512, 128
    g = torch.Generator().manual_seed(11)
    n, page_size = 5, 64
    kv_lens = torch.randint(150, 700, (n,), generator=g)
    cu_k = torch.cat([torch.zeros(1, dtype=torch.int64), kv_lens.cumsum(0)]).to(torch.int32)
    k = torch.randn(int(cu_k[-1]), Hk, Dqk, generator=g).bfloat16()
    q = torch.randn(n, Hq, Dqk, generator=g).bfloat16()
    idx = torch.stack([torch.stack([torch.randperm(int(l), generator=g)[:S]]) for l in kv_lens]).to(torch.int32)
    kp, _, table = _paged(k, k, cu_k, kv_lens, page_size, seed=5)
    dev = torch.device("cuda")
    kpd = kp.to(dev)
    o, lse = ops_b200.sparse_flash_attention_paged(q.to(dev), kpd, kpd[..., :Dv], idx.to(dev), table.to(dev),
                                                   kv_lens.to(dev), 1)
    torch.cuda.synchronize()
    cu_q = torch.arange(n + 1, dtype=torch.int32)
    ro, rl = O.sfa_forward(q.float(), k.float(), k[..., :Dv].float(), idx, 1, None, None, True, cu_q, cu_k)
    assert_close("o", o.cpu(), ro)
    assert_lse(lse.cpu(), rl)
