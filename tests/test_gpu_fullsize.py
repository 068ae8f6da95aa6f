"""GPU parity at the benchmark's own sizes.

The op runs on the full configuration (c2: B=4, T=8192, Hq=64, Hk=4; c3:
T=65536 with 32 selected blocks a row, 32 row ranges in the key-centric pass;
c4's geometry with Hq=128 sharing one latent kv head, D_qk 576 / D_v 512; c5:
128 sequences with kv lengths up to 131072).  The CPU oracle then checks:

* o, lse and dq of sampled query rows (every head): a row depends only on its
  own indices, so the oracle evaluates just those rows
  (``sfa_rows_forward`` / ``sfa_rows_backward`` with the rows' positions);
* dk and dv of sampled key blocks: the oracle runs every query row that
  selected the block (its complete query list, read from the indices), which
  makes those keys' gradients exact.

Tolerances are the op's: max-abs 2e-2 (row-normalised, ``sfa_check``),
rel-L2 5e-3, lse 1e-3.
"""
import pytest
import torch

import ops_b200
from ops_b200 import workloads as W
from oracle import sfa_oracle as O
from sfa_check import assert_close, assert_lse

pytestmark = pytest.mark.gpu


def _run_op(d, cfg, dev, backward=True):
    """The op on device copies of d; returns dict of device tensors."""
    q = d["q"].to(dev).requires_grad_(backward)
    k = d["k"].to(dev).requires_grad_(backward)
    shared = d["v"].data_ptr() == d["k"].data_ptr()
    v = k[..., :cfg.Dv] if shared else d["v"].to(dev).requires_grad_(backward)
    o, lse = ops_b200.sparse_flash_attention(q, k, v, d["idx"].to(dev), cfg.bs, cfg.scale, causal=cfg.causal)
    out = dict(o=o.detach(), lse=lse.detach())
    if backward:
        o.backward(d["do"].to(dev))
        out.update(dq=q.grad, dk=k.grad, dv=None if shared else v.grad)
    torch.cuda.synchronize()
    return out


def _sample_rows(T, n, seed):
    g = torch.Generator().manual_seed(seed)
    fixed = torch.tensor([0, 1, 63, 64, 65, T // 2, T - 65, T - 64, T - 1])
    rows = torch.cat([fixed, torch.randint(0, T, (n,), generator=g)]).unique()
    return rows[(rows >= 0) & (rows < T)]


def _check_rows(d, got, cfg, b, rows):
    """o, lse, dq of `rows` (dense, T == Tk) of batch b, all heads, against the oracle."""
    rd = rows.to(d["q"].device)
    q = d["q"][b, rd].float().cpu()
    k = d["k"][b].float().cpu()
    v = d["v"][b].float().cpu()
    idx = d["idx"][b, rd].cpu()
    ro, rl = O.sfa_rows_forward(q, k, v, idx, rows, cfg.bs, cfg.scale, None, cfg.causal)
    rg = rows.to(got["o"].device)
    assert_close(f"o[b={b}]", got["o"][b, rg].cpu(), ro)
    assert_lse(got["lse"][b, rg].cpu(), rl)
    o_op = got["o"][b, rg].float().cpu()            # delta from the op's own o, as the reference does
    rdq, _, _, _ = O.sfa_rows_backward(q, k, v, idx, rows, o_op, rl, d["do"][b, rd].float().cpu(), cfg.bs,
                                       cfg.scale, None, cfg.causal)
    assert_close(f"dq[b={b}]", got["dq"][b, rg].cpu(), rdq)


def _check_blocks(d, got, cfg, b, hk, blocks):
    """dk, dv of the keys of `blocks` (kv head hk, batch b) from their complete query lists."""
    G = cfg.Hq // cfg.Hk
    idx = d["idx"][b, :, hk]                          # [T, S]
    t = torch.arange(cfg.T, device=idx.device)
    sel = torch.zeros(cfg.T, dtype=torch.bool, device=idx.device)
    for e in blocks:
        sel |= (idx == e).any(-1) & (t >= e * cfg.bs)
    rd = sel.nonzero().flatten()
    rows = rd.cpu()
    hs = slice(hk * G, (hk + 1) * G)
    q = d["q"][b, rd, hs].float().cpu()
    k = d["k"][b, :, hk:hk + 1].float().cpu()
    v = d["v"][b, :, hk:hk + 1].float().cpu()
    ir = d["idx"][b, rd, hk:hk + 1].cpu()
    _, rl = O.sfa_rows_forward(q, k, v, ir, rows, cfg.bs, cfg.scale, None, cfg.causal)
    o_op = got["o"][b, rows.to(got["o"].device), hs].float().cpu()
    _, rdk, rdv, _ = O.sfa_rows_backward(q, k, v, ir, rows, o_op, rl, d["do"][b, rd, hs].float().cpu(), cfg.bs,
                                         cfg.scale, None, cfg.causal)
    for e in blocks:
        keys = slice(e * cfg.bs, (e + 1) * cfg.bs)
        assert_close(f"dk[b={b},hk={hk},blk={e}] ({rows.numel()} rows)", got["dk"][b, keys, hk].cpu(),
                     rdk[keys, 0])
        assert_close(f"dv[b={b},hk={hk},blk={e}]", got["dv"][b, keys, hk].cpu(), rdv[keys, 0])


def test_c2_full_size():
    cfg = W.CONFIGS["c2"]
    dev = torch.device("cuda")
    d = W.make_inputs(cfg, dev, seed=1000)
    got = _run_op(d, cfg, dev)
    for b in range(cfg.B):
        _check_rows(d, got, cfg, b, _sample_rows(cfg.T, 56, seed=b))
    nb = cfg.T // cfg.bs
    g = torch.Generator().manual_seed(7)
    for b, hk in ((0, 0), (1, 3), (2, 1), (3, 2)):
        extra = int(torch.randint(2, nb, (1,), generator=g))
        _check_blocks(d, got, cfg, b, hk, [b % 2, extra, nb - 1])


def test_c3_full_size():
    cfg = W.CONFIGS["c3"]
    dev = torch.device("cuda")
    d = W.make_inputs(cfg, dev, seed=1000)
    got = _run_op(d, cfg, dev)
    _check_rows(d, got, cfg, 0, _sample_rows(cfg.T, 120, seed=3))
    nb = cfg.T // cfg.bs
    _check_blocks(d, got, cfg, 0, 0, [1, nb // 2 + 5])
    _check_blocks(d, got, cfg, 0, 3, [nb - 3, nb - 1])


def test_c4_geometry_g128_shared_latent_kv():
    # Hq = 128 query heads on one latent kv head (D_qk 576 = 512 latent + 64
    # rope, v = kv[..., :512]), token-level causal top-k; T and k scaled so the
    # whole problem runs through the oracle
    cfg = W.scaled(W.CONFIGS["c4"], T=1024, S=256)
    dev = torch.device("cuda")
    d = W.make_inputs(cfg, "cpu", seed=5)
    assert d["v"].data_ptr() == d["k"].data_ptr()
    got = _run_op(d, cfg, dev)
    k, v = d["k"].float(), d["v"].float()
    ro, rl = O.sfa_forward(d["q"].float(), k, v, d["idx"], 1, cfg.scale, None, True)
    assert_close("o", got["o"].cpu(), ro)
    assert_lse(got["lse"].cpu(), rl)
    rdq, rdk, rdv, _ = O.sfa_backward(d["q"].float(), k, v, d["idx"], got["o"].float().cpu(), rl, d["do"].float(), 1,
                                      cfg.scale, None, True)
    assert_close("dq", got["dq"].cpu(), rdq)
    dkv = rdk.clone()
    dkv[..., :cfg.Dv] += rdv                           # one latent tensor: its gradient is dk + dv
    assert_close("dkv", got["dk"].cpu(), dkv)


def test_c5_full_size_forward():
    cfg = W.CONFIGS["c5"]
    dev = torch.device("cuda")
    d = W.make_decode(cfg, dev, seed=1000)
    o, lse = ops_b200.sparse_flash_attention(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale,
                                             cu_seqlens=d["cu_q"], cu_seqlens_k=d["cu_k"], max_seqlen_q=1,
                                             max_seqlen_k=d["max_k"])
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    kv_lens = d["kv_lens"].cpu()
    order = torch.argsort(kv_lens)
    g = torch.Generator().manual_seed(9)
    pick = torch.cat([order[:4], order[-4:], torch.randint(0, cfg.n_seqs, (16,), generator=g)]).unique()
    cu_k = d["cu_k"].cpu()
    for i in pick.tolist():
        k0, k1 = int(cu_k[i]), int(cu_k[i + 1])
        k = d["k"][k0:k1].float().cpu()
        v = d["v"][k0:k1].float().cpu()
        idx = d["idx"][i:i + 1].cpu()
        ro, rl = O.sfa_rows_forward(d["q"][i:i + 1].float().cpu(), k, v, idx, [k1 - k0 - 1], cfg.bs, cfg.scale,
                                    None, True)
        assert_close(f"o[seq {i}, kv {k1 - k0}]", o[i:i + 1].cpu(), ro)
        assert_lse(lse[i:i + 1].cpu(), rl)


@pytest.mark.parametrize("S,B,H,D,topk", [(1024, 2, 64, 128, 512), (256, 1, 128, 576, 128)])
def test_reference_signature_at_scale(S, B, H, D, topk):
    # the drop-in surface (SBHD, one shared kv head whose rows are keys and
    # values, token-level top-k, no causal mask) beyond the golden fixtures'
    # sizes; indices left-packed with a -1 tail on some rows, as the reference
    # expects them
    g = torch.Generator().manual_seed(S + H)
    q = torch.randn(S, B, H, D, generator=g).bfloat16()
    kv = torch.randn(S, B, D, generator=g).bfloat16()
    sink = torch.randn(H, generator=g)
    idx = torch.stack([torch.stack([torch.randperm(S, generator=g)[:topk] for _ in range(B)]) for _ in range(S)])
    idx = idx.to(torch.int32)
    idx[: S // 8, :, topk // 2:] = -1
    do = torch.randn(S, B, H, D, generator=g).bfloat16()
    dev = torch.device("cuda")
    qg = q.to(dev).requires_grad_()
    kvg = kv.to(dev).requires_grad_()
    sg = sink.to(dev).requires_grad_()
    out = ops_b200.SparseFlashAttention.apply(qg, kvg, sg, idx.to(dev), D ** -0.5)
    out.backward(do.to(dev))
    torch.cuda.synchronize()
    ro, rl = O.reference_compat_forward(q.float(), kv.float(), sink, idx, D ** -0.5)
    assert_close("out", out.detach().cpu(), ro)
    rdq, rdkv, rds = O.reference_compat_backward(q.float(), kv.float(), sink, idx, D ** -0.5,
                                                 out.detach().float().cpu(), rl, do.float())
    assert_close("dq", qg.grad.cpu(), rdq)
    assert_close("dkv", kvg.grad.cpu(), rdkv)
    assert_close("dsink", sg.grad.cpu(), rds)
