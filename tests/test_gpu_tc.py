"""The tcgen05 family against the oracle, forced (kernel="tcgen05"), on every
shape it supports: block_size 64, D in {64, 128}, up to 16 query heads per kv
head, topk <= 64, dense and varlen, with the index edge cases."""
import pytest
import torch

from ops_b200 import workloads as W
from sfa_check import check_all, run_op, run_oracle

pytestmark = pytest.mark.gpu


def _case(cfg, seed, sink=True):
    d = W.make_inputs(cfg, "cpu", seed)
    s = torch.randn(cfg.Hq, generator=torch.Generator().manual_seed(seed + 100)) if sink else None
    return d, s


@pytest.mark.parametrize("cfg", [
    W.CONFIGS["c1"],
    W.scaled(W.CONFIGS["c2"], B=2, T=1024, Hq=32, Hk=2, S=8),
    W.scaled(W.CONFIGS["c2"], B=1, T=4096, Hq=16, Hk=1, S=16),
    W.scaled(W.CONFIGS["c3"], T=2048, Hq=32, Hk=2, S=32),
], ids=["c1", "c2s", "c2s_long", "c3s_two_segments"])
def test_tc_forward_backward(cfg):
    d, s = _case(cfg, 5)
    got = run_op(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, s, True, d["do"], kernel="tcgen05")
    ref = run_oracle(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, s, True, d["do"], o_for_bwd=got["o"])
    check_all(got, ref)


@pytest.mark.parametrize("dq_mode", ["separate", "fused"])
@pytest.mark.parametrize("cfg,shared", [
    (W.scaled(W.CONFIGS["c2"], B=2, T=1024, Hq=32, Hk=2, S=8), False),
    (W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hq=8, Hk=1, S=16, Dqk=64, Dv=64), False),
    (W.scaled(W.CONFIGS["c2"], B=1, T=1500, Hq=12, Hk=1, S=12), True),
], ids=["g16_d128", "g8_d64", "g12_shared_kv"])
def test_tc_dq_modes(cfg, shared, dq_mode):
    # dQ in its own query-centric pass, or accumulated by the key-centric dK/dV
    # pass (fp32 reductions): both against the oracle
    d, s = _case(cfg, 13)
    v = d["k"] if shared else d["v"]
    got = run_op(d["q"], d["k"], v, d["idx"], cfg.bs, cfg.scale, s, True, d["do"], kernel="tcgen05",
                 dkv_mode="inverted", shared_kv=shared, dq_mode=dq_mode)
    ref = run_oracle(d["q"], d["k"], v, d["idx"], cfg.bs, cfg.scale, s, True, d["do"], o_for_bwd=got["o"])
    check_all(got, ref, shared_kv=shared)


def test_tc_forward_decode_varlen():
    cfg = W.scaled(W.CONFIGS["c5"], n_seqs=8, kv_min=200, kv_max=5000, Hq=16, Hk=2, S=32)
    d = W.make_inputs(cfg, "cpu", 4)
    got = run_op(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, None, True, None, d["cu_q"], d["cu_k"],
                 1, d["max_k"], kernel="tcgen05")
    ref = run_oracle(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, None, True, None, d["cu_q"], d["cu_k"])
    check_all(got, ref, grads=False)


@pytest.mark.parametrize("G", [1, 8, 12, 16])
@pytest.mark.parametrize("causal", [True, False])
def test_tc_forward_edge_indices(G, causal):
    g = torch.Generator().manual_seed(31 + G)
    B, T, Hk, D, bs, S = 2, 300, 2, 128, 64, 7
    q = torch.randn(B, T, G * Hk, D, generator=g).bfloat16()
    k = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    v = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    nb = (T + bs - 1) // bs
    idx = torch.randint(-1, nb + 2, (B, T, Hk, S), generator=g, dtype=torch.int32)
    idx[:, 0] = -1
    idx[:, 5, :, 0] = -1
    idx[:, 70, :, 2] = idx[:, 70, :, 1]
    idx[:, 90, :, :] = 1
    sink = torch.randn(G * Hk, generator=g)
    do = torch.randn(B, T, G * Hk, D, generator=g).bfloat16()
    got = run_op(q, k, v, idx, bs, None, sink, causal, do, kernel="tcgen05")
    ref = run_oracle(q, k, v, idx, bs, None, sink, causal, do, o_for_bwd=got["o"])
    check_all(got, ref)


def test_tc_matches_general_family():
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hq=16, Hk=1, S=16)
    d, s = _case(cfg, 9)
    a = run_op(d["q"], d["k"], d["v"], d["idx"], 64, None, s, True, None, kernel="tcgen05")
    b = run_op(d["q"], d["k"], d["v"], d["idx"], 64, None, s, True, None, kernel="general")
    assert (a["o"].float() - b["o"].float()).abs().max() < 2e-2
    assert (a["lse"] - b["lse"]).abs().max() < 1e-3


def test_tc_reference_sbhd_strides():
    # the SBHD layout of the reference signature, block-level through the generalised API
    g = torch.Generator().manual_seed(77)
    S_, B, H, D = 256, 2, 16, 64
    q = torch.randn(S_, B, H, D, generator=g).bfloat16()
    kv = torch.randn(S_, B, D, generator=g).bfloat16()
    qb = q.permute(1, 0, 2, 3)
    kvb = kv.permute(1, 0, 2).unsqueeze(2)
    idx = torch.randint(-1, 4, (B, S_, 1, 4), generator=g, dtype=torch.int32)
    got = run_op(qb, kvb, kvb, idx, 64, None, None, True, None, kernel="tcgen05")
    ref = run_oracle(qb.contiguous(), kvb.contiguous(), kvb.contiguous(), idx, 64, None, None, True)
    check_all(got, ref, grads=False)


@pytest.mark.parametrize("dq_mode", ["separate", "fused"])
def test_tc_long_rows_and_varlen_row_ranges(dq_mode):
    # q_len > 2048 splits the fused key-centric pass into row ranges whose
    # dK/dV partials are summed afterwards: dense and varlen (sequences of
    # different lengths, bottom-right causal alignment, blocks of 64)
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=5000, Hq=16, Hk=1, S=16)
    d, s = _case(cfg, 17)
    got = run_op(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, s, True, d["do"], kernel="tcgen05",
                 dkv_mode="inverted", dq_mode=dq_mode)
    ref = run_oracle(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, s, True, d["do"], o_for_bwd=got["o"])
    check_all(got, ref)

    g = torch.Generator().manual_seed(23)
    q_lens, k_lens = [3000, 700, 2500], [3000, 900, 2600]
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, Hk, D, bs, S = 16, 2, 128, 64, 12
    q = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    k = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    v = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    do = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    idx = torch.randint(-1, 47, (int(cu_q[-1]), Hk, S), generator=g, dtype=torch.int32)
    got = run_op(q, k, v, idx, bs, None, None, True, do, cu_q, cu_k, max(q_lens), max(k_lens), kernel="tcgen05",
                 dkv_mode="inverted", dq_mode=dq_mode)
    ref = run_oracle(q, k, v, idx, bs, None, None, True, do, cu_q, cu_k, o_for_bwd=got["o"])
    check_all(got, ref)
