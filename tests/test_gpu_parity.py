"""GPU parity: the CUDA op against the CPU oracle on the same seeded inputs.

Shapes are the benchmark configurations scaled down so the oracle finishes in
seconds (config 1 runs at full size), plus the index edge cases: -1 in any
slot, all -1, ids past the last block, duplicates, the partial current block
under causal masking, varlen boundaries, shared k/v and the attention sink.
Each case runs through every kernel family that supports it.
"""
import math

import pytest
import torch

from ops_b200 import workloads as W
from sfa_check import check_all, run_op, run_oracle

pytestmark = pytest.mark.gpu

FAMILIES = ["auto", "general"]


def _dense_case(cfg, seed=0, sink=True):
    d = W.make_inputs(cfg, "cpu", seed)
    g = torch.Generator().manual_seed(seed + 100)
    s = torch.randn(cfg.Hq, generator=g) if sink else None
    return d, s


def _compare(cfg, d, sink, family, bwd=True, shared=False, dkv_mode="auto"):
    do = d["do"] if bwd else None
    v = d["k"] if shared else d["v"]
    got = run_op(d["q"], d["k"], v, d["idx"], cfg.bs, cfg.scale, sink, cfg.causal, do,
                 kernel=family, shared_kv=shared, dkv_mode=dkv_mode)
    ref = run_oracle(d["q"], d["k"], v, d["idx"], cfg.bs, cfg.scale, sink, cfg.causal, do,
                     o_for_bwd=got["o"])
    check_all(got, ref, shared_kv=shared, grads=bwd)
    return got


@pytest.mark.parametrize("family", FAMILIES)
def test_config1_full_size(family):
    cfg = W.CONFIGS["c1"]
    d, s = _dense_case(cfg)
    _compare(cfg, d, s, family)


@pytest.mark.parametrize("family", FAMILIES)
def test_config2_shape_scaled(family):
    cfg = W.scaled(W.CONFIGS["c2"], B=2, T=1024, Hq=32, Hk=2, S=8)
    d, s = _dense_case(cfg, seed=1)
    _compare(cfg, d, s, family)


@pytest.mark.parametrize("family", FAMILIES)
def test_config3_recent_bias_scaled(family):
    cfg = W.scaled(W.CONFIGS["c3"], T=2048, Hq=32, Hk=2, S=16)
    d, s = _dense_case(cfg, seed=2, sink=False)
    _compare(cfg, d, s, family)


@pytest.mark.parametrize("family", FAMILIES)
def test_config4_mla_token_level_scaled(family):
    cfg = W.scaled(W.CONFIGS["c4"], T=384, Hq=16, S=96)
    d, s = _dense_case(cfg, seed=3)
    _compare(cfg, d, s, family)


@pytest.mark.parametrize("family", FAMILIES)
def test_config5_varlen_decode_scaled(family):
    cfg = W.scaled(W.CONFIGS["c5"], n_seqs=8, kv_min=200, kv_max=3000, Hq=16, Hk=2, S=8)
    d = W.make_inputs(cfg, "cpu", 4)
    g = torch.Generator().manual_seed(44)
    sink = torch.randn(cfg.Hq, generator=g)
    got = run_op(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, sink, True, d["do"], d["cu_q"], d["cu_k"],
                 1, d["max_k"], kernel=family)
    ref = run_oracle(d["q"], d["k"], d["v"], d["idx"], cfg.bs, cfg.scale, sink, True, d["do"], d["cu_q"],
                     d["cu_k"], o_for_bwd=got["o"])
    check_all(got, ref)


def _edge_inputs(seed=11, B=2, T=200, Hq=16, Hk=2, D=64, bs=16, S=6):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hq, D, generator=g).bfloat16()
    k = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    v = torch.randn(B, T, Hk, D, generator=g).bfloat16()
    do = torch.randn(B, T, Hq, D, generator=g).bfloat16()
    nb = (T + bs - 1) // bs
    idx = torch.randint(-1, nb + 3, (B, T, Hk, S), generator=g, dtype=torch.int32)   # ids past the end too
    idx[:, 0] = -1                                  # first query: nothing valid
    idx[:, 5, :, 0] = -1                            # -1 in front of valid entries
    idx[:, 7, :, 2] = idx[:, 7, :, 1]               # duplicate entry
    idx[:, 9, :, :] = 9 // bs                       # the same (current, partial) block in every slot
    idx[1, 3:9, 1, :] = -1                          # a run of empty rows in one head
    return q, k, v, do, idx


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("with_sink", [True, False])
def test_index_edge_cases(family, causal, with_sink):
    q, k, v, do, idx = _edge_inputs()
    sink = torch.randn(q.shape[2], generator=torch.Generator().manual_seed(3)) if with_sink else None
    got = run_op(q, k, v, idx, 16, None, sink, causal, do, kernel=family)
    ref = run_oracle(q, k, v, idx, 16, None, sink, causal, do, o_for_bwd=got["o"])
    check_all(got, ref)
    # query 0 has no valid key: o = 0, lse = -inf (or the sink), zero dq
    assert got["o"][:, 0].abs().max() == 0
    if not with_sink:
        assert torch.isneginf(got["lse"][:, 0]).all()
        assert got["dq"][:, 0].abs().max() == 0


@pytest.mark.parametrize("family", FAMILIES)
def test_shared_kv_and_default_scale(family):
    q, k, v, do, idx = _edge_inputs(seed=12, T=130, D=128, bs=64, S=3)
    got = run_op(q, k, k, idx, 64, None, None, True, do, kernel=family, shared_kv=True)
    ref = run_oracle(q, k, k, idx, 64, 1.0 / math.sqrt(128), None, True, do, o_for_bwd=got["o"])
    check_all(got, ref, shared_kv=True)


@pytest.mark.parametrize("family", FAMILIES)
@pytest.mark.parametrize("G", [1, 8, 12, 32])
def test_group_sizes(family, G):
    Hk = 2
    q, k, v, do, idx = _edge_inputs(seed=13 + G, Hq=G * Hk, Hk=Hk, T=96, bs=32, S=3)
    got = run_op(q, k, v, idx, 32, 0.1, None, True, do, kernel=family)
    ref = run_oracle(q, k, v, idx, 32, 0.1, None, True, do, o_for_bwd=got["o"])
    check_all(got, ref)


@pytest.mark.parametrize("family", FAMILIES)
def test_varlen_boundaries(family):
    g = torch.Generator().manual_seed(21)
    q_lens = [1, 70, 64, 3]
    k_lens = [5, 70, 130, 200]   # q_len <= k_len: bottom-right aligned causal
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, Hk, D, bs, S = 16, 1, 64, 16, 5
    q = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    k = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    v = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    do = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    idx = torch.randint(-1, 14, (int(cu_q[-1]), Hk, S), generator=g, dtype=torch.int32)
    got = run_op(q, k, v, idx, bs, None, None, True, do, cu_q, cu_k, max(q_lens), max(k_lens), kernel=family)
    ref = run_oracle(q, k, v, idx, bs, None, None, True, do, cu_q, cu_k, o_for_bwd=got["o"])
    check_all(got, ref)
