"""Host-side logic on the CPU: index generation for the benchmark configs,
FLOP/pair accounting, the tiling layer, and input validation of the Python
surface (which must refuse CPU tensors — there is no CPU implementation)."""
import os

import pytest
import torch

from oracle import sfa_oracle as O
from ops_b200 import tiling, workloads as W


def test_uniform_causal_indices_follow_the_config_rules():
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hk=2, S=16)
    idx = W.make_indices(cfg)
    T = cfg.T
    cur = torch.arange(T) // cfg.bs
    for h in range(cfg.Hk):
        sel = idx[0, :, h]
        assert (sel == cur[:, None]).any(1).all(), "current block always included"
        valid = sel >= 0
        assert ((sel <= cur[:, None]) | ~valid).all(), "causal range"
        n_avail = torch.clamp(cur + 1, max=cfg.S)
        assert torch.equal(valid.sum(1), n_avail), "-1 only when fewer blocks exist"
        for t in (0, 100, 2047):
            s = sel[t][sel[t] >= 0]
            assert len(set(s.tolist())) == len(s), "without replacement"


def test_recent_biased_indices():
    cfg = W.scaled(W.CONFIGS["c3"], T=4096, Hk=1, S=32)
    idx = W.make_indices(cfg)
    cur = torch.arange(cfg.T) // cfg.bs
    late = idx[0, 2048:, 0].long()
    recent = (late > cur[2048:, None] - 8) & (late >= 0)
    # with half the mass on 8 blocks, nearly all of them are picked
    assert recent.sum(1).float().mean() > 7.5


def test_token_level_indices():
    cfg = W.scaled(W.CONFIGS["c4"], T=300, S=64)
    idx = W.make_indices(cfg)
    t = torch.arange(cfg.T)
    sel = idx[0, :, 0]
    assert ((sel <= t[:, None]) | (sel < 0)).all()
    assert torch.equal((sel >= 0).sum(1), torch.clamp(t + 1, max=64))


def test_decode_inputs():
    cfg = W.scaled(W.CONFIGS["c5"], n_seqs=6, kv_min=100, kv_max=900, Hq=8, Hk=2, S=4)
    d = W.make_decode(cfg)
    assert d["q"].shape == (6, 8, 128) and d["cu_q"].tolist() == list(range(7))
    nb = (d["kv_lens"] + 63) // 64
    valid = d["idx"] >= 0
    assert ((d["idx"] < nb[:, None, None]) | ~valid).all()
    assert torch.equal(valid.sum(-1), torch.clamp(nb, max=4)[:, None].expand(-1, 2))


@pytest.mark.parametrize("name", ["c1"])
def test_pair_count_matches_oracle(name):
    cfg = W.CONFIGS[name]
    idx = W.make_indices(cfg)
    a = W.count_pairs(idx, cfg.bs, cfg.T, cfg.T)
    b = O.selected_pairs(idx, cfg.bs, cfg.T, cfg.T)
    assert a == b
    f = W.sfa_flops(a * cfg.Hq // cfg.Hk, cfg.Dqk, cfg.Dv)
    assert 4.5e9 < f.total < 6e9   # about 5.4 GFLOP for config 1
    # the bench's formula and the oracle's accounting agree
    g = O.sfa_flops(a * cfg.Hq // cfg.Hk, cfg.Dqk, cfg.Dv)
    assert (f.fwd, f.bwd) == (g.fwd, g.bwd)


def test_block_indices_as_tokens_select_the_same_pairs():
    # c1's block indices expanded to token level select the same (query, key)
    # pairs, partial blocks and -1 slots included
    cfg = W.scaled(W.CONFIGS["c1"], T=1000)
    idx = W.make_indices(cfg)
    tok = W.blocks_to_tokens(idx, cfg.bs)
    assert tok.shape == (*idx.shape[:-1], idx.shape[-1] * cfg.bs)
    assert W.count_pairs(idx, cfg.bs, cfg.T, cfg.T) == W.count_pairs(tok, 1, cfg.T, cfg.T)
    assert ((tok < 0) == (idx < 0).repeat_interleave(cfg.bs, -1)).all()


def test_reference_tiling_buckets():
    assert tiling.resolve_tiling_config(128).BLOCK_N == 64
    assert tiling.resolve_tiling_config(150).BLOCK_K_BWD == 40
    assert tiling.resolve_tiling_config(2048).BLOCK_K_BWD == 64
    with pytest.raises(ValueError):
        tiling.resolve_tiling_config(0)
    assert tiling.effective_topk(torch.tensor([[[1, 2, -1]], [[-1, -1, -1]]])) == 2
    with pytest.raises(ValueError):
        tiling.effective_topk(torch.empty(0))


def test_python_surface_refuses_cpu_tensors():
    import ops_b200
    q = torch.randn(1, 4, 2, 8).bfloat16()
    k = torch.randn(1, 4, 1, 8).bfloat16()
    idx = torch.zeros(1, 4, 1, 1, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        ops_b200.sparse_flash_attention(q, k, k, idx, 4)


def test_oracle_index_semantics():
    # block 1 of size 4 for a query at position 5: keys 4,5 valid, 6,7 masked
    keys, ok = O.key_table(torch.tensor([[1, -1, 9, 1]]), 4, torch.tensor([5]), 10, True)
    assert keys[0, :4].tolist() == [4, 5, 0, 0] and ok[0, :4].tolist() == [True, True, False, False]
    assert not ok[0, 4:8].any()              # -1
    assert not ok[0, 8:12].any()             # block 9 is past kv_len 10 (blocks 0..2)
    assert ok[0, 12:].tolist() == [True, True, False, False]   # duplicate counts again


def test_reference_arm_prints_one_contract_line():
    # the reference arm (the CPU restatement) runs without a GPU: its one JSON
    # line must carry the contract's keys, with e2e equal to the value and no
    # host/device copies
    import json
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--config", "c1",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("c1")


def test_valid_key_mask_matches_the_oracle_rule():
    # the reference-quirk lse marks rows with no valid key; the mask follows
    # the kernels' (and the oracle's) validity rule, dense and varlen
    from ops_b200 import sfa as S
    g = torch.Generator().manual_seed(3)
    B, T, Hk, G, Sl, bs = 2, 40, 2, 3, 4, 8
    idx = torch.randint(-1, 7, (B, T, Hk, Sl), generator=g, dtype=torch.int32)
    idx[:, :5] = -1
    for causal in (True, False):
        cfg = S._Cfg(bs, 1.0, causal, False, T, T, 0, 0, False)
        got = S._has_valid_key(idx, cfg, None, None, Hk * G, Hk)
        pos = torch.arange(T)
        for b in range(B):
            for h in range(Hk):
                _, ok = O.key_table(idx[b, :, h], bs, pos, T, causal)
                assert torch.equal(got[b, :, h * G:(h + 1) * G], ok.any(-1)[:, None].expand(T, G))
    q_lens, k_lens = [3, 10, 1], [5, 30, 12]
    cu_q = torch.tensor([0, 3, 13, 14], dtype=torch.int32)
    cu_k = torch.tensor([0, 5, 35, 47], dtype=torch.int32)
    vidx = torch.randint(-1, 5, (14, Hk, Sl), generator=g, dtype=torch.int32)
    cfg = S._Cfg(bs, 1.0, True, True, 10, 30, 0, 0, False)
    got = S._has_valid_key(vidx, cfg, cu_q, cu_k, Hk * G, Hk)
    for i in range(3):
        q0, q1, kl = int(cu_q[i]), int(cu_q[i + 1]), k_lens[i]
        pos = torch.arange(q1 - q0) + kl - (q1 - q0)
        for h in range(Hk):
            _, ok = O.key_table(vidx[q0:q1, h], bs, pos, kl, True)
            assert torch.equal(got[q0:q1, h * G:(h + 1) * G], ok.any(-1)[:, None].expand(q1 - q0, G))


def test_page_kv_keeps_every_row_and_table_maps_back():
    # the paged layout holds every sequence's rows once, at the rows the block
    # table names (the kernels' mapping: page table[s][t // ps], row t % ps)
    g = torch.Generator().manual_seed(4)
    lens = torch.tensor([5, 64, 65, 130])
    cu = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)])
    k = torch.randn(int(cu[-1]), 2, 8, generator=g)
    v = torch.randn(int(cu[-1]), 2, 4, generator=g)
    kp, vp, table = W.page_kv(k, v, cu, 64, seed=1)
    assert kp.shape[1:] == (64, 2, 8) and vp.shape[1:] == (64, 2, 4)
    assert kp.shape[0] == int(((lens + 63) // 64).sum())
    for s in range(lens.numel()):
        t = torch.arange(int(lens[s]))
        pg = table[s, t // 64].long()
        assert torch.equal(kp[pg, t % 64], k[cu[s] + t])
        assert torch.equal(vp[pg, t % 64], v[cu[s] + t])
    assert sorted(table[table >= 0].tolist()) == list(range(kp.shape[0]))


def test_indexer_oracle_selection_rule():
    from oracle import indexer_oracle as IO
    # scores with ties: the lower index wins, output ascending, -1 tail
    sc = torch.tensor([[[1.0, 3.0, 3.0, 2.0, 3.0, 0.5]]])
    q = torch.zeros(1, 1, 1, 1)
    k = torch.zeros(1, 6, 1)
    w = torch.zeros(1, 1, 1)
    got = IO.indexer_topk(q, k, w, 2, causal=False, scores=sc)
    assert got.tolist() == [[[1, 2]]]
    got = IO.indexer_topk(q, k, w, 4, causal=False, scores=sc)
    assert got.tolist() == [[[1, 2, 3, 4]]]
    got = IO.indexer_topk(q, k, w, 8, causal=False, scores=sc)
    assert got.tolist() == [[[0, 1, 2, 3, 4, 5, -1, -1]]]
    # causal with Tq == Tk: row t sees keys 0..t
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 5, 2, 4, generator=g)
    k = torch.randn(1, 5, 4, generator=g)
    w = torch.rand(1, 5, 2, generator=g)
    got = IO.indexer_topk(q, k, w, 3, causal=True)
    assert got[0, 0].tolist() == [0, -1, -1] and got[0, 1].tolist() == [0, 1, -1]
    assert (got[0, 4] >= 0).all()


def test_fp8_kv_quantisation_is_exact_in_bf16():
    # power-of-two row scales: e4m3 value * scale is a bf16 value, so the
    # kernels' widening to bf16 loses nothing beyond the e4m3 rounding itself
    from ops_b200.sfa import quantize_kv_fp8
    g = torch.Generator().manual_seed(2)
    kv = (torch.randn(3, 50, 1, 576, generator=g) * torch.rand(3, 50, 1, 1, generator=g) * 30).bfloat16()
    kv[0, 0] = 0
    q8, sc = quantize_kv_fp8(kv)
    assert q8.dtype == torch.float8_e4m3fn and sc.shape == kv.shape[:-1]
    assert torch.equal(torch.log2(sc), torch.round(torch.log2(sc)))            # powers of two
    deq = q8.float() * sc[..., None]
    assert torch.equal(deq.bfloat16().float(), deq)                             # exact in bf16
    rel = ((deq - kv.float()).abs() / kv.float().abs().amax(-1, keepdim=True).clamp_min(1e-6)).max()
    assert float(rel) <= 2 ** -4                                                # e4m3: 3 mantissa bits


def test_e2e_chunks_cover_every_unit_row_once():
    """bench's end-to-end pipeline cuts each (batch, kv head) unit into row
    ranges when a rank has fewer than 8 units: every row of every unit falls
    in exactly one range, in order, with the unit's first and last marked."""
    import bench
    for name in ("c1", "c2", "c3", "c4", "tok128"):
        cfg = W.CONFIGS[name]
        for world in (1, 2, 4, 8):
            units = bench.unit_range(cfg, world, world - 1)
            if units is None:
                continue
            b0, b1, h0, h1 = units
            per_unit = {}
            for b, h, r0, r1, first, last in bench.e2e_chunks(cfg, "units", units):
                per_unit.setdefault((b, h), []).append((r0, r1, first, last))
            assert sorted(per_unit) == [(b, h) for b in range(b0, b1) for h in range(h0, h1)], (name, world)
            for rs in per_unit.values():
                assert rs[0][0] == 0 and rs[-1][1] == cfg.T
                assert all(a[1] == c[0] and a[0] < a[1] for a, c in zip(rs, rs[1:]))
                assert [x[2] for x in rs] == [True] + [False] * (len(rs) - 1)
                assert [x[3] for x in rs] == [False] * (len(rs) - 1) + [True]
    assert bench.e2e_chunks(W.CONFIGS["c2"], "query", (0, 4, 0, 4)) == [None]


def test_row_ranges_over_leading_keys_reproduce_the_whole_op():
    """What the e2e row ranges rely on: rows [r0, r1) against keys [0, r1)
    keep every row's causal position (bottom-right alignment), so o, lse and
    dq of a range equal the whole op's rows, and the ranges' dk / dv partials
    sum to the whole op's dk / dv."""
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=320, Hq=4, Hk=1, S=4)
    d = W.make_inputs(cfg, "cpu", 0)
    q, k, v, do = (d[n].float() for n in ("q", "k", "v", "do"))
    idx = d["idx"]
    o, lse = O.sfa_forward(q, k, v, idx, cfg.bs, cfg.scale)
    dq, dk, dv, _ = O.sfa_backward(q, k, v, idx, o, lse, do, cfg.bs, cfg.scale)
    dk_sum, dv_sum = torch.zeros_like(dk), torch.zeros_like(dv)
    for r0, r1 in ((0, 96), (96, 200), (200, 320)):
        oc, lc = O.sfa_forward(q[:, r0:r1], k[:, :r1], v[:, :r1], idx[:, r0:r1], cfg.bs, cfg.scale)
        dqc, dkc, dvc, _ = O.sfa_backward(q[:, r0:r1], k[:, :r1], v[:, :r1], idx[:, r0:r1], oc, lc, do[:, r0:r1],
                                          cfg.bs, cfg.scale)
        torch.testing.assert_close(oc, o[:, r0:r1], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(lc, lse[:, r0:r1], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dqc, dq[:, r0:r1], rtol=1e-5, atol=1e-5)
        dk_sum[:, :r1] += dkc
        dv_sum[:, :r1] += dvc
    torch.testing.assert_close(dk_sum, dk, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dv_sum, dv, rtol=1e-4, atol=1e-4)
