"""GPU parity of the token-level (block_size 1) tensor-core forward against the
CPU oracle: the reference's own operating mode (one kv row per index,
SFA.py:399-415) and the MLA geometry (128 query heads on one latent kv head,
D_qk 576 / D_v 512, V = the latent's first 512 dims).

Cases cover head tiles below, at and above 128 heads, D_v split into 256-dim
parts, top-k counts that leave a partial last chunk, -1 / out-of-range /
duplicate indices, rows with nothing selected, causal and non-causal,
varlen, the attention sink, scores that force the running output to be
rescaled, and the reference signature (SBHD, shared kv)."""
import ctypes

import pytest
import torch

import ops_b200
from ops_b200 import _lib
from ops_b200 import sfa as S
from oracle import sfa_oracle as O
from sfa_check import assert_close, assert_lse

pytestmark = pytest.mark.gpu


def _inputs(B, T, Hq, Hk, Dqk, Dv, K, seed, shared=False, causal=True, edge=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hq, Dqk, generator=g).bfloat16()
    k = torch.randn(B, T, Hk, Dqk, generator=g).bfloat16()
    v = k[..., :Dv] if shared else torch.randn(B, T, Hk, Dv, generator=g).bfloat16()
    if causal:
        u = torch.rand(B, T, Hk, T, generator=g)
        t = torch.arange(T)
        u = torch.where(t[None, None, None, :] <= t[None, :, None, None], u, torch.full_like(u, 2.0))
        val, idx = torch.topk(u, min(K, T), dim=-1, largest=False)
        idx = torch.where(val < 2.0, idx, torch.full_like(idx, -1))
    else:
        idx = torch.stack([torch.randperm(T, generator=g)[:K] for _ in range(B * T * Hk)]).view(B, T, Hk, K)
    idx = idx.to(torch.int32)
    if edge:
        idx[:, 1] = -1                                   # nothing selected
        idx[:, 2, :, 0] = -1                             # -1 in front
        idx[:, 3, :, 1] = T + 5                          # past the end
        idx[:, 4, :, 2] = idx[:, 4, :, 3]                # duplicate slot
        idx[:, T // 2, :, ::3] = -1                      # holes
    return q, k, v, idx


def _check_fwd(q, k, v, idx, causal, sink=None, scale=None):
    dev = torch.device("cuda")
    shared = v.data_ptr() == k.data_ptr()
    kd = k.to(dev)
    vd = kd[..., :v.shape[-1]] if shared else v.to(dev)
    o, lse = ops_b200.sparse_flash_attention(q.to(dev), kd, vd, idx.to(dev), 1, scale,
                                             attn_sink=None if sink is None else sink.to(dev), causal=causal,
                                             kernel="tcgen05")
    torch.cuda.synchronize()
    ro, rl = O.sfa_forward(q.float(), k.float(), v.float(), idx, 1, scale, sink, causal)
    assert_close("o", o.cpu(), ro)
    assert_lse(lse.cpu(), rl)
    return o.cpu(), lse.cpu()


@pytest.mark.parametrize("Hq,Hk,Dqk,Dv,K", [
    (16, 1, 64, 64, 128),       # small head tile (rows 16..127 padded)
    (64, 2, 128, 128, 100),     # partial last chunk
    (128, 1, 576, 512, 256),    # MLA: two V parts, nine 64-dim slabs of q/k
    (256, 1, 128, 128, 64),     # two 128-head tiles
    (32, 1, 192, 320, 130),     # odd slab counts: 3 q/k slabs, V parts of 256 + 64
])
def test_token_level_forward(Hq, Hk, Dqk, Dv, K):
    q, k, v, idx = _inputs(2, 300, Hq, Hk, Dqk, Dv, K, seed=Hq + Dqk, edge=True)
    sink = torch.randn(Hq, generator=torch.Generator().manual_seed(1))
    _check_fwd(q, k, v, idx, True, sink)


def test_mla_shared_latent_kv_non_causal():
    q, k, v, idx = _inputs(1, 640, 128, 1, 576, 512, 512, seed=7, shared=True, causal=False)
    _check_fwd(q, k, v, idx, False, scale=576 ** -0.5)


def test_empty_rows_give_zero_and_sink_or_neg_inf():
    q, k, v, idx = _inputs(1, 64, 16, 1, 64, 64, 64, seed=3)
    idx[:, ::2] = -1
    o, lse = _check_fwd(q, k, v, idx, True)
    assert o[:, ::2].abs().max() == 0 and torch.isneginf(lse[:, ::2]).all()
    sink = torch.randn(16, generator=torch.Generator().manual_seed(2))
    o, lse = _check_fwd(q, k, v, idx, True, sink)
    assert o[:, ::2].abs().max() == 0 and torch.allclose(lse[0, ::2], sink.expand(32, 16))


def test_large_scores_rescale_the_running_output():
    # scores growing along the index list raise the running maximum by more
    # than the rescale threshold several times within a row
    q, k, v, _ = _inputs(1, 256, 32, 1, 128, 128, 64, seed=5, causal=False)
    ramp = torch.linspace(0.2, 6.0, 256)[:, None, None]
    k = (k[0].float() * ramp).bfloat16()[None]
    idx = torch.arange(256, dtype=torch.int32).expand(1, 256, 1, 256).contiguous()
    _check_fwd(q, k, v, idx, False, scale=0.5)


def test_varlen_token_level():
    g = torch.Generator().manual_seed(11)
    q_lens, k_lens = [5, 130, 64], [40, 130, 300]
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, Hk, D, K = 32, 2, 128, 96
    q = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    k = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    v = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    idx = torch.randint(-1, 310, (int(cu_q[-1]), Hk, K), generator=g, dtype=torch.int32)
    dev = torch.device("cuda")
    o, lse = ops_b200.sparse_flash_attention(q.to(dev), k.to(dev), v.to(dev), idx.to(dev), 1,
                                             cu_seqlens=cu_q.to(dev), cu_seqlens_k=cu_k.to(dev),
                                             max_seqlen_q=max(q_lens), max_seqlen_k=max(k_lens), kernel="tcgen05")
    ro, rl = O.sfa_forward(q.float(), k.float(), v.float(), idx, 1, None, None, True, cu_q, cu_k)
    assert_close("o", o.cpu(), ro)
    assert_lse(lse.cpu(), rl)


def test_reference_signature_runs_on_tensor_cores():
    # SparseFlashAttention.apply (SBHD, shared kv) picks the token-level
    # tensor-core forward; its output matches the oracle
    Sq, B, H, D, K = 256, 2, 64, 128, 200
    g = torch.Generator().manual_seed(4)
    q = torch.randn(Sq, B, H, D, generator=g).bfloat16()
    kv = torch.randn(Sq, B, D, generator=g).bfloat16()
    sink = torch.randn(H, generator=g)
    idx = torch.stack([torch.randperm(Sq, generator=g)[:K] for _ in range(Sq * B)]).view(Sq, B, K).to(torch.int32)
    dev = torch.device("cuda")
    qd, kvd, idd = q.to(dev), kv.to(dev), idx.to(dev)
    out = torch.empty_like(qd)
    lse = torch.empty(Sq, B, H, device=dev)
    cfg = S._Cfg(1, D ** -0.5, False, False, Sq, Sq, 0, 0, True)
    kvb = kvd.permute(1, 0, 2).unsqueeze(2)
    P = S.build_params(qd.permute(1, 0, 2, 3), kvb, kvb, idd.permute(1, 0, 2).unsqueeze(2),
                       out.permute(1, 0, 2, 3), lse.permute(1, 0, 2), cfg)
    assert _lib.load().sfa_select_kernel(ctypes.byref(P), 0) == _lib.SFA_KERNEL_TCGEN05
    o = ops_b200.SparseFlashAttention.apply(qd, kvd, sink.to(dev), idd, D ** -0.5)
    torch.cuda.synchronize()
    ro, _ = O.reference_compat_forward(q.float(), kv.float(), sink, idx, D ** -0.5)
    assert_close("out", o.cpu(), ro)


# ---------------------------------------------------------------------------
# backward (head dims up to 256): dq directly, dk / dv through fp32 reductions
# ---------------------------------------------------------------------------
def _check_fwd_bwd(q, k, v, idx, causal, sink=None, scale=None, shared=False):
    from sfa_check import check_all, run_op, run_oracle
    got = run_op(q, k, v, idx, 1, scale, sink, causal, _do(q, v), kernel="tcgen05", shared_kv=shared)
    ref = run_oracle(q, k, v, idx, 1, scale, sink, causal, _do(q, v), o_for_bwd=got["o"])
    check_all(got, ref, shared_kv=shared)


def _do(q, v):
    g = torch.Generator().manual_seed(q.shape[-2] * 7 + v.shape[-1])
    return torch.randn(*q.shape[:-1], v.shape[-1], generator=g).bfloat16()


@pytest.mark.parametrize("Hq,Hk,Dqk,Dv,K,shared", [
    (16, 1, 64, 64, 128, False),      # padded head tile, one-slab tiles
    (64, 2, 128, 128, 100, False),    # separate dK / dV tiles, partial last chunk
    (128, 1, 128, 128, 256, True),    # one kv tensor: dV adds into the dK tiles
    (64, 1, 256, 256, 192, True),     # D = 256 merged: TMEM fully used
    (32, 1, 192, 128, 64, False),     # odd slab counts
])
def test_token_level_backward(Hq, Hk, Dqk, Dv, K, shared):
    q, k, v, idx = _inputs(2, 260, Hq, Hk, Dqk, Dv, K, seed=Hq + Dqk + 1, edge=True)
    if shared:
        v = k
    sink = torch.randn(Hq, generator=torch.Generator().manual_seed(8))
    _check_fwd_bwd(q, k, v, idx, True, sink, shared=shared)


def test_token_level_backward_latent_view():
    # v is k's leading dims (one latent tensor): one fp32-summed dk + dv
    q, k, _, idx = _inputs(1, 200, 32, 1, 192, 128, 96, seed=13)
    dev = torch.device("cuda")
    qd = q.to(dev).requires_grad_()
    kd = k.to(dev).requires_grad_()
    do = _do(q, k[..., :128])
    o, _ = ops_b200.sparse_flash_attention(qd, kd, kd[..., :128], idx.to(dev), 1, kernel="tcgen05")
    o.backward(do.to(dev))
    torch.cuda.synchronize()
    ro, rl = O.sfa_forward(q.float(), k.float(), k[..., :128].float(), idx, 1)
    rdq, rdk, rdv, _ = O.sfa_backward(q.float(), k.float(), k[..., :128].float(), idx, o.detach().float().cpu(), rl,
                                      do.float(), 1)
    dkv = rdk.clone()
    dkv[..., :128] += rdv
    assert_close("o", o.detach().cpu(), ro)
    assert_close("dq", qd.grad.cpu(), rdq)
    assert_close("dkv", kd.grad.cpu(), dkv)


def test_token_level_backward_varlen():
    from sfa_check import check_all, run_op, run_oracle
    g = torch.Generator().manual_seed(17)
    q_lens, k_lens = [3, 100, 64], [30, 100, 250]
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, Hk, D, K = 16, 2, 128, 80
    q = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    k = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    v = torch.randn(int(cu_k[-1]), Hk, D, generator=g).bfloat16()
    do = torch.randn(int(cu_q[-1]), Hq, D, generator=g).bfloat16()
    idx = torch.randint(-1, 260, (int(cu_q[-1]), Hk, K), generator=g, dtype=torch.int32)
    got = run_op(q, k, v, idx, 1, None, None, True, do, cu_q, cu_k, max(q_lens), max(k_lens), kernel="tcgen05")
    ref = run_oracle(q, k, v, idx, 1, None, None, True, do, cu_q, cu_k, o_for_bwd=got["o"])
    check_all(got, ref)


def test_reference_signature_backward_on_tensor_cores():
    # SparseFlashAttention.apply end to end (forward and backward on the
    # token-level tensor-core kernels): dq, dkv = dK*scale + dV, dsink
    Sq, B, H, D, K = 200, 2, 32, 128, 150
    g = torch.Generator().manual_seed(23)
    q = torch.randn(Sq, B, H, D, generator=g).bfloat16()
    kv = torch.randn(Sq, B, D, generator=g).bfloat16()
    sink = torch.randn(H, generator=g)
    idx = torch.stack([torch.randperm(Sq, generator=g)[:K] for _ in range(Sq * B)]).view(Sq, B, K).to(torch.int32)
    idx[: Sq // 4, :, K // 2:] = -1
    do = torch.randn(Sq, B, H, D, generator=g).bfloat16()
    dev = torch.device("cuda")
    qg, kvg, sg = q.to(dev).requires_grad_(), kv.to(dev).requires_grad_(), sink.to(dev).requires_grad_()
    out = ops_b200.SparseFlashAttention.apply(qg, kvg, sg, idx.to(dev), D ** -0.5)
    out.backward(do.to(dev))
    torch.cuda.synchronize()
    ro, rl = O.reference_compat_forward(q.float(), kv.float(), sink, idx, D ** -0.5)
    rdq, rdkv, rds = O.reference_compat_backward(q.float(), kv.float(), sink, idx, D ** -0.5,
                                                 out.detach().float().cpu(), rl, do.float())
    assert_close("out", out.detach().cpu(), ro)
    assert_close("dq", qg.grad.cpu(), rdq)
    assert_close("dkv", kvg.grad.cpu(), rdkv)
    assert_close("dsink", sg.grad.cpu(), rds)


# ---------------------------------------------------------------------------
# backward for head dims above 256: the two-pass form (a stacked [S ; dP]
# pass writes P and dS' to a workspace, the gradient half reads them per
# 192-dim part of the head dims); v is k or k's leading dims
# ---------------------------------------------------------------------------
def _check_latent_bwd(q, k, idx, Dv, causal=True, sink=None, cu_q=None, cu_k=None, max_q=None, max_k=None):
    dev = torch.device("cuda")
    qd = q.to(dev).requires_grad_()
    kd = k.to(dev).requires_grad_()
    sd = None if sink is None else sink.to(dev).requires_grad_()
    vd = kd if Dv == k.shape[-1] else kd[..., :Dv]
    do = _do(q, k[..., :Dv])
    o, lse = ops_b200.sparse_flash_attention(
        qd, kd, vd, idx.to(dev), 1, attn_sink=sd, causal=causal, kernel="tcgen05",
        cu_seqlens=None if cu_q is None else cu_q.to(dev), cu_seqlens_k=None if cu_k is None else cu_k.to(dev),
        max_seqlen_q=max_q, max_seqlen_k=max_k)
    o.backward(do.to(dev))
    torch.cuda.synchronize()
    v = k[..., :Dv].float()
    ro, rl = O.sfa_forward(q.float(), k.float(), v, idx, 1, None, sink, causal, cu_q, cu_k)
    rdq, rdk, rdv, rds = O.sfa_backward(q.float(), k.float(), v, idx, o.detach().float().cpu(), rl, do.float(), 1,
                                        None, sink, causal, cu_q, cu_k)
    dkv = rdk.clone()
    dkv[..., :Dv] += rdv                               # one tensor: its gradient is dk + dv
    assert_close("o", o.detach().cpu(), ro)
    assert_lse(lse.detach().cpu(), rl)
    assert_close("dq", qd.grad.cpu(), rdq)
    assert_close("dkv", kd.grad.cpu(), dkv)
    if sink is not None:
        assert_close("dsink", sd.grad.cpu(), rds, maxabs=2e-2, rl2=5e-3)


def _two_pass_selected(q, k, Dv):
    # the backward plan takes the two-pass token-level form on tensor cores
    dev = torch.device("cuda")
    qd, kd = q[:1, :8].to(dev), k[:1, :8].to(dev)
    idx = torch.zeros(1, 8, k.shape[2], 1, dtype=torch.int32, device=dev)
    o = torch.empty(*qd.shape[:-1], Dv, dtype=qd.dtype, device=dev)
    lse = torch.empty(qd.shape[:-1], device=dev)
    cfg = S._Cfg(1, q.shape[-1] ** -0.5, True, False, 8, 8, 0, _lib.SFA_KERNEL_TCGEN05, True)
    P = S.build_params(qd, kd, kd[..., :Dv], idx, o, lse, cfg, None, None, None, torch.empty_like(o),
                       torch.empty_like(qd), torch.empty_like(kd), torch.empty_like(kd))
    return _lib.load().sfa_select_kernel(ctypes.byref(P), 1) == _lib.SFA_KERNEL_TCGEN05


@pytest.mark.parametrize("B,T,Hq,Hk,Dqk,Dv,K,causal", [
    (1, 300, 128, 1, 576, 512, 256, True),    # MLA: two 64-head groups, three 192-dim parts
    (2, 200, 64, 2, 320, 256, 130, True),     # 32 heads a group, parts of 3 + 2 slabs, partial chunk
    (1, 150, 16, 1, 384, 384, 64, False),     # v is k, 16 heads, non-causal
])
def test_two_pass_backward(B, T, Hq, Hk, Dqk, Dv, K, causal):
    q, k, _, idx = _inputs(B, T, Hq, Hk, Dqk, Dv, K, seed=Hq + Dqk + 3, causal=causal, edge=True)
    assert _two_pass_selected(q, k, Dv)
    sink = torch.randn(Hq, generator=torch.Generator().manual_seed(9))
    _check_latent_bwd(q, k, idx, Dv, causal, sink)


def test_two_pass_backward_in_waves(monkeypatch):
    # rows go through in waves of 37 (the last one ragged); results as in one wave
    monkeypatch.setenv("SFA_MLA_WAVE_ROWS", "37")
    q, k, _, idx = _inputs(1, 200, 128, 1, 576, 512, 192, seed=31, edge=True)
    _check_latent_bwd(q, k, idx, 512)


def test_two_pass_backward_varlen():
    g = torch.Generator().manual_seed(41)
    q_lens, k_lens = [3, 100, 64], [30, 100, 250]
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, Hk, Dqk, Dv, K = 64, 1, 576, 512, 80
    q = torch.randn(int(cu_q[-1]), Hq, Dqk, generator=g).bfloat16()
    k = torch.randn(int(cu_k[-1]), Hk, Dqk, generator=g).bfloat16()
    idx = torch.randint(-1, 260, (int(cu_q[-1]), Hk, K), generator=g, dtype=torch.int32)
    _check_latent_bwd(q, k, idx, Dv, True, None, cu_q, cu_k, max(q_lens), max(k_lens))


def test_two_pass_backward_separate_dk_dv_buffers():
    # v is k's leading dims but the caller keeps dk and dv apart (C ABI): the
    # two-pass form that drains dK^T and dV^T into their own accumulators
    B, T, Hq, Dqk, Dv, K = 1, 180, 64, 320, 256, 96
    q, k, _, idx = _inputs(B, T, Hq, 1, Dqk, Dv, K, seed=77, edge=True)
    dev = torch.device("cuda")
    qd, kd = q.to(dev), k.to(dev)
    vd = kd[..., :Dv]
    idd = idx.to(dev)
    o, lse = ops_b200.sparse_flash_attention(qd, kd, vd, idd, 1, kernel="tcgen05")
    do = _do(q, k[..., :Dv]).to(dev)
    dq, dk, dv = torch.empty_like(qd), torch.empty_like(kd), torch.empty(B, T, 1, Dv, dtype=kd.dtype, device=dev)
    cfg = S._Cfg(1, Dqk ** -0.5, True, False, T, T, 0, _lib.SFA_KERNEL_TCGEN05, False)
    P = S.build_params(qd, kd, vd, idd, o, lse, cfg, None, None, None, do, dq, dk, dv)
    lib = _lib.load()
    n = lib.sfa_bwd_workspace_bytes(ctypes.byref(P))
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
    _lib.check(lib.sfa_bwd(ctypes.byref(P), ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream), "sfa_bwd")
    torch.cuda.synchronize()
    ro, rl = O.sfa_forward(q.float(), k.float(), k[..., :Dv].float(), idx, 1)
    rdq, rdk, rdv, _ = O.sfa_backward(q.float(), k.float(), k[..., :Dv].float(), idx, o.float().cpu(), rl,
                                      do.float().cpu(), 1)
    assert_close("dq", dq.cpu(), rdq)
    assert_close("dk", dk.cpu(), rdk)
    assert_close("dv", dv.cpu(), rdv)
