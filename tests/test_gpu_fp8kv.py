"""GPU: the forward over an e4m3 latent kv cache with power-of-two row
scales.  Dequantisation to bf16 is exact for such scales, so the fp8 path
must give bitwise the outputs of the bf16 path over the dequantised cache
(the same kernels, the same bf16 slabs; only where the bytes come from
differs), and both match the oracle on the dequantised cache."""
import pytest
import torch

import ops_b200
from oracle import sfa_oracle as O
from sfa_check import assert_close, assert_lse

pytestmark = pytest.mark.gpu


def _case(B, T, Hq, Dqk, Dv, K, seed, causal=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hq, Dqk, generator=g).bfloat16()
    # rows of different magnitude (different e4m3 scales), scores of the usual size
    kv = (torch.randn(B, T, 1, Dqk, generator=g) * (0.5 + torch.rand(B, T, 1, 1, generator=g))).bfloat16()
    if causal:
        u = torch.rand(B, T, 1, T, generator=g)
        t = torch.arange(T)
        u = torch.where(t[None, None, None, :] <= t[None, :, None, None], u, torch.full_like(u, 2.0))
        val, idx = torch.topk(u, min(K, T), dim=-1, largest=False)
        idx = torch.where(val < 2.0, idx, torch.full_like(idx, -1)).to(torch.int32)
    else:
        idx = torch.stack([torch.randperm(T, generator=g)[:K] for _ in range(B * T)]).view(B, T, 1, K).int()
    idx[:, 1] = -1                                            # a row with nothing selected
    return q, kv, idx


@pytest.mark.parametrize("B,T,Hq,Dqk,Dv,K,causal,kernel", [
    (1, 300, 128, 576, 512, 256, True, "auto"),     # MLA: tensor-core token forward, two V parts
    (2, 200, 16, 128, 128, 100, True, "auto"),      # v is the whole kv row
    (1, 150, 64, 256, 128, 64, False, "auto"),
    (1, 120, 16, 128, 128, 48, True, "general"),    # CUDA-core family
])
def test_fp8_kv_equals_bf16_over_the_dequantised_cache(B, T, Hq, Dqk, Dv, K, causal, kernel):
    q, kv, idx = _case(B, T, Hq, Dqk, Dv, K, seed=Hq + Dqk, causal=causal)
    kv8, sc = ops_b200.quantize_kv_fp8(kv)
    deq = (kv8.float() * sc[..., None]).bfloat16()
    sink = torch.randn(Hq, generator=torch.Generator().manual_seed(4))
    dev = torch.device("cuda")
    qd, dd = q.to(dev), deq.to(dev)
    o1, l1 = ops_b200.sparse_flash_attention(qd, dd, dd[..., :Dv], idx.to(dev), 1, attn_sink=sink.to(dev),
                                             causal=causal, kernel=kernel)
    o2, l2 = ops_b200.sparse_flash_attention_fp8kv(qd, kv8.to(dev), sc.to(dev), idx.to(dev), Dv,
                                                   attn_sink=sink.to(dev), causal=causal, kernel=kernel)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    ro, rl = O.sfa_forward(q.float(), deq.float(), deq[..., :Dv].float(), idx, 1, None, sink, causal)
    assert_close("o", o2.cpu(), ro)
    assert_lse(l2.cpu(), rl)


def test_fp8_kv_varlen():
    g = torch.Generator().manual_seed(8)
    q_lens, k_lens = [1, 1, 1, 1], [300, 64, 1000, 513]              # decode: one query per sequence
    cu_q = torch.tensor([0, 1, 2, 3, 4], dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0)), dtype=torch.int32)
    Hq, D, Dv, K = 64, 576, 512, 128
    q = torch.randn(4, Hq, D, generator=g).bfloat16()
    kv = torch.randn(int(cu_k[-1]), 1, D, generator=g).bfloat16()
    idx = torch.stack([torch.stack([torch.randperm(l, generator=g)[:K]]) if l >= K else
                       torch.stack([torch.cat([torch.randperm(l, generator=g), torch.full((K - l,), -1)])])
                       for l in k_lens]).int()
    kv8, sc = ops_b200.quantize_kv_fp8(kv)
    deq = (kv8.float() * sc[..., None]).bfloat16()
    dev = torch.device("cuda")
    o, lse = ops_b200.sparse_flash_attention_fp8kv(q.to(dev), kv8.to(dev), sc.to(dev), idx.to(dev), Dv,
                                                   cu_seqlens=cu_q.to(dev), cu_seqlens_k=cu_k.to(dev),
                                                   max_seqlen_q=1, max_seqlen_k=max(k_lens))
    torch.cuda.synchronize()
    ro, rl = O.sfa_forward(q.float(), deq.float(), deq[..., :Dv].float(), idx, 1, None, None, True, cu_q, cu_k)
    assert_close("o", o.cpu(), ro)
    assert_lse(lse.cpu(), rl)
