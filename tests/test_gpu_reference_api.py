"""The reference-compatible surface on the GPU against the reference's own
outputs (golden fixtures from SFA.py) and against the oracle."""
import os

import numpy as np
import pytest
import torch

from oracle import sfa_oracle as O
from sfa_check import TOL_LSE, assert_close, max_abs_norm, rel_l2

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: (torch.from_numpy(d[k]) if d[k].ndim else d[k].item()) for k in d.files}


@pytest.mark.parametrize("name", ["tok_bucket128", "tok_bucket160", "tok_bucket640", "empty_row"])
def test_reference_signature_against_golden(name):
    import ops_b200
    d = load(name)
    dev = torch.device("cuda")
    q = d["q"].bfloat16().to(dev).requires_grad_()
    kv = d["kv"].bfloat16().to(dev).requires_grad_()
    sink = d["sink"].to(dev).requires_grad_()
    idx = d["idx"].to(dev)
    out = ops_b200.SparseFlashAttention.apply(q, kv, sink, idx, d["scale"])
    out.backward(d["do"].bfloat16().to(dev))
    out, dq, dkv, dsink = (t.detach().float().cpu() for t in (out, q.grad, kv.grad, sink.grad))
    # against the reference's own outputs: within the reference's bf16 rounding
    assert max_abs_norm(out, d["out"]) < 2e-2 and rel_l2(out, d["out"]) < 1e-2
    assert rel_l2(dq, d["dq"]) < 1.5e-2 and rel_l2(dkv, d["dkv"]) < 1.5e-2
    # dsink sums -p_sink*delta over every row; delta comes from each side's own bf16 o
    assert max_abs_norm(dsink, d["dsink"]) < 2e-2
    # against the oracle: the op's own tolerance
    o_ref, lse_ref = O.reference_compat_forward(d["q"], d["kv"], d["sink"], d["idx"], d["scale"])
    assert_close("o", out, o_ref)
    dq_r, dkv_r, ds_r = O.reference_compat_backward(d["q"], d["kv"], d["sink"], d["idx"], d["scale"], out, lse_ref,
                                                    d["do"])
    assert_close("dq", dq, dq_r)
    assert_close("dkv", dkv, dkv_r)
    assert_close("dsink", dsink, ds_r)


def test_int64_indices_and_errors():
    import ops_b200
    d = load("tok_bucket128")
    dev = torch.device("cuda")
    q = d["q"].bfloat16().to(dev)
    kv = d["kv"].bfloat16().to(dev)
    sink = d["sink"].to(dev)
    a = ops_b200.SparseFlashAttention.apply(q, kv, sink, d["idx"].to(dev), d["scale"])
    b = ops_b200.SparseFlashAttention.apply(q, kv, sink, d["idx"].long().to(dev), d["scale"])
    assert torch.equal(a, b)
    with pytest.raises(ValueError, match="empty"):
        ops_b200.SparseFlashAttention.apply(q, kv, sink, torch.empty(q.shape[0], q.shape[1], 0, dtype=torch.int32,
                                                                     device=dev), d["scale"])
    with pytest.raises(ValueError, match="bfloat16"):
        ops_b200.SparseFlashAttention.apply(q.float(), kv, sink, d["idx"].to(dev), d["scale"])


@pytest.mark.parametrize("name", ["tok_bucket128", "tok_bucket160", "tok_bucket640", "empty_row"])
def test_reference_quirks_mode_against_golden(name):
    # with the reference's own rounding of p (fp16, then bf16) the op's output
    # stays within the reference's tolerance of its saved output (the extra
    # rounding moves o by less than o's own bf16 rounding, so it neither helps
    # nor hurts measurably), and the returned lse is the reference's base-2 lse
    # (+inf on a row with no valid key, as its -1e11 max seed makes it)
    import ops_b200
    d = load(name)
    dev = torch.device("cuda")
    q, kv, sink, idx = d["q"].bfloat16().to(dev), d["kv"].bfloat16().to(dev), d["sink"].to(dev), d["idx"].to(dev)
    plain = ops_b200.SparseFlashAttention.apply(q, kv, sink, idx, d["scale"]).float().cpu()
    quirk = ops_b200.SparseFlashAttentionCompat.apply(q, kv, sink, idx, d["scale"]).float().cpu()
    e_plain, e_quirk = rel_l2(plain, d["out"]), rel_l2(quirk, d["out"])
    assert e_quirk < 1e-2 and max_abs_norm(quirk, d["out"]) < 2e-2, (e_quirk, e_plain)
    assert abs(e_quirk - e_plain) < 1e-3 and max_abs_norm(quirk, plain) < 2e-2
    # the general surface with reference_quirks: base-2 lse with the reference's +inf
    o, lse2 = ops_b200.sparse_flash_attention(q.permute(1, 0, 2, 3), kv.permute(1, 0, 2).unsqueeze(2),
                                              kv.permute(1, 0, 2).unsqueeze(2), idx.permute(1, 0, 2).unsqueeze(2),
                                              1, d["scale"], attn_sink=sink, causal=False, reference_quirks=True)
    lse2 = lse2.permute(1, 0, 2).cpu()
    ref = d["lse2"]
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(lse2), fin) and torch.equal(lse2[~fin], ref[~fin])
    if fin.any():
        assert float((lse2[fin] - ref[fin]).abs().max()) < 1e-5
    assert torch.equal(o.permute(1, 0, 2, 3).float().cpu(), quirk)
