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
