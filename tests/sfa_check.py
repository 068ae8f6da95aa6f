"""Helpers shared by the GPU parity tests: run the CUDA op and the CPU oracle on
the same seeded inputs and compare with the tolerances the op promises.

Tolerances (bf16 outputs against the fp32 oracle): o, dq, dk, dv max-abs 2e-2
and rel-L2 5e-3; lse max-abs 1e-3.  Max-abs is taken on errors normalised by
max(1, RMS of the oracle's row): a dk/dv row sums the contributions of every
query that selected the key, and the bf16 rounding of the MMA operands P and
dS (the reference rounds them the same way, SFA.py:700, 807-808) leaves an
error proportional to that row's magnitude — up to 2^-9 of it — on every
element of the row, including elements whose own value is small.  Measured on
the CPU: bf16 P alone gives 1.6e-2 element-normalised max-abs on a T=4096
dv.  For o and dq rows (RMS below 1) the bound is the plain absolute 2e-2."""
import math

import torch

from oracle import sfa_oracle as O

TOL_MAXABS = 2e-2
TOL_REL_L2 = 5e-3
TOL_LSE = 1e-3


def rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / max(float(b.norm()), 1e-30))


def max_abs_norm(a, b):
    a, b = a.double(), b.double()
    if not a.numel():
        return 0.0
    scale = b.pow(2).mean(-1, keepdim=True).sqrt().clamp_min(1.0) if b.dim() else b.abs().clamp_min(1.0)
    return float(((a - b).abs() / scale).max())


def assert_close(name, got, ref, maxabs=TOL_MAXABS, rl2=TOL_REL_L2):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{name}: non-finite values"
    m = max_abs_norm(got, ref)
    r = rel_l2(got, ref) if ref.norm() > 0 else float(got.norm())
    assert m <= maxabs and r <= rl2, f"{name}: max-abs(norm) {m:.3e} (tol {maxabs}), rel-L2 {r:.3e} (tol {rl2})"


def assert_lse(got, ref):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got), fin), "lse: -inf pattern differs"
    assert torch.equal(got[~fin], ref[~fin]), "lse: non-finite values differ"
    if fin.any():
        d = float((got[fin] - ref[fin]).abs().max())
        assert d <= TOL_LSE, f"lse max-abs {d:.3e}"


def run_op(q, k, v, idx, bs, scale=None, sink=None, causal=True, do=None, cu_q=None, cu_k=None,
           max_q=None, max_k=None, dkv_mode="auto", kernel="auto", shared_kv=False, dq_mode="auto"):
    """CUDA op forward (+ backward if do is given).  Returns dict of CPU tensors."""
    import ops_b200
    dev = torch.device("cuda")
    qg = q.to(dev).requires_grad_(do is not None)
    if shared_kv:
        kg = k.to(dev).requires_grad_(do is not None)
        vg = kg
    else:
        kg = k.to(dev).requires_grad_(do is not None)
        vg = v.to(dev).requires_grad_(do is not None)
    sg = None if sink is None else sink.to(dev).float().requires_grad_(do is not None)
    o, lse = ops_b200.sparse_flash_attention(
        qg, kg, vg, idx.to(dev), bs, scale, cu_seqlens=None if cu_q is None else cu_q.to(dev), attn_sink=sg,
        causal=causal, cu_seqlens_k=None if cu_k is None else cu_k.to(dev), max_seqlen_q=max_q,
        max_seqlen_k=max_k, dkv_mode=dkv_mode, kernel=kernel, dq_mode=dq_mode)
    out = dict(o=o.detach().cpu(), lse=lse.detach().cpu())
    if do is not None:
        o.backward(do.to(dev))
        out["dq"] = qg.grad.cpu()
        out["dk"] = kg.grad.cpu()
        out["dv"] = None if shared_kv else vg.grad.cpu()
        out["dsink"] = None if sg is None else sg.grad.cpu()
    torch.cuda.synchronize()
    return out


def run_oracle(q, k, v, idx, bs, scale=None, sink=None, causal=True, do=None, cu_q=None, cu_k=None,
               o_for_bwd=None):
    qf, kf, vf = q.float(), k.float(), v.float()
    o, lse = O.sfa_forward(qf, kf, vf, idx, bs, scale, sink, causal, cu_q, cu_k)
    out = dict(o=o, lse=lse)
    if do is not None:
        # delta uses the op's own bf16 o, as the reference does (SFA.py:590-610)
        o_in = o_for_bwd.float() if o_for_bwd is not None else o
        dq, dk, dv, ds = O.sfa_backward(qf, kf, vf, idx, o_in, lse, do.float(), bs, scale, sink, causal, cu_q, cu_k)
        out.update(dq=dq, dk=dk, dv=dv, dsink=ds)
    return out


def check_all(got, ref, shared_kv=False, grads=True):
    assert_close("o", got["o"], ref["o"])
    assert_lse(got["lse"], ref["lse"])
    if not grads:
        return
    assert_close("dq", got["dq"], ref["dq"])
    if shared_kv:
        assert_close("dkv", got["dk"], ref["dk"] + ref["dv"])
    else:
        assert_close("dk", got["dk"], ref["dk"])
        assert_close("dv", got["dv"], ref["dv"])
    if ref.get("dsink") is not None and got.get("dsink") is not None:
        assert_close("dsink", got["dsink"], ref["dsink"], maxabs=2e-2, rl2=5e-3)
