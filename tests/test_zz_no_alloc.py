"""sfa_bwd_noalloc: the backward without a caller-provided workspace.

Some callers cannot allocate device memory at all — a host that runs from a
pre-sized arena, a serving loop with a fixed budget, a plugin whose host owns
every device allocation.  For them the library keeps the backward's scratch in
a static device array (32 MiB, reserved on every GPU that loads the library).
These tests call the entry point through the C ABI, twice in a row (the array
keeps the previous call's contents), and compare against sfa_bwd with a
regular workspace.  This file is collected last so a failure here cannot hide
the other tests when pytest stops at the first failure.
"""
import ctypes

import pytest
import torch

from ops_b200 import _lib, sfa as S, workloads as W
from sfa_check import assert_close

pytestmark = pytest.mark.gpu


def _problem(cfg, bs, kernel, seed):
    dev = torch.device("cuda")
    d = W.make_inputs(cfg, "cpu", seed)
    q, k, v, idx, do = (d[n].to(dev) for n in ("q", "k", "v", "idx", "do"))
    sink = torch.randn(cfg.Hq, generator=torch.Generator().manual_seed(seed)).to(dev)
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=dev)
    c = S._Cfg(bs, cfg.scale, True, False, cfg.T, cfg.T, _lib.SFA_DKV_AUTO, kernel, False)
    grads = dict(dq=torch.empty_like(q), dk=torch.empty_like(k), dv=torch.empty_like(v),
                 dsink=torch.empty(cfg.Hq, dtype=torch.float32, device=dev))
    P = S.build_params(q, k, v, idx, o, lse, c, sink, None, None, do, grads["dq"], grads["dk"], grads["dv"],
                       grads["dsink"])
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, st), "sfa_fwd")
    # the struct holds raw pointers: keep every tensor it points at alive
    keep = (q, k, v, idx, do, sink, o, lse)
    return P, grads, keep


def _snapshot(grads):
    return {n: t.clone() for n, t in grads.items()}


@pytest.mark.parametrize("kernel,cfg,bs,fused_fits", [
    (_lib.SFA_KERNEL_TCGEN05, W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hq=32, Hk=2, S=16), 64, False),
    (_lib.SFA_KERNEL_TCGEN05, W.scaled(W.CONFIGS["c2"], B=1, T=1024, Hq=16, Hk=1, S=8), 64, True),
    (_lib.SFA_KERNEL_GENERAL, W.scaled(W.CONFIGS["c1"], T=512), 64, False),
], ids=["tcgen05_separate_dq", "tcgen05_fused_dq", "general_atomic"])
def test_noalloc_backward_matches_workspace_backward(kernel, cfg, bs, fused_fits):
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    P, grads, _keep = _problem(cfg, bs, kernel, seed=21)
    nbytes = lib.sfa_bwd_workspace_bytes(ctypes.byref(P))
    if kernel == _lib.SFA_KERNEL_TCGEN05:
        # the first case needs the separate dQ pass to fit the static array;
        # the second keeps the fused dQ (its accumulator fits as well)
        dkv, dq = ctypes.c_int32(), ctypes.c_int32()
        lib.sfa_bwd_plan(ctypes.byref(P), ctypes.byref(dkv), ctypes.byref(dq))
        assert dq.value == _lib.SFA_DQ_FUSED
        assert (nbytes <= (32 << 20)) == fused_fits
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.sfa_bwd(ctypes.byref(P), ws.data_ptr(), nbytes, st), "sfa_bwd")
    ref = _snapshot(grads)
    for call in range(2):
        for t in grads.values():
            t.fill_(float("nan"))
        _lib.check(lib.sfa_bwd_noalloc(ctypes.byref(P), st), f"sfa_bwd_noalloc call {call}")
        torch.cuda.synchronize()
        for n in grads:
            assert_close(f"{n} (call {call})", grads[n], ref[n])


def test_noalloc_rejects_problems_beyond_its_scratch():
    lib = _lib.load()
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=2048, Hq=32, Hk=2, S=16)
    P, _, _keep = _problem(cfg, 64, _lib.SFA_KERNEL_TCGEN05, seed=3)
    # pretend the batch is large enough that its scratch exceeds 32 MiB; the call
    # must refuse before launching anything
    big = _lib.SfaParams.from_buffer_copy(P)
    big.batch = 64
    big.q_len = 16384
    big.kv_len = 16384
    need = lib.sfa_bwd_workspace_bytes(ctypes.byref(big))
    assert need > (32 << 20)
    n0 = lib.sfa_kernel_launches()
    rc = lib.sfa_bwd_noalloc(ctypes.byref(big), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SFA_ERR_WORKSPACE
    assert b"static" in lib.sfa_last_error_string()
    assert lib.sfa_kernel_launches() == n0
