"""The kernels' bounded waits, exercised on a GPU without a fault: a wait that
nothing satisfies runs out after its limit, its code lands in the device status
word, the kernel returns, and the context keeps running the op correctly."""
import ctypes
import time

import pytest
import torch

from ops_b200 import _lib
from ops_b200 import workloads as W
from sfa_check import check_all, run_op, run_oracle

pytestmark = pytest.mark.gpu


def _status(lib, st):
    s = ctypes.c_int32(-1)
    _lib.check(lib.sfa_device_status(st, ctypes.byref(s)), "sfa_device_status")
    return s.value


def test_expired_wait_reports_its_status_and_the_context_stays_usable():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sfa_reset_device_status(st), "reset")
    assert _status(lib, st) == 0
    t0 = time.perf_counter()
    _lib.check(lib.sfa_selftest_wait_timeout(st, 20000), "selftest")   # a 20 ms limit
    assert _status(lib, st) == _lib.SFA_SELFTEST_STATUS
    assert time.perf_counter() - t0 >= 0.015                           # it waited out its limit
    _lib.check(lib.sfa_reset_device_status(st), "reset")
    assert _status(lib, st) == 0
    # the same context runs the op afterwards, with results as before
    cfg = W.scaled(W.CONFIGS["c2"], B=1, T=512, Hq=16, Hk=1, S=4)
    d = W.make_inputs(cfg, "cpu", 3)
    got = run_op(d["q"], d["k"], d["v"], d["idx"], 64, None, None, True, d["do"], kernel="tcgen05")
    ref = run_oracle(d["q"], d["k"], d["v"], d["idx"], 64, None, None, True, d["do"], o_for_bwd=got["o"])
    check_all(got, ref)
    assert _status(lib, st) == 0


def test_selftest_rejects_out_of_range_limits():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.sfa_selftest_wait_timeout(st, 0) == _lib.SFA_ERR_INVALID_ARGUMENT
    assert lib.sfa_selftest_wait_timeout(st, 2000000) == _lib.SFA_ERR_INVALID_ARGUMENT
