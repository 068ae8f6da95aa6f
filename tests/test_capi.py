"""The C-ABI library: loads without a GPU, exports every declared symbol, and
its parameter struct matches the header byte for byte (checked with gcc)."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from ops_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sfa_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(sfa_[a-z0-9_]+)\s*\(", src, re.M)))


def test_library_loads_and_exports_all_declared_symbols():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.EXPORTS, f"{n} has no ctypes signature"
    assert lib.sfa_abi_version() == _lib.ABI_VERSION == 3
    assert b"sm_100a" in lib.sfa_build_info()


@pytest.mark.parametrize("struct", ["SfaParams", "SfaIndexerParams"])
def test_struct_layout_matches_header(struct):
    cls = getattr(_lib, struct)
    fields = [f[0] for f in cls._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
            f'printf("%zu\\n", sizeof({struct}));']
    for f in fields:
        prog.append(f'printf("%zu\\n", offsetof({struct}, {f}));')
    prog.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        open(c, "w").write("\n".join(prog))
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", c, "-o", exe], check=True)
        out = [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert out[0] == ctypes.sizeof(cls)
    for f, off in zip(fields, out[1:]):
        assert getattr(cls, f).offset == off, f


def _params(**kw):
    P = _lib.SfaParams()
    fake = 0x10000
    for n in ("q", "k", "v", "block_indices", "o", "lse"):
        setattr(P, n, fake)
    P.batch, P.q_len, P.kv_len, P.h_q, P.h_kv, P.d_qk, P.d_v = 1, 64, 64, 16, 1, 64, 64
    P.block_size, P.topk, P.scale, P.causal = 64, 1, 0.125, 1
    for k, v in kw.items():
        setattr(P, k, v)
    return P


@pytest.mark.parametrize("field,value,msg", [
    ("h_kv", 3, "multiple"), ("topk", 0, "topk"), ("block_size", 0, "block_size"), ("q", None, "non-NULL"),
    ("d_v", 0, "positive"), ("kernel", 7, "kernel"),
])
def test_argument_validation_without_gpu(field, value, msg):
    lib = _lib.load()
    P = _params(**{field: value})
    rc = lib.sfa_select_kernel(ctypes.byref(P), 0)
    assert rc == _lib.SFA_ERR_INVALID_ARGUMENT
    assert msg in lib.sfa_last_error_string().decode()


def test_backward_requires_gradient_buffers():
    lib = _lib.load()
    P = _params()
    assert lib.sfa_select_kernel(ctypes.byref(P), 1) == _lib.SFA_ERR_INVALID_ARGUMENT
    assert lib.sfa_bwd_workspace_bytes(ctypes.byref(P)) == 0


def test_oversized_head_dims_are_unsupported_by_general_family():
    lib = _lib.load()
    P = _params(d_qk=8192, d_v=8192, kernel=_lib.SFA_KERNEL_GENERAL)
    assert lib.sfa_select_kernel(ctypes.byref(P), 0) == _lib.SFA_ERR_UNSUPPORTED


def test_backward_plan_is_consistent_with_the_launch_table():
    # without a GPU the tensor-core family is unavailable: the general family
    # always takes the atomic dK/dV pass with dQ in the same (separate) pass
    lib = _lib.load()
    fake = 0x20000
    P = _params(dout=fake, dq=fake, dk=fake, dv=fake + 0x1000)
    dkv, dq = ctypes.c_int32(-9), ctypes.c_int32(-9)
    fam = lib.sfa_bwd_plan(ctypes.byref(P), ctypes.byref(dkv), ctypes.byref(dq))
    assert fam == lib.sfa_select_kernel(ctypes.byref(P), 1)
    if fam == _lib.SFA_KERNEL_GENERAL:
        assert (dkv.value, dq.value) == (_lib.SFA_DKV_ATOMIC, _lib.SFA_DQ_SEPARATE)
    else:
        assert dkv.value in (_lib.SFA_DKV_INVERTED, _lib.SFA_DKV_ATOMIC)
        assert dq.value in (_lib.SFA_DQ_SEPARATE, _lib.SFA_DQ_FUSED)
    P.dq_mode = 5
    assert lib.sfa_bwd_plan(ctypes.byref(P), ctypes.byref(dkv), ctypes.byref(dq)) == _lib.SFA_ERR_INVALID_ARGUMENT
    assert "dq_mode" in lib.sfa_last_error_string().decode()


def test_paged_cache_rules_without_gpu():
    # a paged kv cache is a varlen forward format: the backward is refused, the
    # page size must hold whole blocks and the table must cover kv_len
    lib = _lib.load()
    fake = 0x30000
    paged = dict(block_table=fake, bt_stride=4, page_size=64, cu_seqlens_q=fake, cu_seqlens_k=fake,
                 total_q=1, total_kv=256, kv_len=200)
    P = _params(**paged)
    assert lib.sfa_select_kernel(ctypes.byref(P), 0) >= 0
    Pb = _params(dout=fake, dq=fake, dk=fake, dv=fake + 0x1000, **paged)
    assert lib.sfa_select_kernel(ctypes.byref(Pb), 1) == _lib.SFA_ERR_UNSUPPORTED
    assert "backward" in lib.sfa_last_error_string().decode()
    for bad, msg in ((dict(page_size=96), "page_size"), (dict(bt_stride=3), "bt_stride"),
                     (dict(cu_seqlens_q=None, cu_seqlens_k=None), "varlen")):
        P = _params(**{**paged, **bad})
        assert lib.sfa_select_kernel(ctypes.byref(P), 0) == _lib.SFA_ERR_INVALID_ARGUMENT
        assert msg in lib.sfa_last_error_string().decode()


def test_indexer_argument_validation_without_gpu():
    lib = _lib.load()
    fake = 0x40000
    base = dict(q_idx=fake, k_idx=fake, weights=fake, out=fake, q_sb=64 * 64 * 128, q_st=64 * 128, q_sh=128,
                k_sb=64 * 128, k_st=128, w_sb=64 * 64, w_st=64, o_sb=64 * 8, o_st=8,
                batch=1, q_len=64, kv_len=64, heads=64, dim=128, topk=8, causal=1)
    P = _lib.SfaIndexerParams(**base)
    assert lib.sfa_indexer_workspace_bytes(ctypes.byref(P)) == 64 * 128 * 4
    for bad, code, msg in ((dict(heads=48), _lib.SFA_ERR_UNSUPPORTED, "heads"),
                           (dict(dim=96), _lib.SFA_ERR_UNSUPPORTED, "dim"),
                           (dict(topk=0), _lib.SFA_ERR_INVALID_ARGUMENT, "topk"),
                           (dict(kv_len=60000), _lib.SFA_ERR_UNSUPPORTED, "kv_len"),
                           (dict(q_idx=0), _lib.SFA_ERR_INVALID_ARGUMENT, "non-NULL")):
        P = _lib.SfaIndexerParams(**{**base, **bad})
        assert lib.sfa_indexer_topk(ctypes.byref(P), None, 0, None) == code
        assert msg in lib.sfa_last_error_string().decode()


def test_fp8_kv_rules_without_gpu():
    lib = _lib.load()
    fake = 0x50000
    P = _params(kv_dtype=_lib.SFA_KV_FP8_E4M3, kv_scale=fake, block_size=1, topk=8)
    assert lib.sfa_select_kernel(ctypes.byref(P), 0) >= 0
    Pb = _params(kv_dtype=_lib.SFA_KV_FP8_E4M3, kv_scale=fake, dout=fake, dq=fake, dk=fake, dv=fake + 0x1000)
    assert lib.sfa_select_kernel(ctypes.byref(Pb), 1) == _lib.SFA_ERR_UNSUPPORTED
    for bad, msg in ((dict(kv_scale=None), "kv_scale"), (dict(v=fake + 0x100), "latent"), (dict(kv_dtype=5), "kv_dtype")):
        P = _params(**{**dict(kv_dtype=_lib.SFA_KV_FP8_E4M3, kv_scale=fake), **bad})
        assert lib.sfa_select_kernel(ctypes.byref(P), 0) == _lib.SFA_ERR_INVALID_ARGUMENT
        assert msg in lib.sfa_last_error_string().decode()
