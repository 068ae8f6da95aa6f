"""ctypes binding of libsfa_b200.so (the C ABI declared in include/sfa_b200.h).

The library is the product; this module only mirrors its struct and function
signatures.  Loading fails loudly when the library is missing — there is no
CPU or framework fallback for the SFA kernels.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libsfa_b200.so")

SFA_OK = 0
SFA_ERR_INVALID_ARGUMENT = -1
SFA_ERR_UNSUPPORTED = -2
SFA_ERR_WORKSPACE = -3
SFA_ERR_CUDA = -4
SFA_ERR_DEVICE_TIMEOUT = -5

SFA_DKV_AUTO, SFA_DKV_INVERTED, SFA_DKV_ATOMIC = 0, 1, 2
SFA_KERNEL_AUTO, SFA_KERNEL_TCGEN05, SFA_KERNEL_GENERAL = 0, 1, 2
SFA_DQ_AUTO, SFA_DQ_SEPARATE, SFA_DQ_FUSED = 0, 1, 2
SFA_COMPAT_REFERENCE_P = 1
SFA_KV_BF16, SFA_KV_FP8_E4M3 = 0, 1
SFA_SELFTEST_STATUS = (15 << 16) | 1   # status code of sfa_selftest_wait_timeout

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
ABI_VERSION = 3


class SfaParams(ctypes.Structure):
    """Field-for-field mirror of ``SfaParams`` in include/sfa_b200.h."""

    _fields_ = [
        ("q", _c_void_p), ("k", _c_void_p), ("v", _c_void_p), ("block_indices", _c_void_p),
        ("cu_seqlens_q", _c_void_p), ("cu_seqlens_k", _c_void_p), ("attn_sink", _c_void_p),
        ("o", _c_void_p), ("lse", _c_void_p), ("dout", _c_void_p), ("dq", _c_void_p),
        ("dk", _c_void_p), ("dv", _c_void_p), ("dsink", _c_void_p),
    ] + [(f"{t}_{s}", _i64) for t in ("q", "k", "v", "i", "o", "l", "do", "dq", "dk", "dv")
         for s in ("sb", "st", "sh")] + [
        ("batch", _i32), ("q_len", _i32), ("kv_len", _i32), ("total_q", _i32), ("total_kv", _i32),
        ("h_q", _i32), ("h_kv", _i32), ("d_qk", _i32), ("d_v", _i32), ("block_size", _i32),
        ("topk", _i32), ("scale", ctypes.c_float), ("causal", _i32), ("dkv_mode", _i32),
        ("kernel", _i32), ("dq_mode", _i32), ("compat", _i32), ("page_size", _i32),
        ("block_table", _c_void_p), ("bt_stride", _i64),
        ("kv_dtype", _i32), ("reserved", _i32), ("kv_scale", _c_void_p),
        ("ks_sb", _i64), ("ks_st", _i64), ("ks_sh", _i64),
    ]


class SfaIndexerParams(ctypes.Structure):
    """Field-for-field mirror of ``SfaIndexerParams`` in include/sfa_b200.h."""

    _fields_ = [
        ("q_idx", _c_void_p), ("k_idx", _c_void_p), ("weights", _c_void_p), ("out", _c_void_p),
        ("q_sb", _i64), ("q_st", _i64), ("q_sh", _i64), ("k_sb", _i64), ("k_st", _i64),
        ("w_sb", _i64), ("w_st", _i64), ("o_sb", _i64), ("o_st", _i64),
        ("batch", _i32), ("q_len", _i32), ("kv_len", _i32), ("heads", _i32), ("dim", _i32), ("topk", _i32),
        ("causal", _i32), ("reserved", _i32),
    ]


EXPORTS = {
    "sfa_abi_version": ([], _i32),
    "sfa_build_info": ([], ctypes.c_char_p),
    "sfa_last_error_string": ([], ctypes.c_char_p),
    "sfa_kernel_launches": ([], ctypes.c_ulonglong),
    "sfa_select_kernel": ([ctypes.POINTER(SfaParams), _i32], _i32),
    "sfa_bwd_plan": ([ctypes.POINTER(SfaParams), ctypes.POINTER(_i32), ctypes.POINTER(_i32)], _i32),
    "sfa_fwd_workspace_bytes": ([ctypes.POINTER(SfaParams)], ctypes.c_size_t),
    "sfa_bwd_workspace_bytes": ([ctypes.POINTER(SfaParams)], ctypes.c_size_t),
    "sfa_fwd": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_bwd": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_bwd_noalloc": ([ctypes.POINTER(SfaParams), _c_void_p], _i32),
    "sfa_bwd_preprocess": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_bwd_dq": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_bwd_dkdv": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_build_inverted_index": ([ctypes.POINTER(SfaParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
    "sfa_inverted_index_layout": ([ctypes.POINTER(SfaParams), ctypes.POINTER(ctypes.c_size_t),
                                   ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(_i32),
                                   ctypes.POINTER(_i32)], _i32),
    "sfa_device_status": ([_c_void_p, ctypes.POINTER(_i32)], _i32),
    "sfa_selftest_wait_timeout": ([_c_void_p, ctypes.c_uint32], _i32),
    "sfa_reset_device_status": ([_c_void_p], _i32),
    "sfa_launch_trace": ([ctypes.POINTER(_c_void_p), _i32], _i32),
    "sfa_launch_trace_count": ([], _i32),
    "sfa_launch_trace_name": ([_i32], ctypes.c_char_p),
    "sfa_indexer_workspace_bytes": ([ctypes.POINTER(SfaIndexerParams)], ctypes.c_size_t),
    "sfa_indexer_topk": ([ctypes.POINTER(SfaIndexerParams), _c_void_p, ctypes.c_size_t, _c_void_p], _i32),
}

_lib = None


class SfaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"SFA error {code}: {msg}")
        self.code = code


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m ops_b200.build` "
                          "(the SFA op has no fallback implementation)")
    lib = ctypes.CDLL(path)
    for name, (args, res) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if lib.sfa_abi_version() != ABI_VERSION:
        raise ImportError("libsfa_b200.so ABI version mismatch")
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != SFA_OK:
        msg = load().sfa_last_error_string().decode(errors="replace")
        if rc == SFA_ERR_INVALID_ARGUMENT:
            raise ValueError(f"{what}: {msg}")
        raise SfaError(rc, f"{what}: {msg}")
