"""Tiling / launch-configuration layer.

The reference picks Ascend tile sizes from the max valid top-k count
(``TilingBlockConfig``, ``CONFIG_MAP``, ``_resolve_tiling_config``,
``_effective_topk`` — ``SFA.py:16-66``); computing that count costs a
device->host sync on every call and every new value recompiles the kernels
(``TOPK`` is a constexpr, ``SFA.py:514-519``).

On sm_100a the launch table lives in the C library (``sfa_select_kernel``) and
is keyed on static shape only — (D_qk, D_v, group size, block_size, alignment)
— so it needs no sync.  ``select_kernel`` asks it which family a call runs;
the tile constants live with each kernel.  The reference-compatible helpers
below keep the reference's bucket semantics and errors for callers that use
them directly.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib


@dataclass(frozen=True)
class TilingBlockConfig:
    """Same fields as the reference's config (``SFA.py:16-23``)."""
    BLOCK_N: int
    BLOCK_H: int
    BLOCK_Q_BWD: int
    BLOCK_K_BWD: int
    BLOCK_H_BWD: int
    extra_args: dict = field(default_factory=dict)


# The reference's buckets (SFA.py:35-48); the Ascend compiler knobs
# (SFA.py:26-32) have no sm_100a meaning and are dropped.
CONFIG_MAP = {
    128: TilingBlockConfig(64, 32, 64, 64, 32),
    160: TilingBlockConfig(80, 32, 80, 40, 32),
    640: TilingBlockConfig(80, 32, 80, 64, 32),
}


def resolve_tiling_config(topk: int) -> TilingBlockConfig:
    """Bucket choice of ``_resolve_tiling_config`` (``SFA.py:51-59``)."""
    if topk <= 0:
        raise ValueError(f"Unsupported topk value: {topk}. Please make sure it is a positive integer.")
    if topk <= 128:
        return CONFIG_MAP[128]
    if topk <= 160:
        return CONFIG_MAP[160]
    return CONFIG_MAP[640]


def effective_topk(topk_idxs: torch.Tensor) -> int:
    """Max count of ``idx >= 0`` per row (``SFA.py:62-66``).  Synchronises the
    host with the device; the B200 kernels never call it."""
    if topk_idxs.numel() == 0:
        raise ValueError("topk_idxs tensor is empty. Cannot determine effective topk.")
    return int((topk_idxs >= 0).sum(dim=-1).max().item())


FAMILY_NAMES = {_lib.SFA_KERNEL_TCGEN05: "tcgen05", _lib.SFA_KERNEL_GENERAL: "general"}


def select_kernel(params: "_lib.SfaParams", backward: bool = False) -> str:
    """Ask the C launch table which family a call with ``params`` would run."""
    lib = _lib.load()
    rc = lib.sfa_select_kernel(ctypes.byref(params), 1 if backward else 0)
    _lib.check(rc if rc < 0 else 0, "sfa_select_kernel")
    return FAMILY_NAMES[rc]
