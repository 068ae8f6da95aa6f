"""Host-side mirror of the reference's SFA operator interface.

Two surfaces, both calling libsfa_b200.so through its C ABI on the current
CUDA stream:

* ``SparseFlashAttention.apply(q, kv, attn_sink, topk_idxs, sm_scale)`` — the
  reference's ``SparseFlashAttentionTriton`` signature (lilac-me/ops
  ``SFA.py:69-306``): SBHD layout, one shared kv head whose rows are both keys and
  values, token-level ``topk_idxs``, returns ``out``; backward returns
  ``(dq, dkv, dsink, None, None)`` (``SFA.py:300-306``).
* ``sparse_flash_attention(q, k, v, block_indices, ...) -> (o, lse)`` — the
  generalised surface: grouped-query heads, separate k/v (D_v may differ from
  D_qk), block_size keys per selected id, causal masking, optional attention sink
  and varlen batches through ``cu_seqlens``.

Errors follow the reference where it has them (``ValueError`` for an empty
index tensor or a non-positive topk, ``SFA.py:53``, ``SFA.py:64``); everything
else the C ABI rejects surfaces as ``ValueError`` (bad arguments) or
``ops_b200.SfaError``.  Unlike the reference, neither direction synchronises the
host with the device (no ``_effective_topk``, ``SFA.py:62-66``), and indices may
be padded with -1 in any slot.  The one exception: a varlen call that leaves
``max_seqlen_q`` / ``max_seqlen_k`` unset reads them from ``cu_seqlens`` on the
host (one device->host copy each); pass them to keep the call sync-free.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import SfaParams

_DKV = {"auto": _lib.SFA_DKV_AUTO, "inverted": _lib.SFA_DKV_INVERTED, "atomic": _lib.SFA_DKV_ATOMIC}
_KERNEL = {"auto": _lib.SFA_KERNEL_AUTO, "tcgen05": _lib.SFA_KERNEL_TCGEN05, "general": _lib.SFA_KERNEL_GENERAL}
_DQ = {"auto": _lib.SFA_DQ_AUTO, "separate": _lib.SFA_DQ_SEPARATE, "fused": _lib.SFA_DQ_FUSED}


@dataclass(frozen=True)
class _Cfg:
    block_size: int
    scale: float
    causal: bool
    varlen: bool
    max_q: int
    max_k: int
    dkv_mode: int
    kernel: int
    shared_kv: bool
    dq_mode: int = 0
    compat: int = 0


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _strides(t: torch.Tensor, varlen: bool, ndim_tail: int):
    """(batch, token, head) element strides; the trailing ``ndim_tail`` dims must
    be contiguous-innermost."""
    if varlen:
        return 0, t.stride(0), (t.stride(1) if t.dim() > 1 + ndim_tail - 1 else 0)
    return t.stride(0), t.stride(1), t.stride(2)


def _inner_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def build_params(q, k, v, idx, o, lse, cfg: _Cfg, sink=None, cu_q=None, cu_k=None,
                 dout=None, dq=None, dk=None, dv=None, dsink=None) -> SfaParams:
    """Fill the C struct from tensors (layouts in include/sfa_b200.h)."""
    P = SfaParams()
    P.q, P.k, P.v, P.block_indices = _ptr(q), _ptr(k), _ptr(v), _ptr(idx)
    P.cu_seqlens_q, P.cu_seqlens_k = _ptr(cu_q), _ptr(cu_k)
    P.attn_sink = _ptr(sink)
    P.o, P.lse, P.dout = _ptr(o), _ptr(lse), _ptr(dout)
    P.dq, P.dk, P.dv, P.dsink = _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dsink)
    vl = cfg.varlen

    def s3(t, is_lse=False):
        if t is None:
            return (0, 0, 0)
        if vl:
            return (0, t.stride(0), t.stride(1))
        return (t.stride(0), t.stride(1), t.stride(2))

    for name, t in (("q", q), ("k", k), ("v", v), ("i", idx), ("o", o), ("l", lse), ("do", dout),
                    ("dq", dq), ("dk", dk), ("dv", dv)):
        sb, st, sh = s3(t)
        setattr(P, f"{name}_sb", sb)
        setattr(P, f"{name}_st", st)
        setattr(P, f"{name}_sh", sh)
    if vl:
        P.batch = cu_q.numel() - 1
        P.total_q, P.total_kv = q.shape[0], k.shape[0]
        P.q_len, P.kv_len = cfg.max_q, cfg.max_k
        P.h_q, P.h_kv = q.shape[1], k.shape[1]
    else:
        P.batch, P.q_len, P.h_q = q.shape[0], q.shape[1], q.shape[2]
        P.kv_len, P.h_kv = k.shape[1], k.shape[2]
        P.total_q, P.total_kv = P.batch * P.q_len, P.batch * P.kv_len
    P.d_qk, P.d_v = q.shape[-1], v.shape[-1]
    P.block_size = cfg.block_size
    P.topk = idx.shape[-1]
    P.scale = cfg.scale
    P.causal = 1 if cfg.causal else 0
    P.dkv_mode = cfg.dkv_mode
    P.kernel = cfg.kernel
    P.dq_mode = cfg.dq_mode
    P.compat = cfg.compat
    return P


def _fwd(q, k, v, idx, sink, cu_q, cu_k, cfg: _Cfg):
    lib = _lib.load()
    o = q.new_empty(*q.shape[:-1], v.shape[-1])
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device)
    P = build_params(q, k, v, idx, o, lse, cfg, sink, cu_q, cu_k)
    _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, _stream()), "sfa_fwd")
    return o, lse


def _bwd(q, k, v, idx, sink, cu_q, cu_k, o, lse, do, cfg: _Cfg, need_dsink: bool):
    lib = _lib.load()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = dk if cfg.shared_kv else torch.empty_like(v)
    dsink = torch.empty(q.shape[-2], dtype=torch.float32, device=q.device) if need_dsink else None
    P = build_params(q, k, v, idx, o, lse, cfg, sink, cu_q, cu_k, _inner_contig(do), dq, dk, dv, dsink)
    nbytes = lib.sfa_bwd_workspace_bytes(ctypes.byref(P))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    _lib.check(lib.sfa_bwd(ctypes.byref(P), ws.data_ptr(), nbytes, _stream()), "sfa_bwd")
    return dq, dk, dv, dsink


def _check_inputs(q, k, v, idx):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (the SFA op has no CPU implementation)")
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    if idx.numel() == 0:
        raise ValueError("block indices tensor is empty. Cannot determine effective topk.")
    if idx.dtype not in (torch.int32, torch.int64, torch.int16):
        raise ValueError(f"block indices must be an integer tensor, got {idx.dtype}")


def _leading_view(v: torch.Tensor, k: torch.Tensor) -> bool:
    """v is k's leading dims (``v = k[..., :Dv]``, the MLA latent kv): the two
    share rows, so one gradient ``dk + dv`` (summed in fp32) flows back to k."""
    return (v.data_ptr() == k.data_ptr() and v.stride() == k.stride() and v.shape[:-1] == k.shape[:-1]
            and v.shape[-1] <= k.shape[-1] and k.stride(-1) == 1)


def _idx32(idx: torch.Tensor) -> torch.Tensor:
    if idx.dtype == torch.int32:
        return _inner_contig(idx)
    # values >= 2**31 cannot address a kv row the kernels accept; clamp keeps them invalid
    return idx.clamp(min=-1, max=2**31 - 1).to(torch.int32).contiguous()


class _SFAFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, idx, sink, cu_q, cu_k, cfg: _Cfg):
        o, lse = _fwd(q, k, v, idx, sink, cu_q, cu_k, cfg)
        ctx.save_for_backward(q, k, v, idx, sink, cu_q, cu_k, o, lse)
        ctx.cfg = cfg
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, do, dlse):
        q, k, v, idx, sink, cu_q, cu_k, o, lse = ctx.saved_tensors
        cfg = ctx.cfg
        need_dsink = sink is not None and ctx.needs_input_grad[4]
        dq, dk, dv, dsink = _bwd(q, k, v, idx, sink, cu_q, cu_k, o, lse, do, cfg, need_dsink)
        if cfg.shared_kv:
            return dq, dk, None, None, dsink, None, None, None
        return dq, dk, dv, None, dsink, None, None, None


def sparse_flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
                           block_size: int = 64, scale: Optional[float] = None,
                           cu_seqlens: Optional[torch.Tensor] = None, attn_sink: Optional[torch.Tensor] = None,
                           causal: bool = True, cu_seqlens_k: Optional[torch.Tensor] = None,
                           max_seqlen_q: Optional[int] = None, max_seqlen_k: Optional[int] = None,
                           dkv_mode: str = "auto", kernel: str = "auto",
                           dq_mode: str = "auto", reference_quirks: bool = False
                           ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Block-sparse attention over selected kv blocks; returns ``(o, lse)``.

    Dense: ``q [B,T,Hq,Dqk]``, ``k [B,Tk,Hk,Dqk]``, ``v [B,Tk,Hk,Dv]``,
    ``block_indices [B,T,Hk,S]``.  Varlen: drop the batch axis and pass
    ``cu_seqlens`` (query offsets; also the kv offsets unless ``cu_seqlens_k``
    is given).  Varlen calls should pass ``max_seqlen_q/k``: left unset, they are
    read back from ``cu_seqlens`` with a device->host sync.  ``lse`` is the
    natural-log log-sum-exp ``[.., Hq]`` (fp32); it carries no gradient.
    ``attn_sink`` (``[Hq]`` fp32) adds ``exp(sink)`` to every denominator.
    If ``k is v``, or v is k's leading dims (``v = k[..., :Dv]``, one latent kv
    tensor), their rows are shared and one gradient ``dk + dv`` flows back to k.
    ``dkv_mode`` ("inverted" | "atomic"), ``dq_mode`` ("separate" | "fused") and
    ``kernel`` ("tcgen05" | "general") override the launch table ("auto").

    ``reference_quirks=True`` reproduces the reference's own arithmetic and
    lse format for bit-level comparisons with its saved values: probabilities
    rounded to fp16 and then bf16 before the PV product (``SFA.py:446, 456``),
    ``lse`` returned in base 2 (``SFA.py:474``) and ``+inf`` for a row with no
    valid key when a sink is given (the reference's ``exp2(sink - m)`` with its
    ``-1e11`` max seed overflows, ``SFA.py:381, 469-474``).  Gradients use the
    natural-log lse internally either way.
    """
    _check_inputs(q, k, v, block_indices)
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    varlen = cu_seqlens is not None
    if varlen:
        cu_q = cu_seqlens.to(torch.int32).contiguous()
        cu_k = (cu_seqlens_k if cu_seqlens_k is not None else cu_seqlens).to(torch.int32).contiguous()
        if max_seqlen_q is None:
            max_seqlen_q = int((cu_q[1:] - cu_q[:-1]).max().item()) if cu_q.numel() > 1 else 0
        if max_seqlen_k is None:
            max_seqlen_k = int((cu_k[1:] - cu_k[:-1]).max().item()) if cu_k.numel() > 1 else 0
    else:
        cu_q = cu_k = None
        max_seqlen_q, max_seqlen_k = q.shape[1], k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    shared = k is v or _leading_view(v, k)
    cfg = _Cfg(int(block_size), float(scale), bool(causal), varlen, int(max_seqlen_q), int(max_seqlen_k),
               _DKV[dkv_mode], _KERNEL[kernel], shared, _DQ[dq_mode],
               _lib.SFA_COMPAT_REFERENCE_P if reference_quirks else 0)
    sink = None if attn_sink is None else attn_sink.float()
    kk = _inner_contig(k)
    vv = (kk if k is v else v) if shared else _inner_contig(v)
    idx = _idx32(block_indices)
    o, lse = _SFAFunction.apply(_inner_contig(q), kk, vv, idx, sink, cu_q, cu_k, cfg)
    if reference_quirks:
        lse = reference_lse2(lse)
        if sink is not None:
            lse = torch.where(_has_valid_key(idx, cfg, cu_q, cu_k, q.shape[-2], k.shape[-2]), lse,
                              torch.full_like(lse, float("inf")))
    return o, lse


def sparse_flash_attention_paged(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                 block_indices: torch.Tensor, block_table: torch.Tensor, cache_seqlens: torch.Tensor,
                                 block_size: int = 64, scale: Optional[float] = None,
                                 cu_seqlens: Optional[torch.Tensor] = None, attn_sink: Optional[torch.Tensor] = None,
                                 causal: bool = True, max_seqlen_q: Optional[int] = None,
                                 max_seqlen_k: Optional[int] = None, kernel: str = "auto"
                                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sparse attention forward over a paged kv cache (the serving / decode
    format); returns ``(o, lse)``, no autograd.

    ``k_cache [num_pages, page_size, Hk, Dqk]`` and ``v_cache [num_pages,
    page_size, Hk, Dv]`` are page pools (``v_cache`` may be ``k_cache`` or its
    leading dims); ``block_table [n, max_pages]`` (int32) maps sequence s's
    logical page j to a pool page; ``cache_seqlens [n]`` are the kv lengths.
    ``q [total_q, Hq, Dqk]`` with ``cu_seqlens [n + 1]`` (default: one query per
    sequence, the decode step); ``block_indices [total_q, Hk, S]`` selects
    logical blocks (tokens when ``block_size`` is 1) of each sequence, exactly
    as on the contiguous varlen surface.  ``page_size`` must be a multiple of
    ``block_size``.  ``max_seqlen_k`` left unset is read back with a host sync.
    """
    _check_inputs(q, k_cache, v_cache, block_indices)
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("k_cache / v_cache must be [num_pages, page_size, Hk, D] page pools")
    n = block_table.shape[0]
    npg, ps, hk = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
    for name, c in (("k_cache", k_cache), ("v_cache", v_cache)):
        if c.shape[:3] != k_cache.shape[:3] or c.stride(-1) != 1 or c.stride(0) != ps * c.stride(1):
            raise ValueError(f"{name}: pages must be [page_size, Hk, D] row ranges of one pool, innermost dim "
                             "contiguous")
    if cu_seqlens is None:
        if q.shape[0] != n:
            raise ValueError("without cu_seqlens, q must hold one query per sequence")
        cu_q = torch.arange(n + 1, dtype=torch.int32, device=q.device)
        max_seqlen_q = 1
    else:
        cu_q = cu_seqlens.to(torch.int32).contiguous()
        if max_seqlen_q is None:
            max_seqlen_q = int((cu_q[1:] - cu_q[:-1]).max().item()) if n else 0
    lens = cache_seqlens.to(torch.int32)
    cu_k = torch.cat([torch.zeros(1, dtype=torch.int32, device=q.device), lens.cumsum(0, dtype=torch.int32)])
    if max_seqlen_k is None:
        max_seqlen_k = int(lens.max().item()) if n else 0
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    # the pools as rows: [num_pages * page_size, Hk, D] (page p = rows p*ps .. p*ps + ps - 1)
    kpool = torch.as_strided(k_cache, (npg * ps, hk, k_cache.shape[3]), (k_cache.stride(1), k_cache.stride(2), 1))
    vpool = torch.as_strided(v_cache, (npg * ps, hk, v_cache.shape[3]), (v_cache.stride(1), v_cache.stride(2), 1))
    table = block_table.to(torch.int32)
    table = table if table.stride(-1) == 1 else table.contiguous()
    cfg = _Cfg(int(block_size), float(scale), bool(causal), True, int(max_seqlen_q), int(max_seqlen_k),
               _lib.SFA_DKV_AUTO, _KERNEL[kernel], False)
    sink = None if attn_sink is None else attn_sink.float()
    qq, idx = _inner_contig(q), _idx32(block_indices)
    o = qq.new_empty(*qq.shape[:-1], v_cache.shape[-1])
    lse = torch.empty(qq.shape[:-1], dtype=torch.float32, device=q.device)
    P = build_params(qq, kpool, vpool, idx, o, lse, cfg, sink, cu_q, cu_k)
    P.block_table, P.bt_stride, P.page_size = table.data_ptr(), table.stride(0), ps
    _lib.check(_lib.load().sfa_fwd(ctypes.byref(P), None, 0, _stream()), "sfa_fwd (paged)")
    return o, lse


def quantize_kv_fp8(kv: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """e4m3 copy of a kv tensor with one power-of-two fp32 scale per row (its
    last dim): ``kv ~= kv_fp8 * scale[..., None]``.  Power-of-two scales make
    the kernels' dequantisation (e4m3 value * scale -> bf16) exact, so a
    forward over ``(kv_fp8, scale)`` equals one over the dequantised bf16 kv."""
    amax = kv.detach().abs().amax(-1).float()
    e = torch.ceil(torch.log2(torch.clamp(amax, min=1e-30) / 448.0))
    scale = torch.where(amax > 0, torch.exp2(e), torch.ones_like(amax))
    q = (kv.detach().float() / scale[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q, scale


def sparse_flash_attention_fp8kv(q: torch.Tensor, kv_fp8: torch.Tensor, kv_scale: torch.Tensor,
                                 block_indices: torch.Tensor, d_v: int, block_size: int = 1,
                                 scale: Optional[float] = None, cu_seqlens: Optional[torch.Tensor] = None,
                                 attn_sink: Optional[torch.Tensor] = None, causal: bool = True,
                                 cu_seqlens_k: Optional[torch.Tensor] = None, max_seqlen_q: Optional[int] = None,
                                 max_seqlen_k: Optional[int] = None, kernel: str = "auto"
                                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Forward (no autograd) over one latent kv tensor stored as e4m3 with a
    fp32 scale per row — the MLA cache format: keys are ``kv_fp8 * scale``
    over all ``Dqk`` dims, values their first ``d_v`` dims.  Layouts as
    ``sparse_flash_attention`` (dense ``kv_fp8 [B, Tk, Hk, Dqk]``,
    ``kv_scale [B, Tk, Hk]``; varlen drops B).  The kernels gather half the
    bytes of a bf16 cache and widen the rows to bf16 in shared memory; see
    ``quantize_kv_fp8``."""
    if not q.is_cuda or q.dtype != torch.bfloat16:
        raise ValueError("q must be a bfloat16 CUDA tensor")
    if kv_fp8.dtype not in (torch.float8_e4m3fn, torch.uint8) or not kv_fp8.is_cuda:
        raise ValueError("kv_fp8 must be a float8_e4m3fn (or uint8) CUDA tensor")
    if kv_scale.dtype != torch.float32 or tuple(kv_scale.shape) != tuple(kv_fp8.shape[:-1]):
        raise ValueError("kv_scale must be fp32 with kv_fp8's shape minus the last dim")
    if block_indices.numel() == 0:
        raise ValueError("block indices tensor is empty. Cannot determine effective topk.")
    varlen = cu_seqlens is not None
    if varlen:
        cu_q = cu_seqlens.to(torch.int32).contiguous()
        cu_k = (cu_seqlens_k if cu_seqlens_k is not None else cu_seqlens).to(torch.int32).contiguous()
        if max_seqlen_q is None:
            max_seqlen_q = int((cu_q[1:] - cu_q[:-1]).max().item()) if cu_q.numel() > 1 else 0
        if max_seqlen_k is None:
            max_seqlen_k = int((cu_k[1:] - cu_k[:-1]).max().item()) if cu_k.numel() > 1 else 0
    else:
        cu_q = cu_k = None
        max_seqlen_q, max_seqlen_k = q.shape[1], kv_fp8.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    k8 = _inner_contig(kv_fp8.view(torch.uint8))
    v8 = k8[..., :d_v]
    cfg = _Cfg(int(block_size), float(scale), bool(causal), varlen, int(max_seqlen_q), int(max_seqlen_k),
               _lib.SFA_DKV_AUTO, _KERNEL[kernel], True)
    sink = None if attn_sink is None else attn_sink.float()
    qq, idx = _inner_contig(q), _idx32(block_indices)
    o = qq.new_empty(*qq.shape[:-1], d_v)
    lse = torch.empty(qq.shape[:-1], dtype=torch.float32, device=q.device)
    P = build_params(qq, k8, v8, idx, o, lse, cfg, sink, cu_q, cu_k)
    P.kv_dtype = _lib.SFA_KV_FP8_E4M3
    P.kv_scale = kv_scale.data_ptr()
    if varlen:
        P.ks_sb, P.ks_st, P.ks_sh = 0, kv_scale.stride(0), kv_scale.stride(1)
    else:
        P.ks_sb, P.ks_st, P.ks_sh = kv_scale.stride(0), kv_scale.stride(1), kv_scale.stride(2)
    _lib.check(_lib.load().sfa_fwd(ctypes.byref(P), None, 0, _stream()), "sfa_fwd (fp8 kv)")
    return o, lse


def _has_valid_key(idx: torch.Tensor, cfg: "_Cfg", cu_q, cu_k, hq: int, hk: int) -> torch.Tensor:
    """[.., Hq] bool: the row selected at least one valid key (the kernels'
    rule: block id in range, a key below kv_len and, when causal, at or before
    the query's position).  Elementwise on the device, no host sync."""
    bs = cfg.block_size
    e = idx.to(torch.int64)
    if cu_q is None:
        T, Tk = idx.shape[1], cfg.max_k
        pos = (torch.arange(T, device=idx.device) + (Tk - T))[None, :, None, None]
        kv_len = torch.full_like(pos, Tk)
    else:
        rows = idx.shape[0]
        r = torch.arange(rows, device=idx.device, dtype=torch.int32)
        seq = torch.searchsorted(cu_q, r, right=True) - 1
        q0, k0 = cu_q[seq], cu_k[seq]
        ql, kl = cu_q[seq + 1] - q0, cu_k[seq + 1] - k0
        pos = (r - q0 + kl - ql).to(torch.int64)[:, None, None]
        kv_len = kl.to(torch.int64)[:, None, None]
    first = e * bs
    end = torch.minimum(first + bs, kv_len)
    if cfg.causal:
        end = torch.minimum(end, pos + 1)
    ok = (e >= 0) & (first < kv_len) & (end > first)
    anyk = ok.any(-1)                                    # [.., Hk]
    return anyk.repeat_interleave(hq // hk, dim=-1)


class SparseFlashAttention(torch.autograd.Function):
    """Drop-in for the reference's ``SparseFlashAttentionTriton`` (``SFA.py:69``).

    ``forward(ctx, q [S,B,H,D], kv [S_kv,B,D], attn_sink [H], topk_idxs [S,B,TopK], sm_scale) -> out``
    Token-level top-k over one shared kv head (rows are keys and values), no
    causal mask (causality lives in the indices, as in the reference).
    """

    @staticmethod
    def forward(ctx, q, kv, attn_sink, topk_idxs, sm_scale):
        return _reference_forward(ctx, q, kv, attn_sink, topk_idxs, sm_scale, 0)

    @staticmethod
    def backward(ctx, grad_out):
        return _reference_backward(ctx, grad_out)


def _reference_forward(ctx, q, kv, attn_sink, topk_idxs, sm_scale, compat):
    _check_inputs(q, kv, kv, topk_idxs)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    cfg = _Cfg(1, float(sm_scale), False, False, q.shape[0], kv.shape[0], _lib.SFA_DKV_AUTO,
               _lib.SFA_KERNEL_AUTO, True, compat=compat)
    qi = _inner_contig(q)
    kvi = _inner_contig(kv)
    idx = _idx32(topk_idxs)
    qb = qi.permute(1, 0, 2, 3)
    kvb = kvi.permute(1, 0, 2).unsqueeze(2)
    ib = idx.permute(1, 0, 2).unsqueeze(2)
    sink = None if attn_sink is None else attn_sink.float()
    out = torch.empty_like(qi)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device)
    lib = _lib.load()
    P = build_params(qb, kvb, kvb, ib, out.permute(1, 0, 2, 3), lse.permute(1, 0, 2), cfg, sink)
    _lib.check(lib.sfa_fwd(ctypes.byref(P), None, 0, _stream()), "sfa_fwd")
    ctx.save_for_backward(qi, kvi, sink, idx, out, lse)
    ctx.cfg = cfg
    ctx.sink_given = attn_sink is not None
    return out


def _reference_backward(ctx, grad_out):
    q, kv, sink, idx, out, lse = ctx.saved_tensors
    cfg = ctx.cfg
    lib = _lib.load()
    dq = torch.empty_like(q)
    dkv = torch.empty_like(kv)
    need_dsink = ctx.sink_given and ctx.needs_input_grad[2]
    dsink = torch.empty(q.shape[2], dtype=torch.float32, device=q.device) if need_dsink else None
    qb = q.permute(1, 0, 2, 3)
    kvb = kv.permute(1, 0, 2).unsqueeze(2)
    dkvb = dkv.permute(1, 0, 2).unsqueeze(2)
    ib = idx.permute(1, 0, 2).unsqueeze(2)
    do = _inner_contig(grad_out)
    P = build_params(qb, kvb, kvb, ib, out.permute(1, 0, 2, 3), lse.permute(1, 0, 2), cfg, sink,
                     dout=do.permute(1, 0, 2, 3), dq=dq.permute(1, 0, 2, 3), dk=dkvb, dv=dkvb, dsink=dsink)
    nbytes = lib.sfa_bwd_workspace_bytes(ctypes.byref(P))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    _lib.check(lib.sfa_bwd(ctypes.byref(P), ws.data_ptr(), nbytes, _stream()), "sfa_bwd")
    return dq, dkv, dsink, None, None


class SparseFlashAttentionCompat(SparseFlashAttention):
    """``SparseFlashAttention`` with the reference's probability rounding
    (fp16, then bf16, before the PV product, ``SFA.py:446, 456``): the same
    signature and gradients, for callers that compare against outputs the
    reference produced bit for bit.  (The reference's base-2 / +inf lse is
    internal to its autograd context; ``sparse_flash_attention(...,
    reference_quirks=True)`` returns it.)"""

    @staticmethod
    def forward(ctx, q, kv, attn_sink, topk_idxs, sm_scale):
        return _reference_forward(ctx, q, kv, attn_sink, topk_idxs, sm_scale, _lib.SFA_COMPAT_REFERENCE_P)

    @staticmethod
    def backward(ctx, grad_out):
        return _reference_backward(ctx, grad_out)


def reference_lse2(lse: torch.Tensor) -> torch.Tensor:
    """The reference keeps base-2 lse (``SFA.py:474``); convert natural-log lse."""
    return lse * 1.4426950408889634
