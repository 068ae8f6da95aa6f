"""ops_b200 — B200-native (sm_100a) sparse flash attention.

Public surface:
  sparse_flash_attention(q, k, v, block_indices, ...) -> (o, lse)
  SparseFlashAttention.apply(q, kv, attn_sink, topk_idxs, sm_scale) -> out   # reference signature
  sparse_flash_attention_paged(q, k_cache, v_cache, block_indices, block_table, cache_seqlens, ...)
                                                      # forward over a paged kv cache (decode)
  lightning_indexer_topk(q_idx, k_idx, weights, topk) -> token indices for the op
  sparse_flash_attention_fp8kv(q, kv_fp8, kv_scale, block_indices, d_v, ...)  # e4m3 latent kv cache
The kernels live in libsfa_b200.so (C ABI: include/sfa_b200.h).
"""
from ._lib import SfaError, SfaParams, load as load_library
from .sfa import (SparseFlashAttention, SparseFlashAttentionCompat, quantize_kv_fp8, reference_lse2,
                  sparse_flash_attention, sparse_flash_attention_fp8kv, sparse_flash_attention_paged)
from . import tiling
from .indexer import lightning_indexer_topk

__all__ = ["sparse_flash_attention", "sparse_flash_attention_paged", "SparseFlashAttention",
           "SparseFlashAttentionCompat", "SfaError", "SfaParams", "load_library", "reference_lse2", "tiling",
           "lightning_indexer_topk", "sparse_flash_attention_fp8kv", "quantize_kv_fp8"]
