// sfa_common.cuh — shared device-side helpers for the SFA kernels (sm_100a).
//
// Index semantics implemented here are the single source of truth for every
// kernel family: a selected block id e is valid iff 0 <= e < ceil(kv_len/bs);
// key e*bs + j is valid iff < kv_len and (causal) <= pos where
// pos = t + kv_len - q_len.  They generalise the reference's `idx >= 0` test
// (SFA.py:394-396) to block_size > 1, causal masking and out-of-range ids.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sfa_b200.h"

namespace sfa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device status word: kernels with bounded waits record why they gave up in a
// word whose address the host passes in.  0 = healthy; otherwise
// (kernel id << 16) | (site id).
__device__ __forceinline__ void record_status(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, 0, code);
}

// Per-row coordinates of a query row (dense: row = b*Tq + t; varlen: global row).
struct Row {
  int b;          // batch index used with *_sb strides (0 for varlen)
  int t;          // query index within its sequence
  int64_t tq;     // token index used with *_st strides for q/o/lse/indices
  int64_t kv0;    // first kv token (used with *_st strides for k/v; 0 for a paged cache)
  int kv_len;     // kv length of the sequence
  int q_len;      // query length of the sequence
  int pos;        // causal position of the query
  int seq;        // sequence index (dense: b)
};

__device__ __forceinline__ Row row_info(const SfaParams& p, int row) {
  Row r;
  if (p.cu_seqlens_q == nullptr) {
    r.b = row / p.q_len;
    r.t = row - r.b * p.q_len;
    r.tq = r.t;
    r.kv0 = 0;
    r.kv_len = p.kv_len;
    r.q_len = p.q_len;
    r.seq = r.b;
  } else {
    int lo = 0, hi = p.batch;  // find s with cu[s] <= row < cu[s+1]
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (__ldg(p.cu_seqlens_q + mid) <= row) lo = mid; else hi = mid;
    }
    int q0 = __ldg(p.cu_seqlens_q + lo);
    int k0 = __ldg(p.cu_seqlens_k + lo);
    r.b = 0;
    r.t = row - q0;
    r.tq = row;
    // a paged cache addresses rows through the block table (kv_row)
    r.kv0 = p.block_table ? 0 : k0;
    r.kv_len = __ldg(p.cu_seqlens_k + lo + 1) - k0;
    r.q_len = __ldg(p.cu_seqlens_q + lo + 1) - q0;
    r.seq = lo;
  }
  r.pos = r.t + r.kv_len - r.q_len;
  return r;
}

// Row of kv position t (0 <= t < kv_len) of the row's sequence: kv0 + t, or,
// for a paged cache, its page's rows in the pool.  With block_size > 1 the
// caller passes a block's first key (page_size is a multiple of block_size,
// so the block's keys are consecutive rows).
__device__ __forceinline__ int64_t kv_row(const SfaParams& p, const Row& r, int t) {
  if (p.block_table == nullptr) return r.kv0 + t;
  const int ps = p.page_size;
  const int pg = __ldg(p.block_table + (int64_t)r.seq * p.bt_stride + t / ps);
  return (int64_t)pg * ps + t % ps;
}

__device__ __forceinline__ int num_rows(const SfaParams& p) {
  return p.cu_seqlens_q == nullptr ? p.batch * p.q_len : p.total_q;
}

// Number of valid keys contributed by block id e for a query at `pos`.
// Returns the count n (keys e*bs .. e*bs+n-1 are valid), 0 if none.
__device__ __forceinline__ int block_valid_keys(int e, int bs, int kv_len, int pos, int causal) {
  if (e < 0) return 0;
  int64_t first = (int64_t)e * bs;
  if (first >= kv_len) return 0;
  int64_t end = first + bs;
  if (end > kv_len) end = kv_len;
  if (causal && end > (int64_t)pos + 1) end = (int64_t)pos + 1;
  int64_t n = end - first;
  return n > 0 ? (int)n : 0;
}

// A probability as the reference's PV matmul sees it under
// SFA_COMPAT_REFERENCE_P: stored as fp16 (SFA.py:446), so values below fp16's
// range flush and the mantissa is cut to 10 bits before the bf16 rounding.
__device__ __forceinline__ float ref_p(float p) { return __half2float(__float2half_rn(p)); }

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace sfa
