/*
 * sfa_b200.h — C ABI of the B200 (sm_100a) sparse flash attention library.
 *
 * The library computes block-sparse / top-k indexed attention forward and
 * backward with the semantics of the reference op
 * `SparseFlashAttentionTriton` (lilac-me/ops, SFA.py:69-306), generalised to
 * grouped-query heads, separate k and v, block_size > 1, causal masking and
 * varlen batches.  Every entry point:
 *   - takes plain device pointers, element strides and sizes (no framework types);
 *   - enqueues work on the given CUDA stream (a `cudaStream_t` passed as void*);
 *   - allocates no memory (scratch comes from the caller's workspace);
 *   - never synchronises the host with the device;
 *   - returns SFA_OK (0) or a negative SFA_ERR_* code; sfa_last_error_string()
 *     describes the last failure on the calling thread.
 *
 * Layouts.  Dense: q [B, Tq, Hq, Dqk], k [B, Tk, Hk, Dqk], v [B, Tk, Hk, Dv],
 * block_indices [B, Tq, Hk, S] (int32), o/dout [B, Tq, Hq, Dv], lse [B, Tq, Hq].
 * Varlen (cu_seqlens_q != NULL): the batch axis is dropped, rows of sequence i
 * are [cu_seqlens_q[i], cu_seqlens_q[i+1]) for q/o/lse/indices and
 * [cu_seqlens_k[i], cu_seqlens_k[i+1]) for k/v; block ids are relative to the
 * sequence start.  Strides are in elements; the innermost dimension of every
 * tensor is contiguous.  The reference's SBHD layout (SFA.py:87-90) is the
 * dense layout with batch and token strides swapped.
 *
 * Index semantics.  A selected block id e is valid iff 0 <= e < ceil(kv_len /
 * block_size); key e*block_size + j (j < block_size) is valid iff it is < kv_len
 * and, when causal, <= t + kv_len - q_len.  Entries may sit in any slot; a
 * duplicate entry counts once per slot.  lse is natural-log; a row with no valid
 * key and no sink has o = 0 and lse = -inf.
 */
#ifndef SFA_B200_H
#define SFA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SFA_ABI_VERSION 3

enum {
  SFA_OK = 0,
  SFA_ERR_INVALID_ARGUMENT = -1,   /* bad shape, stride, alignment or null pointer */
  SFA_ERR_UNSUPPORTED = -2,        /* shape outside every kernel family's limits */
  SFA_ERR_WORKSPACE = -3,          /* workspace missing or smaller than required */
  SFA_ERR_CUDA = -4,               /* a CUDA runtime/driver call failed */
  SFA_ERR_DEVICE_TIMEOUT = -5      /* a kernel's bounded wait expired (see sfa_device_status) */
};

/* dK/dV algorithm (SfaParams.dkv_mode). */
enum {
  SFA_DKV_AUTO = 0,      /* pick from the launch table (measured throughput) */
  SFA_DKV_INVERTED = 1,  /* block->query inverted index + key-centric pass; deterministic */
  SFA_DKV_ATOMIC = 2     /* query-centric pass with fp32 atomics */
};

/* dQ algorithm (SfaParams.dq_mode) of the tensor-core backward with the
 * inverted-index dK/dV pass; other paths always compute dQ in their own pass. */
enum {
  SFA_DQ_AUTO = 0,      /* FUSED where it applies */
  SFA_DQ_SEPARATE = 1,  /* query-centric pass that recomputes S and dP; deterministic */
  SFA_DQ_FUSED = 2      /* accumulated by the key-centric dK/dV pass from its dS (fp32
                           reductions into a workspace accumulator, order not fixed);
                           needs rows * h_q * d_qk * 4 more workspace bytes */
};

/* Opt-in reference arithmetic (SfaParams.compat).  SFA_COMPAT_REFERENCE_P
 * rounds the forward's probabilities the way SparseFlashAttentionTriton does
 * before its PV matmul: stored as fp16, read back as bf16 (SFA.py:446, 456); the
 * row sums keep the unrounded values, as there.  Default: one rounding to bf16. */
#define SFA_COMPAT_REFERENCE_P 1

/* kv storage (SfaParams.kv_dtype). */
enum {
  SFA_KV_BF16 = 0,
  SFA_KV_FP8_E4M3 = 1   /* e4m3 bytes + one fp32 scale per kv row (forward only) */
};

/* Kernel family (SfaParams.kernel); AUTO picks the tensor-core path when it
 * supports the shape and the general CUDA-core path otherwise. */
enum {
  SFA_KERNEL_AUTO = 0,
  SFA_KERNEL_TCGEN05 = 1,
  SFA_KERNEL_GENERAL = 2
};

typedef struct SfaParams {
  /* inputs (device pointers) */
  const void* q;              /* bf16 */
  const void* k;              /* bf16 */
  const void* v;              /* bf16 */
  const int32_t* block_indices;
  const int32_t* cu_seqlens_q; /* [num_seqs + 1] or NULL for dense */
  const int32_t* cu_seqlens_k; /* [num_seqs + 1] or NULL for dense */
  const float* attn_sink;     /* [Hq] fp32 or NULL */
  /* forward outputs / backward inputs */
  void* o;                    /* bf16 */
  float* lse;                 /* fp32, natural log */
  /* backward */
  const void* dout;           /* bf16 */
  void* dq;                   /* bf16 */
  void* dk;                   /* bf16 */
  void* dv;                   /* bf16; may equal dk when k and v are one tensor (then dk := dk + dv) */
  float* dsink;               /* [Hq] fp32 or NULL; overwritten */

  /* element strides: batch (dense only), token, head */
  int64_t q_sb, q_st, q_sh;
  int64_t k_sb, k_st, k_sh;
  int64_t v_sb, v_st, v_sh;
  int64_t i_sb, i_st, i_sh;   /* block_indices; the S axis is contiguous */
  int64_t o_sb, o_st, o_sh;
  int64_t l_sb, l_st, l_sh;   /* lse */
  int64_t do_sb, do_st, do_sh;
  int64_t dq_sb, dq_st, dq_sh;
  int64_t dk_sb, dk_st, dk_sh;
  int64_t dv_sb, dv_st, dv_sh;

  int32_t batch;      /* B (dense) or number of sequences (varlen) */
  int32_t q_len;      /* Tq (dense) or max query length over sequences (varlen) */
  int32_t kv_len;     /* Tk (dense) or max kv length over sequences (varlen) */
  int32_t total_q;    /* varlen: cu_seqlens_q[batch]; dense: ignored */
  int32_t total_kv;   /* varlen: cu_seqlens_k[batch]; dense: ignored */
  int32_t h_q, h_kv;  /* h_q % h_kv == 0 */
  int32_t d_qk, d_v;
  int32_t block_size; /* keys per selected block (1 = token-level) */
  int32_t topk;       /* S, slots per (query, kv head) */
  float scale;        /* softmax scale applied to q.k */
  int32_t causal;     /* 0 / 1 */
  int32_t dkv_mode;   /* SFA_DKV_* */
  int32_t kernel;     /* SFA_KERNEL_* */
  int32_t dq_mode;    /* SFA_DQ_* (was reserved: zero = AUTO) */
  int32_t compat;     /* SFA_COMPAT_* bits (was reserved: zero = none) */
  /* Paged kv cache (forward only; no reference counterpart): when block_table
   * is non-NULL, k and v are page pools of total_kv rows (page p holds rows
   * [p*page_size, (p+1)*page_size), row stride k_st / v_st), the call is
   * varlen, cu_seqlens_k gives only the kv lengths (cu_seqlens_k[s+1] -
   * cu_seqlens_k[s]), and kv position t of sequence s is pool row
   * block_table[s*bt_stride + t/page_size]*page_size + t%page_size.  With
   * block_size > 1, page_size must be a multiple of block_size. */
  int32_t page_size;
  const int32_t* block_table;
  int64_t bt_stride;
  /* fp8 kv (forward only; no reference counterpart): with kv_dtype =
   * SFA_KV_FP8_E4M3, k points to e4m3 bytes (strides in bytes; v must be k or
   * its leading d_v dims, the MLA latent) and kv_scale to one fp32 scale per
   * kv row, indexed b*ks_sb + t*ks_st + h*ks_sh (t the kv row, through the
   * block table when paged): key = e4m3 value * scale, rounded to bf16 for
   * the bf16 MMAs (exact when the scales are powers of two). */
  int32_t kv_dtype;   /* SFA_KV_* */
  int32_t reserved;
  const float* kv_scale;
  int64_t ks_sb, ks_st, ks_sh;
} SfaParams;

/* Library / ABI identification. */
int sfa_abi_version(void);
const char* sfa_build_info(void);

/* Message for the last non-OK return on this thread. */
const char* sfa_last_error_string(void);

/* Number of kernels this library has enqueued since it was loaded (all
 * threads); a caller brackets a region with two reads to count its launches. */
unsigned long long sfa_kernel_launches(void);

/* Launch trace, for benchmarks that time each kernel with CUDA events (no
 * counterpart in the reference).  `events` holds n_events cudaEvent_t handles
 * (as void*) created by the caller; while it is set, every kernel or memset the
 * library enqueues from the calling thread is followed by a cudaEventRecord of
 * the next unused event on the same stream, so the time between consecutive
 * events (the first one against an event the caller records before its call)
 * is one operation.  sfa_launch_trace_count() gives how many events were
 * recorded and sfa_launch_trace_name(i) the operation event i closes.  Passing
 * NULL stops tracing; a new call restarts the count.  The events must outlive
 * the trace. */
int sfa_launch_trace(void* const* events, int n_events);
int sfa_launch_trace_count(void);
const char* sfa_launch_trace_name(int i);

/* Which kernel family a call with these params would launch (SFA_KERNEL_*), or
 * a negative error code if the shape is unsupported. */
int sfa_select_kernel(const SfaParams* p, int is_backward);

/* The backward's resolved algorithms for these params: *dkv_mode gets
 * SFA_DKV_INVERTED or SFA_DKV_ATOMIC, *dq_mode SFA_DQ_SEPARATE or SFA_DQ_FUSED
 * (the launch-table counterpart of SFA.py:51-59; no reference entry point).
 * Returns the kernel family or a negative error code. */
int sfa_bwd_plan(const SfaParams* p, int32_t* dkv_mode, int32_t* dq_mode);

/* Workspace (device bytes) the forward / backward need for these params.  The
 * token-level backward above 256 head dims runs in two passes over bf16 P and
 * dS' rows (topk slots per query head); its workspace holds them for a wave of
 * query rows sized to stay within 4 GiB (the environment variable
 * SFA_MLA_WAVE_ROWS, read at each call, sets the rows per wave instead). */
size_t sfa_fwd_workspace_bytes(const SfaParams* p);
size_t sfa_bwd_workspace_bytes(const SfaParams* p);

/* Forward: writes o and lse.  Replaces SparseFlashAttentionTriton.forward
 * (SFA.py:75-164): the reference's `_attn_fwd` launch (SFA.py:122-159) and its
 * per-launch workspaces (SFA.py:117-120), without the host sync of
 * `_effective_topk` (SFA.py:62-66). */
int sfa_fwd(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);

/* Backward: writes dq, dk, dv and (if non-NULL) dsink.  Replaces
 * SparseFlashAttentionTriton.backward (SFA.py:167-306): `_attn_bwd_dq_dsink`
 * (SFA.py:199-251) and `_attn_bwd_dk_dv` (SFA.py:266-298). */
int sfa_bwd(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);

/* The backward's stages, for callers that schedule them separately.  Each takes
 * the same workspace as sfa_bwd.
 *  - preprocess: delta = rowsum(o * dout) in fp32 and dsink
 *    (replaces `_get_delta_split`, SFA.py:590-610, and the dsink atomics,
 *    SFA.py:964-970);
 *  - dq: replaces `_attn_bwd_dq_dsink` / `_inner_dq` (SFA.py:613-716, 856-1002);
 *    with SFA_DQ_FUSED it only clears the dQ accumulator;
 *  - dkdv: replaces `_attn_bwd_dk_dv` / `_inner_dkv` (SFA.py:719-853, 1005-1145);
 *    with SFA_DKV_INVERTED it first builds the block->query index; with
 *    SFA_DQ_FUSED it also accumulates dQ and writes dq.
 * Run them in this order on one stream. */

int sfa_bwd_preprocess(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);
int sfa_bwd_dq(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);
int sfa_bwd_dkdv(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);

/* Backward for callers that cannot allocate device memory (no counterpart in the
 * reference).  Same results as sfa_bwd, but the scratch comes from a 32 MiB
 * static device array inside the library instead of a caller workspace; every
 * GPU that loads the library reserves that array until the process exits.
 * With dq_mode SFA_DQ_AUTO, dQ runs as its own pass (SFA_DQ_SEPARATE) when the
 * fused accumulator would not fit; problems whose workspace still exceeds
 * 32 MiB are refused with SFA_ERR_WORKSPACE before anything is launched.  The first call on a device
 * looks up the array's device address; make it before any stream capture.
 * Calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  The looked-up address is kept for the life of the
 * process: after a device reset (cudaDeviceReset, or a primary-context reset)
 * the library must be reloaded before this entry point is called again. */
int sfa_bwd_noalloc(const SfaParams* p, void* stream);

/* Inverted index alone (for tests): for every (sequence, kv head, block) the
 * list of query rows that selected it, ascending by (query, slot).  Layout in
 * the workspace is described by sfa_inverted_index_layout(). */
int sfa_build_inverted_index(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream);
/* Byte offsets inside the backward workspace of: block offsets (int32,
 * [units * nblk + 1]) and query-row entries (int32, [pairs]); also reports
 * nblk (blocks per unit) and units (= batch * h_kv). */
int sfa_inverted_index_layout(const SfaParams* p, size_t* offsets_off, size_t* entries_off,
                              int32_t* nblk, int32_t* units);

/* Device status word written by kernels whose bounded waits expired.
 * sfa_device_status copies it to *status (synchronising `stream`); sfa_reset_device_status
 * clears it (stream-ordered). 0 = healthy. */
int sfa_device_status(void* stream, int32_t* status);
int sfa_reset_device_status(void* stream);

/* Self-test of that failure path: one warp waits, with a limit of limit_us
 * (1 .. 1e6), on an mbarrier nothing ever arrives on, through the same bounded
 * wait the kernels use.  The wait runs out and the status word receives
 * SFA_SELFTEST_STATUS (unless an earlier code is still there); the kernel
 * returns and the context stays usable.  Stream-ordered. */
#define SFA_SELFTEST_STATUS ((15 << 16) | 1)
int sfa_selftest_wait_timeout(void* stream, uint32_t limit_us);

/* ------------------------------------------------------------------------
 * Top-k token indexer: the step before the op, producing its token-level
 * indices (the reference consumes topk_idxs and has no indexer, SFA.py:90).
 * Scores follow the lightning-indexer formula of DeepSeek-V3.2's sparse
 * attention:  I[t, s] = sum_h w[t, h] * ReLU(q_idx[t, h] . k_idx[s]),  s a key
 * of t's sequence (s <= t + kv_len - q_len when causal).  The output row of t
 * holds the indices of the topk highest scores (ties: the lower index first)
 * in ascending order, then -1 when fewer keys exist — the layout the op's
 * token-level surface and the reference take as-is.
 *
 * Dense layout: q_idx [B, Tq, H, D] bf16, k_idx [B, Tk, D] bf16 (one head
 * shared by every query head), weights [B, Tq, H] fp32, out [B, Tq, topk]
 * int32; strides in elements, innermost dims contiguous.  H is 64 or 32,
 * D is 64 or 128, topk <= 4096 (fp32 scores of a row go through shared
 * memory: Tk <= 49152).  The workspace holds fp32 scores for a wave of rows. */
typedef struct SfaIndexerParams {
  const void* q_idx;
  const void* k_idx;
  const float* weights;
  int32_t* out;
  int64_t q_sb, q_st, q_sh;
  int64_t k_sb, k_st;
  int64_t w_sb, w_st;
  int64_t o_sb, o_st;
  int32_t batch, q_len, kv_len, heads, dim, topk;
  int32_t causal;
  int32_t reserved;
} SfaIndexerParams;

size_t sfa_indexer_workspace_bytes(const SfaIndexerParams* p);
int sfa_indexer_topk(const SfaIndexerParams* p, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SFA_B200_H */
