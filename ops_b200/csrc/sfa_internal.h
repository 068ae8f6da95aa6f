// sfa_internal.h — host-side declarations shared by the SFA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "../../include/sfa_b200.h"

namespace sfa {

inline int num_rows_host(const SfaParams& p) {
  return p.cu_seqlens_q == nullptr ? p.batch * p.q_len : p.total_q;
}
inline int64_t kv_rows_host(const SfaParams& p) {
  return p.cu_seqlens_q == nullptr ? (int64_t)p.batch * p.kv_len : (int64_t)p.total_kv;
}

// Backward workspace carve-up (all regions 256-byte aligned).
struct BwdLayout {
  size_t delta;        // float [rows * h_q]
  size_t dsink_part;   // float [pre_ctas * h_q]
  size_t dk_acc;       // float [kv_rows * h_kv * d_qk]   (atomic dk/dv path)
  size_t dv_acc;       // float [kv_rows * h_kv * d_v]    (atomic dk/dv path; unused when dv == dk)
  size_t inv_offsets;  // int32 [units * nblk + 1]        (inverted path)
  size_t inv_entries;  // int32 [pairs]                   (inverted path)
  size_t inv_cursor;   // int32 [units * nblk]            (inverted path scratch)
  size_t sched;        // int32 work counter               (inverted path)
  size_t dq_acc;       // float [rows * h_q * d_qk]       (fused dQ)
  size_t dkv_part;     // float [units*nblk*nranges][2][64][d_qk] (row-range split)
  size_t mla_pd;       // bf16 P and dS' of one wave (two-pass token-level backward)
  size_t total;
  int inv_nsub;        // 128-row sub-chunks per unit in the index counts (padded)
  int sub_per_range;   // sub-chunks per row range of the key-centric pass
  int nranges;         // row ranges (1: no split)
  int pre_ctas;
  int nblk;
  int units;
  int64_t pairs;
  bool atomic_dkv;
  bool inverted_dkv;
  bool fused_dq;
  bool two_pass;       // token-level backward in two passes (head dims above 256)
};

constexpr int kPreRows = 16;  // query rows per preprocess CTA (x h_q must stay a multiple of 16: the
                              // delta kernel's half-warps loop in step)

BwdLayout bwd_layout(const SfaParams& p, int kernel_family, int dkv_mode, int dq_mode);

// general (CUDA-core) family
cudaError_t launch_fwd_general(const SfaParams& p, cudaStream_t st);
cudaError_t launch_bwd_general(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc,
                               cudaStream_t st);
size_t fwd_general_smem(const SfaParams& p, int HG);
size_t bwd_general_smem(const SfaParams& p, int HG);
int general_head_group(const SfaParams& p);

// backward preprocessing / epilogues
cudaError_t launch_preprocess(const SfaParams& p, float* delta, float* dsink_part, int pre_ctas, cudaStream_t st);
cudaError_t launch_convert_dkdv(const SfaParams& p, const float* dk_acc, const float* dv_acc, cudaStream_t st);
// dk/dv from the row-range partials of the key-centric pass, summed in range order
cudaError_t launch_reduce_dkdv_ranges(const SfaParams& p, const BwdLayout& L, const char* ws, cudaStream_t st);
// dq = bf16(scale * dq_acc), dq_acc fp32 [rows][h_q][d_qk]
// one warp waits, with a limit of limit_us, on an mbarrier nothing arrives on (sfa_selftest.cu)
cudaError_t launch_wait_probe(uint32_t limit_us, int32_t* status, cudaStream_t st);
cudaError_t launch_convert_dq(const SfaParams& p, const float* dq_acc, cudaStream_t st);

// inverted block->query index
cudaError_t launch_inverted_index(const SfaParams& p, const BwdLayout& L, char* ws, cudaStream_t st);

// tensor-core (tcgen05) family: block-sparse kernels (block_size 64) and the
// token-level forward (block_size 1, sfa_tok_fwd.cu)
bool tok_fwd_supported(const SfaParams& p, const char** why);
cudaError_t launch_fwd_tok(const SfaParams& p, cudaStream_t st);
// token-level backward (sfa_tok_bwd.cu): dq, and dk/dv added into the fp32
// accumulators (zeroed by the caller) of the atomic workspace layout
bool tok_bwd_supported(const SfaParams& p, const char** why);
cudaError_t launch_bwd_tok(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc, cudaStream_t st);
// its two-pass form's gradient half: rows [r0, r1) with P and dS' read from the
// workspace rows [r1 - r0][h_q][ld] (bf16)
bool tok_bwd_parts_supported(const SfaParams& p, const char** why);
cudaError_t launch_bwd_tok_parts(const SfaParams& p, float* dk_acc, float* dv_acc, const void* pws, const void* dsws,
                                 int64_t ld, int r0, int r1, cudaStream_t st);
// two-pass token-level backward for head dims above 256 (sfa_mla_bwd.cu): the
// stacked [S ; dP] pass writes P and dS' to a workspace of mla_ws_bytes, the
// gradient half adds dk/dv into the fp32 accumulators and writes dq; rows go
// through in waves of mla_wave_rows
bool mla_bwd_supported(const SfaParams& p, const char** why);
int64_t mla_ws_ld(const SfaParams& p);
int64_t mla_wave_rows(const SfaParams& p);
size_t mla_ws_bytes(const SfaParams& p);
cudaError_t launch_bwd_mla(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc, void* pd,
                           cudaStream_t st);
bool tc_fwd_supported(const SfaParams& p, const char** why);
bool tc_bwd_supported(const SfaParams& p, const char** why);
cudaError_t launch_fwd_tc(const SfaParams& p, cudaStream_t st);
cudaError_t launch_bwd_dq_tc(const SfaParams& p, const float* delta, cudaStream_t st);
bool tc_dkdv_available();
// dq_acc: fused dQ accumulator (fp32 [rows][h_q][d_qk], zeroed) or null
cudaError_t launch_bwd_dkdv_tc(const SfaParams& p, const BwdLayout& L, char* ws, const float* delta, float* dq_acc,
                               cudaStream_t st);

int device_sm_count();
int device_cc();

// Count of kernels this library has enqueued (reported by sfa_kernel_launches);
// also a point of the calling thread's launch trace (sfa_launch_trace).
void note_launch(const char* name, cudaStream_t st);
// A memset enqueued by the library: a trace point, not a kernel of its own.
void note_memset(const char* name, cudaStream_t st);

// Record `msg` for sfa_last_error_string() and return `code`.
int report_error(int code, const std::string& msg);

}  // namespace sfa
