// sfa_capi.cu — the extern "C" boundary of libsfa_b200.so.
//
// Validates SfaParams, picks a kernel family through the launch table
// (the sm_100a counterpart of the reference's CONFIG_MAP /
// _resolve_tiling_config, SFA.py:16-59, keyed on shape instead of a host-synced
// max valid count), carves the caller's workspace and enqueues kernels on the
// caller's stream.  No allocation, no host synchronisation.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "sfa_common.cuh"
#include "sfa_internal.h"

namespace sfa {

static thread_local std::string g_err;

static int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int report_error(int code, const std::string& msg) { return fail(code, msg); }

static int cuda_fail(cudaError_t e, const char* where) {
  return fail(SFA_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

// Device status word (see sfa_common.cuh).  Host code takes its address per
// device with cudaGetSymbolAddress; kernels receive that pointer.
__device__ int32_t g_status_word = 0;

static int32_t* status_ptr_for_current_device() {
  static std::mutex mu;
  static int32_t* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_status_word) != cudaSuccess) return nullptr;
    ptrs[dev] = reinterpret_cast<int32_t*>(ptr);
  }
  return ptrs[dev];
}

int32_t* device_status_ptr() { return status_ptr_for_current_device(); }

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

int device_cc() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!cache[dev]) {
    int ma = 0, mi = 0;
    cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, dev);
    cache[dev] = ma * 10 + mi;
  }
  return cache[dev];
}

static std::atomic<unsigned long long> g_launches{0};

// Launch trace (sfa_launch_trace): while a caller has handed in events, each
// kernel or memset this thread enqueues is followed by a record of the next
// event on the same stream, so consecutive events bracket one operation.
struct LaunchTrace {
  void* const* events = nullptr;
  int n = 0;
  int count = 0;
  const char* names[64] = {nullptr};
};
static thread_local LaunchTrace g_trace;

static void trace_point(const char* name, cudaStream_t st) {
  if (!g_trace.events || g_trace.count >= g_trace.n) return;
  cudaEventRecord(reinterpret_cast<cudaEvent_t>(g_trace.events[g_trace.count]), st);
  if (g_trace.count < 64) g_trace.names[g_trace.count] = name;
  ++g_trace.count;
}

void note_launch(const char* name, cudaStream_t st) {
  g_launches.fetch_add(1ull, std::memory_order_relaxed);
  trace_point(name, st);
}

void note_memset(const char* name, cudaStream_t st) { trace_point(name, st); }

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static int validate(const SfaParams* p, bool bwd) {
  if (!p) return fail(SFA_ERR_INVALID_ARGUMENT, "params is NULL");
  if (!p->q || !p->k || !p->v || !p->block_indices || !p->o || !p->lse)
    return fail(SFA_ERR_INVALID_ARGUMENT, "q, k, v, block_indices, o and lse must be non-NULL");
  if (bwd && (!p->dout || !p->dq || !p->dk || !p->dv))
    return fail(SFA_ERR_INVALID_ARGUMENT, "dout, dq, dk and dv must be non-NULL for the backward");
  if (p->batch < 0 || p->q_len < 0 || p->kv_len < 0)
    return fail(SFA_ERR_INVALID_ARGUMENT, "batch, q_len and kv_len must be >= 0");
  if (p->h_q <= 0 || p->h_kv <= 0 || p->h_q % p->h_kv)
    return fail(SFA_ERR_INVALID_ARGUMENT, "h_q must be a positive multiple of h_kv");
  if (p->d_qk <= 0 || p->d_v <= 0) return fail(SFA_ERR_INVALID_ARGUMENT, "head dims must be positive");
  if (p->block_size <= 0) return fail(SFA_ERR_INVALID_ARGUMENT, "block_size must be positive");
  if (p->topk <= 0) return fail(SFA_ERR_INVALID_ARGUMENT, "topk must be positive (empty index tensor)");
  if ((p->cu_seqlens_q == nullptr) != (p->cu_seqlens_k == nullptr))
    return fail(SFA_ERR_INVALID_ARGUMENT, "cu_seqlens_q and cu_seqlens_k must both be set or both be NULL");
  if (p->cu_seqlens_q && (p->total_q < 0 || p->total_kv < 0))
    return fail(SFA_ERR_INVALID_ARGUMENT, "total_q / total_kv must be >= 0 for varlen");
  if (bwd && p->dk == p->dv &&
      (p->k != p->v || p->d_v > p->d_qk || p->v_sb != p->k_sb || p->v_st != p->k_st || p->v_sh != p->k_sh ||
       p->dv_sb != p->dk_sb || p->dv_st != p->dk_st || p->dv_sh != p->dk_sh))
    return fail(SFA_ERR_INVALID_ARGUMENT,
                "dk may alias dv only when v is k or its leading d_v dims (same pointer and strides)");
  if (bwd && p->dkv_mode != SFA_DKV_AUTO && p->dkv_mode != SFA_DKV_INVERTED && p->dkv_mode != SFA_DKV_ATOMIC)
    return fail(SFA_ERR_INVALID_ARGUMENT, "unknown dkv_mode");
  if (p->kernel != SFA_KERNEL_AUTO && p->kernel != SFA_KERNEL_TCGEN05 && p->kernel != SFA_KERNEL_GENERAL)
    return fail(SFA_ERR_INVALID_ARGUMENT, "unknown kernel family");
  if (bwd && p->dq_mode != SFA_DQ_AUTO && p->dq_mode != SFA_DQ_SEPARATE && p->dq_mode != SFA_DQ_FUSED)
    return fail(SFA_ERR_INVALID_ARGUMENT, "unknown dq_mode");
  if (p->kv_dtype != SFA_KV_BF16 && p->kv_dtype != SFA_KV_FP8_E4M3)
    return fail(SFA_ERR_INVALID_ARGUMENT, "unknown kv_dtype");
  if (p->kv_dtype == SFA_KV_FP8_E4M3) {
    if (bwd) return fail(SFA_ERR_UNSUPPORTED, "fp8 kv is a forward (inference) format: no backward");
    if (!p->kv_scale) return fail(SFA_ERR_INVALID_ARGUMENT, "fp8 kv needs kv_scale");
    if (p->v != p->k || p->v_sb != p->k_sb || p->v_st != p->k_st || p->v_sh != p->k_sh || p->d_v > p->d_qk)
      return fail(SFA_ERR_INVALID_ARGUMENT, "fp8 kv: v must be k or its leading d_v dims (one latent kv tensor)");
  }
  if (p->block_table) {
    if (bwd) return fail(SFA_ERR_UNSUPPORTED, "a paged kv cache is a forward (decode) format: no backward");
    if (!p->cu_seqlens_q) return fail(SFA_ERR_INVALID_ARGUMENT, "a paged kv cache needs the varlen layout");
    if (p->page_size <= 0 || p->page_size % p->block_size)
      return fail(SFA_ERR_INVALID_ARGUMENT, "page_size must be a positive multiple of block_size");
    if (p->bt_stride < (p->kv_len + p->page_size - 1) / p->page_size)
      return fail(SFA_ERR_INVALID_ARGUMENT, "bt_stride must cover ceil(kv_len / page_size) pages a sequence");
  }
  return SFA_OK;
}

static bool general_supported(const SfaParams& p, bool bwd, std::string* why) {
  int HG = general_head_group(p);
  size_t need = bwd ? bwd_general_smem(p, HG) : fwd_general_smem(p, HG);
  if (need > 227 * 1024) {
    *why = "head dims too large for the general kernel's shared memory (" + std::to_string(need) + " bytes)";
    return false;
  }
  return true;
}

// Launch table: family for (shape, direction).
static int select_family(const SfaParams& p, bool bwd, std::string* why) {
  const char* tc_why = "";
  bool tc_ok;
  if (bwd)
    tc_ok = p.block_size == 1 ? (tok_bwd_supported(p, &tc_why) || mla_bwd_supported(p, &tc_why))
                              : tc_bwd_supported(p, &tc_why);
  else
    tc_ok = p.block_size == 1 ? tok_fwd_supported(p, &tc_why) : tc_fwd_supported(p, &tc_why);
  if (p.kernel == SFA_KERNEL_TCGEN05) {
    if (!tc_ok) { *why = std::string("tcgen05 family: ") + tc_why; return SFA_ERR_UNSUPPORTED; }
    return SFA_KERNEL_TCGEN05;
  }
  if (p.kernel == SFA_KERNEL_AUTO && tc_ok) return SFA_KERNEL_TCGEN05;
  if (!general_supported(p, bwd, why)) return SFA_ERR_UNSUPPORTED;
  return SFA_KERNEL_GENERAL;
}

static int resolve_dkv_mode(const SfaParams& p, int family) {
  // token-level selections have no shared block structure for a key-centric
  // pass: the query-centric kernels add dk/dv with fp32 reductions
  if (family == SFA_KERNEL_GENERAL || p.block_size == 1) return SFA_DKV_ATOMIC;
  if (p.dkv_mode == SFA_DKV_ATOMIC || !tc_dkdv_available()) return SFA_DKV_ATOMIC;
  return SFA_DKV_INVERTED;
}

// dQ fused into the key-centric pass needs its dS, so only the tensor-core
// family with the inverted-index dK/dV offers it; AUTO takes it.
static int resolve_dq_mode(const SfaParams& p, int family, int dkv_mode) {
  if (family != SFA_KERNEL_TCGEN05 || dkv_mode != SFA_DKV_INVERTED) return SFA_DQ_SEPARATE;
  return p.dq_mode == SFA_DQ_SEPARATE ? SFA_DQ_SEPARATE : SFA_DQ_FUSED;
}

BwdLayout bwd_layout(const SfaParams& p, int family, int dkv_mode, int dq_mode) {
  BwdLayout L{};
  const int64_t rows = num_rows_host(p);
  const int64_t kvr = kv_rows_host(p);
  size_t off = 0;
  L.delta = off;
  off = align256(off + sizeof(float) * rows * p.h_q);
  L.pre_ctas = (int)((rows + kPreRows - 1) / kPreRows);
  L.dsink_part = off;
  off = align256(off + sizeof(float) * (size_t)L.pre_ctas * p.h_q);
  L.units = p.batch * p.h_kv;
  L.nblk = (p.kv_len + p.block_size - 1) / p.block_size;
  L.atomic_dkv = (dkv_mode == SFA_DKV_ATOMIC);
  L.inverted_dkv = !L.atomic_dkv;
  if (L.atomic_dkv) {
    L.dk_acc = off;
    off = align256(off + sizeof(float) * kvr * p.h_kv * p.d_qk);
    if (p.dk != p.dv || p.d_v != p.d_qk) {
      L.dv_acc = off;
      off = align256(off + sizeof(float) * kvr * p.h_kv * p.d_v);
    } else {
      L.dv_acc = L.dk_acc;
    }
    const char* why = "";
    L.two_pass = family == SFA_KERNEL_TCGEN05 && p.block_size == 1 && !tok_bwd_supported(p, &why);
    if (L.two_pass) {
      L.mla_pd = off;
      off = align256(off + mla_ws_bytes(p));
    }
  } else {
    const int64_t nlists = (int64_t)L.units * L.nblk;
    L.inv_offsets = off;
    off = align256(off + sizeof(int32_t) * (nlists + 1));
    L.pairs = rows * p.h_kv * (int64_t)p.topk;
    L.inv_entries = off;
    off = align256(off + sizeof(int32_t) * L.pairs);
    // counts [units][nblk][nsub_pad] + tile sums + total (see launch_inverted_index)
    const int rows_per_warp = 128, warps = 8;
    int64_t nsub = (p.q_len + rows_per_warp - 1) / rows_per_warp;
    int64_t nsub_pad = ((nsub + warps - 1) / warps) * warps;
    L.inv_nsub = (int)nsub_pad;
    int64_t ncount = nlists * nsub_pad;
    int64_t ntiles = (ncount + 2047) / 2048;
    L.inv_cursor = off;
    off = align256(off + sizeof(int32_t) * (ncount + ntiles + 1));
    L.sched = off;
    off = align256(off + sizeof(int32_t));
  }
  L.fused_dq = (family == SFA_KERNEL_TCGEN05 && L.inverted_dkv && dq_mode == SFA_DQ_FUSED);
  L.nranges = 1;
  L.sub_per_range = L.inv_nsub;
  if (L.fused_dq) {
    L.dq_acc = off;
    off = align256(off + sizeof(float) * (size_t)rows * p.h_q * p.d_qk);
    // Row ranges of kRangeRows queries: the CTAs working at one time then touch
    // one range's q/dO rows and dQ accumulator rows, which stay in L2; each
    // range leaves an fp32 dK/dV partial per block, summed in range order.
    // (at most 64 ranges: longer sequences get longer ranges)
    constexpr int kRangeRows = 2048, kMaxRanges = 64;
    const int64_t nsub = (p.q_len + 127) / 128;
    L.sub_per_range = (int)std::max<int64_t>(kRangeRows / 128, (nsub + kMaxRanges - 1) / kMaxRanges);
    L.nranges = (int)((nsub + L.sub_per_range - 1) / L.sub_per_range);
    if (L.nranges > 1) {
      L.dkv_part = off;
      off = align256(off + sizeof(float) * (size_t)L.units * L.nblk * L.nranges * 2 * 64 * p.d_qk);
    } else {
      L.nranges = 1;
    }
  }
  L.total = off;
  return L;
}

}  // namespace sfa

using namespace sfa;

extern "C" {

int sfa_abi_version(void) { return SFA_ABI_VERSION; }

const char* sfa_build_info(void) {
  return "sfa_b200 sm_100a (tcgen05/TMA/TMEM + CUDA-core general family), ABI " "3";
}

const char* sfa_last_error_string(void) { return g_err.c_str(); }

unsigned long long sfa_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int sfa_select_kernel(const SfaParams* p, int is_backward) {
  int rc = validate(p, is_backward != 0);
  if (rc) return rc;
  std::string why;
  int fam = select_family(*p, is_backward != 0, &why);
  if (fam < 0) return fail(fam, why);
  return fam;
}

int sfa_bwd_plan(const SfaParams* p, int32_t* dkv_mode, int32_t* dq_mode) {
  int rc = validate(p, true);
  if (rc) return rc;
  std::string why;
  const int fam = select_family(*p, true, &why);
  if (fam < 0) return fail(fam, why);
  const int dkv = resolve_dkv_mode(*p, fam);
  if (dkv_mode) *dkv_mode = dkv;
  if (dq_mode) *dq_mode = resolve_dq_mode(*p, fam, dkv);
  return fam;
}

size_t sfa_fwd_workspace_bytes(const SfaParams* p) {
  (void)p;
  return 0;
}

size_t sfa_bwd_workspace_bytes(const SfaParams* p) {
  if (validate(p, true)) return 0;
  std::string why;
  int fam = select_family(*p, true, &why);
  if (fam < 0) return 0;
  const int dkv = resolve_dkv_mode(*p, fam);
  return bwd_layout(*p, fam, dkv, resolve_dq_mode(*p, fam, dkv)).total;
}

int sfa_fwd(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  int rc = validate(p, false);
  if (rc) return rc;
  std::string why;
  int fam = select_family(*p, false, &why);
  if (fam < 0) return fail(fam, why);
  if (num_rows_host(*p) == 0) return SFA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = (fam != SFA_KERNEL_TCGEN05) ? launch_fwd_general(*p, st)
                  : (p->block_size == 1 ? launch_fwd_tok(*p, st) : launch_fwd_tc(*p, st));
  if (e != cudaSuccess) return cuda_fail(e, "sfa_fwd launch");
  return SFA_OK;
}

static int bwd_common(const SfaParams* p, void* ws, size_t ws_bytes, int* fam, int* mode, BwdLayout* L) {
  int rc = validate(p, true);
  if (rc) return rc;
  std::string why;
  *fam = select_family(*p, true, &why);
  if (*fam < 0) return fail(*fam, why);
  *mode = resolve_dkv_mode(*p, *fam);
  *L = bwd_layout(*p, *fam, *mode, resolve_dq_mode(*p, *fam, *mode));
  if (L->total > 0 && (ws == nullptr || ws_bytes < L->total))
    return fail(SFA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(L->total) + " bytes, got " +
                                       std::to_string(ws_bytes));
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(SFA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  return SFA_OK;
}

int sfa_bwd_preprocess(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int fam, mode;
  BwdLayout L;
  int rc = bwd_common(p, workspace, workspace_bytes, &fam, &mode, &L);
  if (rc) return rc;
  char* ws = reinterpret_cast<char*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = launch_preprocess(*p, reinterpret_cast<float*>(ws + L.delta),
                                    reinterpret_cast<float*>(ws + L.dsink_part), L.pre_ctas, st);
  if (e != cudaSuccess) return cuda_fail(e, "sfa_bwd_preprocess");
  return SFA_OK;
}

int sfa_bwd_dq(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int fam, mode;
  BwdLayout L;
  int rc = bwd_common(p, workspace, workspace_bytes, &fam, &mode, &L);
  if (rc) return rc;
  char* ws = reinterpret_cast<char*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float* delta = reinterpret_cast<const float*>(ws + L.delta);
  cudaError_t e;
  if (L.fused_dq) {
    // the dK/dV pass accumulates dQ: start from zero
    e = cudaMemsetAsync(ws + L.dq_acc, 0, sizeof(float) * (size_t)num_rows_host(*p) * p->h_q * p->d_qk, st);
    note_memset("memset_dq_acc", st);
  } else if (fam == SFA_KERNEL_TCGEN05 && p->block_size != 1) {
    e = launch_bwd_dq_tc(*p, delta, st);
  } else {
    // the general kernel and the token-level tensor-core kernel compute dq
    // together with the dk/dv reductions
    float* dk_acc = reinterpret_cast<float*>(ws + L.dk_acc);
    float* dv_acc = reinterpret_cast<float*>(ws + L.dv_acc);
    const int64_t kvr = kv_rows_host(*p);
    e = cudaMemsetAsync(dk_acc, 0, sizeof(float) * kvr * p->h_kv * p->d_qk, st);
    if (e == cudaSuccess && dv_acc != dk_acc) e = cudaMemsetAsync(dv_acc, 0, sizeof(float) * kvr * p->h_kv * p->d_v, st);
    note_memset("memset_dkdv_acc", st);
    if (e == cudaSuccess)
      e = fam != SFA_KERNEL_TCGEN05 ? launch_bwd_general(*p, delta, dk_acc, dv_acc, st)
          : L.two_pass              ? launch_bwd_mla(*p, delta, dk_acc, dv_acc, ws + L.mla_pd, st)
                                    : launch_bwd_tok(*p, delta, dk_acc, dv_acc, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "sfa_bwd_dq");
  return SFA_OK;
}

int sfa_bwd_dkdv(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int fam, mode;
  BwdLayout L;
  int rc = bwd_common(p, workspace, workspace_bytes, &fam, &mode, &L);
  if (rc) return rc;
  char* ws = reinterpret_cast<char*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float* delta = reinterpret_cast<const float*>(ws + L.delta);
  cudaError_t e;
  if (mode == SFA_DKV_INVERTED) {
    float* dq_acc = L.fused_dq ? reinterpret_cast<float*>(ws + L.dq_acc) : nullptr;
    e = launch_inverted_index(*p, L, ws, st);
    if (e == cudaSuccess) e = launch_bwd_dkdv_tc(*p, L, ws, delta, dq_acc, st);
    if (e == cudaSuccess && L.nranges > 1) e = launch_reduce_dkdv_ranges(*p, L, ws, st);
    if (e == cudaSuccess && dq_acc) e = launch_convert_dq(*p, dq_acc, st);
  } else {
    float* dk_acc = reinterpret_cast<float*>(ws + L.dk_acc);
    float* dv_acc = reinterpret_cast<float*>(ws + L.dv_acc);
    e = cudaSuccess;
    if (fam == SFA_KERNEL_TCGEN05 && p->block_size != 1) {
      // dq came from the tensor-core kernel; the atomic pass adds dk/dv only
      const int64_t kvr = kv_rows_host(*p);
      e = cudaMemsetAsync(dk_acc, 0, sizeof(float) * kvr * p->h_kv * p->d_qk, st);
      if (e == cudaSuccess && dv_acc != dk_acc)
        e = cudaMemsetAsync(dv_acc, 0, sizeof(float) * kvr * p->h_kv * p->d_v, st);
      note_memset("memset_dkdv_acc", st);
      SfaParams q = *p;
      q.dq = nullptr;
      if (e == cudaSuccess) e = launch_bwd_general(q, delta, dk_acc, dv_acc, st);
    }
    // else: the accumulators were filled by sfa_bwd_dq's fused pass
    if (e == cudaSuccess) e = launch_convert_dkdv(*p, dk_acc, dv_acc, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "sfa_bwd_dkdv");
  return SFA_OK;
}

int sfa_bwd(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = sfa_bwd_preprocess(p, workspace, workspace_bytes, stream);
  if (rc) return rc;
  rc = sfa_bwd_dq(p, workspace, workspace_bytes, stream);
  if (rc) return rc;
  return sfa_bwd_dkdv(p, workspace, workspace_bytes, stream);
}

int sfa_build_inverted_index(const SfaParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate(p, true);
  if (rc) return rc;
  BwdLayout L = bwd_layout(*p, SFA_KERNEL_TCGEN05, SFA_DKV_INVERTED, SFA_DQ_SEPARATE);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(SFA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(L.total) + " bytes");
  cudaError_t e = launch_inverted_index(*p, L, reinterpret_cast<char*>(workspace),
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sfa_build_inverted_index");
  return SFA_OK;
}

int sfa_inverted_index_layout(const SfaParams* p, size_t* offsets_off, size_t* entries_off, int32_t* nblk,
                              int32_t* units) {
  int rc = validate(p, true);
  if (rc) return rc;
  BwdLayout L = bwd_layout(*p, SFA_KERNEL_TCGEN05, SFA_DKV_INVERTED, SFA_DQ_SEPARATE);
  if (offsets_off) *offsets_off = L.inv_offsets;
  if (entries_off) *entries_off = L.inv_entries;
  if (nblk) *nblk = L.nblk;
  if (units) *units = L.units;
  return SFA_OK;
}

int sfa_device_status(void* stream, int32_t* status) {
  int32_t* ptr = device_status_ptr();
  if (!ptr || !status) return fail(SFA_ERR_CUDA, "device status word unavailable");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, ptr, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "sfa_device_status");
  return SFA_OK;
}

int sfa_selftest_wait_timeout(void* stream, uint32_t limit_us) {
  int32_t* ptr = device_status_ptr();
  if (!ptr) return fail(SFA_ERR_CUDA, "device status word unavailable");
  if (limit_us == 0 || limit_us > 1000000u) return fail(SFA_ERR_INVALID_ARGUMENT, "limit_us must be in [1, 1000000]");
  cudaError_t e = launch_wait_probe(limit_us, ptr, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sfa_selftest_wait_timeout");
  return SFA_OK;
}

int sfa_launch_trace(void* const* events, int n_events) {
  if (events != nullptr && n_events <= 0) return fail(SFA_ERR_INVALID_ARGUMENT, "n_events must be positive");
  g_trace.events = events;
  g_trace.n = events ? n_events : 0;
  g_trace.count = 0;
  return SFA_OK;
}

int sfa_launch_trace_count(void) { return g_trace.count; }

const char* sfa_launch_trace_name(int i) {
  if (i < 0 || i >= g_trace.count || i >= 64 || !g_trace.names[i]) return "";
  return g_trace.names[i];
}

int sfa_reset_device_status(void* stream) {
  int32_t* ptr = device_status_ptr();
  if (!ptr) return fail(SFA_ERR_CUDA, "device status word unavailable");
  cudaError_t e = cudaMemsetAsync(ptr, 0, sizeof(int32_t), reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "sfa_reset_device_status");
  return SFA_OK;
}

}  // extern "C"
