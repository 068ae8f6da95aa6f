// sfa_noalloc.cu — a backward entry point that allocates nothing, for callers
// that cannot call cudaMalloc.
//
// Who needs it: hosts that run under a pre-sized device arena or inside a
// framework that forbids allocation during the step (a serving loop with a
// fixed memory budget, an embedded runtime without a device allocator, a
// plugin called from a host that owns all device memory).  sfa_bwd asks its
// caller for a workspace; these callers have none to give.
//
// How: the backward's scratch (delta, dsink partial sums, the block->query
// inverted index and its counters) lives in one file-scope device array of
// kNoAllocScratchBytes.  Every GPU that loads the library reserves it until the
// process exits.  In host code the array's name is only a host-side stand-in,
// so its device address is taken with cudaGetSymbolAddress once per device
// (with that device current) on the first call made on that device; make that
// first call before any stream capture.  Calls share the array: two calls that
// overlap on the GPU (different streams, or different host threads on one
// device) race on it and must be serialised by the caller.  Everything that
// must start at zero is cleared by the backward's own stages on every call.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "sfa_common.cuh"
#include "sfa_internal.h"

namespace sfa {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;   // 32 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* noalloc_scratch_ptr(cudaError_t* err) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* ptr = nullptr;
    *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    ptrs[dev] = ptr;
  }
  return ptrs[dev];
}

}  // namespace sfa

extern "C" int sfa_bwd_noalloc(const SfaParams* p, void* stream) {
  using namespace sfa;
  size_t need = sfa_bwd_workspace_bytes(p);
  SfaParams sep;
  if (need > kNoAllocScratchBytes && p != nullptr && p->dq_mode == SFA_DQ_AUTO) {
    // the fused dQ's accumulator does not fit: compute dQ in its own pass
    sep = *p;
    sep.dq_mode = SFA_DQ_SEPARATE;
    const size_t need_sep = sfa_bwd_workspace_bytes(&sep);
    if (need_sep != 0 && need_sep <= kNoAllocScratchBytes) {
      p = &sep;
      need = need_sep;
    }
  }
  if (need == 0) {
    // invalid or unsupported parameters (or nothing to stage): sfa_bwd reports
    // the reason before launching anything
    return sfa_bwd(p, nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes)
    return report_error(SFA_ERR_WORKSPACE, "sfa_bwd_noalloc: this problem needs " + std::to_string(need) +
                                               " bytes of scratch, more than the library's static " +
                                               std::to_string(kNoAllocScratchBytes) +
                                               "-byte array; call sfa_bwd with a workspace instead");
  cudaError_t e = cudaSuccess;
  void* ws = noalloc_scratch_ptr(&e);
  if (!ws)
    return report_error(SFA_ERR_CUDA, std::string("sfa_bwd_noalloc: cudaGetSymbolAddress of the scratch array: ") +
                                          cudaGetErrorString(e));
  return sfa_bwd(p, ws, kNoAllocScratchBytes, stream);
}
