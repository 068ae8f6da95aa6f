// sfa_tc_host.h — host helpers for the tensor-core kernels: TMA tensor-map
// encoding through the driver entry point (no libcuda link dependency) and the
// alignment rules a TMA-fed operand must satisfy.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <array>

namespace sfa {

int32_t* device_status_ptr();

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Base 16-byte aligned and every stride (elements of bf16) a multiple of 8.
inline bool tma_compatible(const void* base, int64_t sb, int64_t st, int64_t sh) {
  if (reinterpret_cast<uintptr_t>(base) & 15) return false;
  return (sb % 8 == 0) && (st % 8 == 0) && (sh % 8 == 0);
}

// 4-D bf16 tensor map, innermost dim first; strides in elements for dims 1..3.
// A dim of extent 1 gets a synthetic stride (its value is never used).
// 128-byte swizzle, zero fill outside the tensor.
inline cudaError_t make_tmap_bf16_4d(CUtensorMap* map, const void* base, std::array<uint64_t, 4> dims,
                                     std::array<int64_t, 3> strides_el, std::array<uint32_t, 4> box,
                                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t gdim[4];
  cuuint64_t gstr[3];
  cuuint32_t bdim[4], estr[4] = {1, 1, 1, 1};
  uint64_t prev = dims[0] * 2;
  for (int i = 0; i < 4; ++i) {
    gdim[i] = dims[i] ? dims[i] : 1;
    bdim[i] = box[i];
  }
  for (int i = 0; i < 3; ++i) {
    int64_t sbytes = strides_el[i] * 2;
    if (gdim[i + 1] == 1 || sbytes <= 0) sbytes = (int64_t)((prev + 15) / 16 * 16);
    if (sbytes % 16) return cudaErrorInvalidValue;
    gstr[i] = (cuuint64_t)sbytes;
    prev = (uint64_t)sbytes * gdim[i + 1];
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), gdim, gstr, bdim, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace sfa
