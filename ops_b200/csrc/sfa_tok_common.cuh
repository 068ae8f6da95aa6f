// sfa_tok_common.cuh — building blocks shared by the token-level (block_size 1)
// tensor-core kernels: TMA tile::gather4 row gathers, 32-column TMEM loads and
// stores, and the host-side description of kv rows as one 2-D gather tensor.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "sfa_common.cuh"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"

namespace sfa {
namespace tok {

using tc::smem_u32;

// Four rows (r0..r3) x one 64-dim slab (starting at element col) of a 2-D
// tensor map whose box is {64, 1}: 512 bytes, landing 128B-swizzled at dst.
__device__ __forceinline__ void gather4(void* dst, const CUtensorMap* map, uint64_t* bar, int col, int r0, int r1,
                                        int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit (thread i of the warp: TMEM lane quadrant*32 + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2-D bf16 map for row gathers: dim 0 the head dim (extent d, contiguous),
// dim 1 the gather rows (stride rs elements), 64-dim x 1-row box, 128B swizzle.
inline cudaError_t make_tmap_rows(CUtensorMap* map, const void* base, uint64_t d, uint64_t rows, int64_t rs) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t gdim[2] = {d, rows};
  cuuint64_t gstr[1] = {(cuuint64_t)(rs * 2)};
  cuuint32_t box[2] = {64, 1}, estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstr, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Element stride of one gather row of a [batch, token, head, dim] tensor, or 0
// when batch/token/head do not fold into evenly spaced rows; *rows = count.
inline int64_t gather_rows(const SfaParams& p, int64_t sb, int64_t stt, int64_t sh, int64_t d, int64_t* rows) {
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t nb = vl ? 1 : p.batch, nt = vl ? p.total_kv : p.kv_len, nh = p.h_kv;
  int64_t cand[3];
  int n = 0;
  if (nt > 1) cand[n++] = stt;
  if (nh > 1) cand[n++] = sh;
  if (nb > 1) cand[n++] = sb;
  int64_t rs = d;
  if (n) {
    rs = cand[0];
    for (int i = 1; i < n; ++i) rs = cand[i] < rs ? cand[i] : rs;
  }
  if (rs < d || rs % 8) return 0;
  for (int i = 0; i < n; ++i)
    if (cand[i] <= 0 || cand[i] % rs) return 0;
  const int64_t last = (nb > 1 ? (nb - 1) * sb : 0) + (nt > 1 ? (nt - 1) * stt : 0) + (nh > 1 ? (nh - 1) * sh : 0);
  *rows = last / rs + 1;
  return rs;
}

}  // namespace tok
}  // namespace sfa
