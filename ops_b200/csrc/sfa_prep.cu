// sfa_prep.cu — backward preprocessing and bookkeeping kernels (CUDA cores,
// HBM-bound):
//   * delta = rowsum(o * dO) per (row, head) in fp32 plus per-CTA partial
//     dsink sums, reduced in a fixed order (deterministic).  Replaces the
//     reference's `_get_delta_split` (SFA.py:590-610), which both backward
//     kernels recompute, and its dsink atomics (SFA.py:964-970).
//   * fp32 dk/dv accumulators -> bf16 outputs (atomic dk/dv path).
//   * the block->query inverted index used by the key-centric dk/dv pass:
//     count -> exclusive scan -> fill, deterministic (no atomics on positions).
#include <type_traits>

#include "sfa_common.cuh"
#include "sfa_internal.h"

namespace sfa {

// ---------------------------------------------------------------------------
// delta + dsink partials
// ---------------------------------------------------------------------------
constexpr int kPreThreads = 256;

__global__ void __launch_bounds__(kPreThreads)
preprocess_kernel(SfaParams p, float* __restrict__ delta, float* __restrict__ dsink_part) {
  extern __shared__ float sdelta[];  // [kPreRows][h_q]
  const int rows = num_rows(p);
  const int row0 = blockIdx.x * kPreRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = kPreThreads / 32;
  const int Dv = p.d_v;
  for (int pr = warp; pr < kPreRows * p.h_q; pr += nw) {
    int rl = pr / p.h_q, h = pr - rl * p.h_q;
    int row = row0 + rl;
    float acc = 0.f;
    if (row < rows) {
      Row r = row_info(p, row);
      const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(p.o) + r.b * p.o_sb + r.tq * p.o_st + (int64_t)h * p.o_sh;
      const __nv_bfloat16* dO = reinterpret_cast<const __nv_bfloat16*>(p.dout) + r.b * p.do_sb + r.tq * p.do_st + (int64_t)h * p.do_sh;
      if ((Dv & 1) == 0) {
        const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(o);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(dO);
        for (int d = lane; d < Dv / 2; d += 32) {
          float2 a = __bfloat1622float2(o2[d]);
          float2 b = __bfloat1622float2(d2[d]);
          acc = fmaf(a.x, b.x, acc);
          acc = fmaf(a.y, b.y, acc);
        }
      } else {
        for (int d = lane; d < Dv; d += 32) acc = fmaf(bf2f(o[d]), bf2f(dO[d]), acc);
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
      if (lane == 0) delta[(int64_t)row * p.h_q + h] = acc;
    }
    if (lane == 0) sdelta[pr] = acc;
  }
  __syncthreads();
  if (dsink_part == nullptr) return;
  for (int h = threadIdx.x; h < p.h_q; h += kPreThreads) {
    float sink2 = __ldg(p.attn_sink + h) * kLog2e;
    float acc = 0.f;
    for (int rl = 0; rl < kPreRows; ++rl) {
      int row = row0 + rl;
      if (row >= rows) break;
      Row r = row_info(p, row);
      float lse = p.lse[r.b * p.l_sb + r.tq * p.l_st + (int64_t)h * p.l_sh];
      if (lse == -INFINITY) continue;
      acc -= exp2f(sink2 - lse * kLog2e) * sdelta[rl * p.h_q + h];
    }
    dsink_part[(int64_t)blockIdx.x * p.h_q + h] = acc;
  }
}

// The same delta with 16-byte loads: 16 lanes per (row, head), each lane 8
// consecutive elements per step (d_v % 8 == 0, 16-byte aligned rows and
// strides), two (row, head) pairs per warp, and each half-warp loads four
// pairs before reducing any (one pair's two loads per lane leave too little
// in flight to cover the memory latency).  kDv = 64 / 128: one 16-byte chunk
// per lane; kDv = 0: any multiple of 8.  The dsink partials follow as above.
static_assert(kPreRows % (kPreThreads / 16) == 0, "a CTA's (row, head) pairs must split evenly over its half-warps");

template <int kDv>
__global__ void __launch_bounds__(kPreThreads)
preprocess_vec_kernel(SfaParams p, float* __restrict__ delta, float* __restrict__ dsink_part) {
  extern __shared__ float sdelta[];  // [kPreRows][h_q]
  constexpr int kU = 4;   // (row, head) pairs in flight per half-warp (8 measured slower)
  const int rows = num_rows(p);
  const int row0 = blockIdx.x * kPreRows;
  const int hw = threadIdx.x >> 4, l16 = threadIdx.x & 15;   // half-warp = one (row, head)
  const int nhw = kPreThreads / 16;
  const int Dv = kDv ? kDv : p.d_v;
  const int total = kPreRows * p.h_q;   // a multiple of nhw: both half-warps of a warp loop alike
  auto dot8 = [](const uint4& a, const uint4& b, float acc) {
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[k]));
      const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bv[k]));
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
    return acc;
  };
  for (int pr0 = hw; pr0 < total; pr0 += nhw * kU) {
    float acc[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int pr = pr0 + u * nhw;
      const int rl = pr / p.h_q, h = pr - rl * p.h_q;
      const int row = row0 + rl;
      acc[u] = 0.f;
      if (pr < total && row < rows) {
        const Row r = row_info(p, row);
        const uint4* o = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.o) + r.b * p.o_sb +
                                                        r.tq * p.o_st + (int64_t)h * p.o_sh);
        const uint4* dO = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.dout) +
                                                         r.b * p.do_sb + r.tq * p.do_st + (int64_t)h * p.do_sh);
        if (kDv) {
          if (l16 < kDv / 8) acc[u] = dot8(__ldg(o + l16), __ldg(dO + l16), 0.f);
        } else {
          for (int c = l16; c < Dv / 8; c += 16) acc[u] = dot8(__ldg(o + c), __ldg(dO + c), acc[u]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
#pragma unroll
      for (int off = 8; off; off >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);
    }
    if (l16 == 0) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int pr = pr0 + u * nhw;
        if (pr < total) {
          const int rl = pr / p.h_q, h = pr - rl * p.h_q;
          if (row0 + rl < rows) delta[(int64_t)(row0 + rl) * p.h_q + h] = acc[u];
          sdelta[pr] = acc[u];
        }
      }
    }
  }
  __syncthreads();
  if (dsink_part == nullptr) return;
  for (int h = threadIdx.x; h < p.h_q; h += kPreThreads) {
    float sink2 = __ldg(p.attn_sink + h) * kLog2e;
    float acc = 0.f;
    for (int rl = 0; rl < kPreRows; ++rl) {
      int row = row0 + rl;
      if (row >= rows) break;
      Row r = row_info(p, row);
      float lse = p.lse[r.b * p.l_sb + r.tq * p.l_st + (int64_t)h * p.l_sh];
      if (lse == -INFINITY) continue;
      acc -= exp2f(sink2 - lse * kLog2e) * sdelta[rl * p.h_q + h];
    }
    dsink_part[(int64_t)blockIdx.x * p.h_q + h] = acc;
  }
}

__global__ void dsink_reduce_kernel(const float* __restrict__ part, int nparts, int hq, float* __restrict__ dsink) {
  // one warp per head, fixed-order pairwise tree over lanes: deterministic
  int h = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (h >= hq) return;
  float acc = 0.f;
  for (int i = lane; i < nparts; i += 32) acc += part[(int64_t)i * hq + h];
#pragma unroll
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) dsink[h] = acc;
}

cudaError_t launch_preprocess(const SfaParams& p, float* delta, float* dsink_part, int pre_ctas, cudaStream_t st) {
  if (pre_ctas == 0) {
    if (p.dsink) return cudaMemsetAsync(p.dsink, 0, sizeof(float) * p.h_q, st);
    return cudaSuccess;
  }
  size_t smem = sizeof(float) * kPreRows * p.h_q;
  cudaError_t e = cudaFuncSetAttribute(preprocess_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  float* part = (p.dsink && p.attn_sink) ? dsink_part : nullptr;
  const bool vec = p.d_v % 8 == 0 && reinterpret_cast<uintptr_t>(p.o) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(p.dout) % 16 == 0 && p.o_sb % 8 == 0 && p.o_st % 8 == 0 &&
                   p.o_sh % 8 == 0 && p.do_sb % 8 == 0 && p.do_st % 8 == 0 && p.do_sh % 8 == 0;
  if (vec) {
    auto kern = p.d_v == 128 ? preprocess_vec_kernel<128> : p.d_v == 64 ? preprocess_vec_kernel<64>
                                                                       : preprocess_vec_kernel<0>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<pre_ctas, kPreThreads, smem, st>>>(p, delta, part);
  } else {
    preprocess_kernel<<<pre_ctas, kPreThreads, smem, st>>>(p, delta, part);
  }
  note_launch("preprocess", st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.dsink) {
    if (!p.attn_sink) return cudaMemsetAsync(p.dsink, 0, sizeof(float) * p.h_q, st);
    dsink_reduce_kernel<<<(p.h_q + 7) / 8, 256, 0, st>>>(part, pre_ctas, p.h_q, p.dsink);
    note_launch("dsink_reduce", st);
    e = cudaGetLastError();
  }
  return e;
}

// ---------------------------------------------------------------------------
// fp32 accumulators -> bf16 dk / dv (or dk := dk + dv when they alias)
// ---------------------------------------------------------------------------
__global__ void convert_kernel(SfaParams p, const float* __restrict__ acc, int D, int64_t sb, int64_t st,
                               int64_t sh, __nv_bfloat16* __restrict__ out, const float* __restrict__ acc2, int D2) {
  int64_t n = (p.cu_seqlens_q == nullptr ? (int64_t)p.batch * p.kv_len : (int64_t)p.total_kv) * p.h_kv * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int d = (int)(i % D);
    int64_t rest = i / D;
    int hk = (int)(rest % p.h_kv);
    int64_t kr = rest / p.h_kv;
    int64_t b = 0, t = kr;
    if (p.cu_seqlens_q == nullptr) { b = kr / p.kv_len; t = kr - b * p.kv_len; }
    float v = acc[i];
    if (acc2 && d < D2) v += acc2[rest * D2 + d];   // dv into the leading D2 dims of a shared kv
    out[b * sb + t * st + hk * sh + d] = f2bf(v);
  }
}

cudaError_t launch_convert_dkdv(const SfaParams& p, const float* dk_acc, const float* dv_acc, cudaStream_t st) {
  int sms = device_sm_count();
  int grid = sms * 8;
  bool shared_kv = (p.dk == p.dv);
  convert_kernel<<<grid, 256, 0, st>>>(p, dk_acc, p.d_qk, p.dk_sb, p.dk_st, p.dk_sh,
                                       reinterpret_cast<__nv_bfloat16*>(p.dk),
                                       (shared_kv && dv_acc != dk_acc) ? dv_acc : nullptr, p.d_v);
  note_launch("convert_dk", st);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || shared_kv) return e;
  convert_kernel<<<grid, 256, 0, st>>>(p, dv_acc, p.d_v, p.dv_sb, p.dv_st, p.dv_sh,
                                       reinterpret_cast<__nv_bfloat16*>(p.dv), nullptr, 0);
  note_launch("convert_dv", st);
  return cudaGetLastError();
}

// dk/dv of one (unit, block) from the key-centric pass's row-range partials
// (fp32 [range][dK|dV][key][dim]); only ranges whose list part is non-empty
// wrote a partial, and they are added in range order — deterministic.
__global__ void reduce_dkdv_ranges_kernel(SfaParams p, const float* __restrict__ part,
                                          const int32_t* __restrict__ starts, const int32_t* __restrict__ offsets,
                                          int nblk, int nsub, int sub_per_range, int nranges) {
  __shared__ int have[64];
  const int ue = blockIdx.x;
  const int u = ue / nblk, e = ue - u * nblk;
  const int seq = u / p.h_kv, hk = u - seq * p.h_kv;
  int kv0 = 0, kv_len = p.kv_len, b = seq;
  if (p.cu_seqlens_q != nullptr) {
    kv0 = __ldg(p.cu_seqlens_k + seq);
    kv_len = __ldg(p.cu_seqlens_k + seq + 1) - kv0;
    b = 0;
  }
  if (e * 64 >= kv_len) return;
  for (int r = threadIdx.x; r < nranges; r += blockDim.x) {
    const int64_t sb = (int64_t)ue * nsub;
    const int s0 = r * sub_per_range, s1 = s0 + sub_per_range;
    const int end = s1 < nsub ? starts[sb + s1] : offsets[ue + 1];
    have[r] = end > starts[sb + s0];
  }
  __syncthreads();
  const int D = p.d_qk;
  const bool shared_kv = p.dk == p.dv;
  // four consecutive dims per thread (d_qk % 4 == 0): 16-byte loads of the partials
  for (int i4 = threadIdx.x; i4 < 16 * D; i4 += blockDim.x) {
    const int i = i4 * 4;
    const int key = i / D, dim = i - key * D;
    if (e * 64 + key >= kv_len) continue;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
    // ranges in order, four loads in flight at a time
    for (int r0 = 0; r0 < nranges; r0 += 4) {
      float4 a[4], c[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = r0 + k;
        const bool use = r < nranges && have[r];
        const float* pr = part + ((int64_t)ue * nranges + (use ? r : 0)) * (2 * 64 * D);
        a[k] = use ? *reinterpret_cast<const float4*>(pr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        c[k] = use ? *reinterpret_cast<const float4*>(pr + 64 * D + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        sk.x += a[k].x; sk.y += a[k].y; sk.z += a[k].z; sk.w += a[k].w;
        sv.x += c[k].x; sv.y += c[k].y; sv.z += c[k].z; sv.w += c[k].w;
      }
    }
    const int64_t t = (int64_t)kv0 + e * 64 + key;
    __nv_bfloat16* dk = reinterpret_cast<__nv_bfloat16*>(p.dk) + b * p.dk_sb + t * p.dk_st + hk * p.dk_sh + dim;
    const float k4[4] = {sk.x, sk.y, sk.z, sk.w}, v4[4] = {sv.x, sv.y, sv.z, sv.w};
    if (shared_kv) {
#pragma unroll
      for (int q = 0; q < 4; ++q) dk[q] = f2bf(k4[q] * p.scale + v4[q]);
    } else {
      __nv_bfloat16* dv = reinterpret_cast<__nv_bfloat16*>(p.dv) + b * p.dv_sb + t * p.dv_st + hk * p.dv_sh + dim;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        dk[q] = f2bf(k4[q] * p.scale);
        dv[q] = f2bf(v4[q]);
      }
    }
  }
}

cudaError_t launch_reduce_dkdv_ranges(const SfaParams& p, const BwdLayout& L, const char* ws, cudaStream_t st) {
  if (L.nranges > 64) return cudaErrorInvalidValue;
  const int nlists = L.units * L.nblk;
  if (nlists == 0) return cudaSuccess;
  reduce_dkdv_ranges_kernel<<<nlists, 256, 0, st>>>(
      p, reinterpret_cast<const float*>(ws + L.dkv_part), reinterpret_cast<const int32_t*>(ws + L.inv_cursor),
      reinterpret_cast<const int32_t*>(ws + L.inv_offsets), L.nblk, L.inv_nsub, L.sub_per_range, L.nranges);
  note_launch("reduce_dkdv_ranges", st);
  return cudaGetLastError();
}

// dq = bf16(scale * acc) for the fused dQ: acc is fp32 [rows][h_q][d_qk].
// kVec: eight consecutive dims per thread (d_qk % 8 == 0), one 16-byte store
// (16-byte aligned dq rows); otherwise four dims and element stores.
// kIdx32: the element-group count fits 32 bits, so the index arithmetic (three
// divisions per group) stays in 32-bit integers; 64-bit divisions otherwise
// cost more issue slots than the group's 48 bytes of traffic leave room for.
template <bool kVec, bool kIdx32>
__global__ void convert_dq_kernel(SfaParams p, const float* __restrict__ acc) {
  constexpr int kE = kVec ? 8 : 4;
  using Idx = typename std::conditional<kIdx32, uint32_t, int64_t>::type;
  const int D = p.d_qk;
  const int64_t rows = p.cu_seqlens_q == nullptr ? (int64_t)p.batch * p.q_len : (int64_t)p.total_q;
  const Idx n = (Idx)(rows * p.h_q * (D / kE));
  const Idx groups = (Idx)(D / kE), hq = (Idx)p.h_q;
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(p.dq);
  for (Idx i = (Idx)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (Idx)gridDim.x * blockDim.x) {
    const int d = (int)(i % groups) * kE;
    const Idx rh = i / groups;
    const int h = (int)(rh % hq);
    const int row = (int)(rh / hq);
    int64_t b = 0, t = row;
    if (p.cu_seqlens_q == nullptr) { b = row / p.q_len; t = row - b * p.q_len; }
    const float4* src = reinterpret_cast<const float4*>(acc + rh * D + d);
    __nv_bfloat16* o = dq + b * p.dq_sb + t * p.dq_st + h * p.dq_sh + d;
    const float4 v = __ldg(src);
    if (kVec) {
      const float4 w = __ldg(src + 1);
      uint4 u;
      u.x = pack_bf16x2_rn(v.x * p.scale, v.y * p.scale);
      u.y = pack_bf16x2_rn(v.z * p.scale, v.w * p.scale);
      u.z = pack_bf16x2_rn(w.x * p.scale, w.y * p.scale);
      u.w = pack_bf16x2_rn(w.z * p.scale, w.w * p.scale);
      *reinterpret_cast<uint4*>(o) = u;
    } else {
      o[0] = f2bf(v.x * p.scale);
      o[1] = f2bf(v.y * p.scale);
      o[2] = f2bf(v.z * p.scale);
      o[3] = f2bf(v.w * p.scale);
    }
  }
}

cudaError_t launch_convert_dq(const SfaParams& p, const float* dq_acc, cudaStream_t st) {
  const int grid = device_sm_count() * 8;
  const bool vec = p.d_qk % 8 == 0 && (reinterpret_cast<uintptr_t>(p.dq) % 16 == 0) && p.dq_sb % 8 == 0 &&
                   p.dq_st % 8 == 0 && p.dq_sh % 8 == 0;
  const int64_t rows = p.cu_seqlens_q == nullptr ? (int64_t)p.batch * p.q_len : (int64_t)p.total_q;
  const bool i32 = rows * p.h_q * p.d_qk < ((int64_t)1 << 31);
  if (vec && i32)
    convert_dq_kernel<true, true><<<grid, 256, 0, st>>>(p, dq_acc);
  else if (vec)
    convert_dq_kernel<true, false><<<grid, 256, 0, st>>>(p, dq_acc);
  else if (i32)
    convert_dq_kernel<false, true><<<grid, 256, 0, st>>>(p, dq_acc);
  else
    convert_dq_kernel<false, false><<<grid, 256, 0, st>>>(p, dq_acc);
  note_launch("convert_dq", st);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// inverted index: for unit u = (sequence, kv head) and block e, the query rows
// that selected e.  Order inside a list: (sub-chunk of 32 rows, slot, lane) —
// fixed, so the key-centric pass sums in a reproducible order.
//
// counts layout: [units][nblk][nsub] (flat exclusive scan gives positions)
// ---------------------------------------------------------------------------
constexpr int kInvWarps = 8;
constexpr int kInvRowsPerWarp = 128;   // 4 batches of 32 rows

struct UnitRows {
  int row0;   // first global row of the unit's sequence
  int q_len;
};

__device__ __forceinline__ UnitRows unit_rows(const SfaParams& p, int seq) {
  UnitRows u;
  if (p.cu_seqlens_q == nullptr) {
    u.row0 = seq * p.q_len;
    u.q_len = p.q_len;
  } else {
    u.row0 = __ldg(p.cu_seqlens_q + seq);
    u.q_len = __ldg(p.cu_seqlens_q + seq + 1) - u.row0;
  }
  return u;
}

template <bool kFill>
__global__ void __launch_bounds__(kInvWarps * 32)
inv_pass_kernel(SfaParams p, int nblk, int nsub, int32_t* __restrict__ counts, int32_t* __restrict__ entries) {
  extern __shared__ int32_t scnt[];  // [kInvWarps][nblk]
  const int seq = blockIdx.y / p.h_kv, hk = blockIdx.y - seq * p.h_kv;
  const int unit = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const UnitRows ur = unit_rows(p, seq);
  const int sub = blockIdx.x * kInvWarps + warp;  // sub-chunk of kInvRowsPerWarp rows
  int32_t* cnt = scnt + warp * nblk;
  int32_t* cbase = counts + (int64_t)unit * nblk * nsub + sub;  // stride nsub over blocks
  for (int e = lane; e < nblk; e += 32) cnt[e] = kFill ? cbase[(int64_t)e * nsub] : 0;
  __syncwarp();
  const int t_begin = sub * kInvRowsPerWarp;
  for (int tb = t_begin; tb < t_begin + kInvRowsPerWarp && tb < ur.q_len; tb += 32) {
    int t = tb + lane;
    bool live = t < ur.q_len;
    Row r;
    const int32_t* idx = nullptr;
    if (live) {
      r = row_info(p, ur.row0 + t);
      idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
    }
    for (int s = 0; s < p.topk; ++s) {
      int e = -1;
      if (live) {
        int ev = __ldg(idx + s);
        if (block_valid_keys(ev, p.block_size, r.kv_len, r.pos, p.causal) > 0 && ev < nblk) e = ev;
      }
      unsigned grp = __match_any_sync(0xffffffffu, e);
      int leader = __ffs(grp) - 1;
      if (e >= 0) {
        int rank = __popc(grp & ((1u << lane) - 1u));
        int basepos = 0;
        if (lane == leader) basepos = cnt[e];
        basepos = __shfl_sync(grp, basepos, leader);
        if (kFill) entries[basepos + rank] = ur.row0 + t;
        if (lane == leader) cnt[e] = basepos + __popc(grp);
      }
      __syncwarp();
    }
  }
  __syncwarp();
  if (!kFill)
    for (int e = lane; e < nblk; e += 32) cbase[(int64_t)e * nsub] = cnt[e];
}

// exclusive scan in three launches: tile sums, scan of tile sums, tile scans
constexpr int kScanTile = 2048;
constexpr int kScanThreads = 256;

__global__ void scan_tile_sums(const int32_t* __restrict__ in, int64_t n, int32_t* __restrict__ sums) {
  __shared__ int32_t red[kScanThreads / 32];
  int64_t base = (int64_t)blockIdx.x * kScanTile;
  int acc = 0;
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    int64_t j = base + i;
    if (j < n) acc += in[j];
  }
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kScanThreads / 32; ++w) s += red[w];
    sums[blockIdx.x] = s;
  }
}

__global__ void scan_sums_single(int32_t* __restrict__ sums, int nt, int32_t* __restrict__ total_out) {
  // one CTA; sequential chunks per thread then a block scan of chunk totals
  __shared__ int32_t part[1024];
  int per = (nt + blockDim.x - 1) / blockDim.x;
  int b = threadIdx.x * per, e = min(nt, b + per);
  int s = 0;
  for (int i = b; i < e; ++i) s += sums[i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < (int)blockDim.x; ++i) { int v = part[i]; part[i] = run; run += v; }
    *total_out = run;
  }
  __syncthreads();
  int run = part[threadIdx.x];
  for (int i = b; i < e; ++i) { int v = sums[i]; sums[i] = run; run += v; }
}

__global__ void scan_tiles(int32_t* __restrict__ data, int64_t n, const int32_t* __restrict__ tile_off) {
  __shared__ int32_t wsum[kScanThreads / 32];
  int64_t base = (int64_t)blockIdx.x * kScanTile;
  constexpr int per = kScanTile / kScanThreads;  // 8 consecutive items per thread
  int local[per];
  int s = 0;
  for (int k = 0; k < per; ++k) {
    int64_t j = base + threadIdx.x * per + k;
    local[k] = j < n ? data[j] : 0;
    s += local[k];
  }
  // warp inclusive scan of per-thread sums
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = s;
  for (int off = 1; off < 32; off <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < kScanThreads / 32; ++i) { int v = wsum[i]; wsum[i] = run; run += v; }
  }
  __syncthreads();
  int run = tile_off[blockIdx.x] + wsum[w] + incl - s;
  for (int k = 0; k < per; ++k) {
    int64_t j = base + threadIdx.x * per + k;
    if (j < n) data[j] = run;
    run += local[k];
  }
}

// offsets[u*nblk + e] = scanned[(u*nblk + e)*nsub]; offsets[units*nblk] = total
__global__ void gather_offsets(const int32_t* __restrict__ scanned, int64_t nlists, int nsub,
                               const int32_t* __restrict__ total, int32_t* __restrict__ offsets) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= nlists; i += (int64_t)gridDim.x * blockDim.x)
    offsets[i] = i < nlists ? scanned[i * nsub] : *total;
}

cudaError_t launch_inverted_index(const SfaParams& p, const BwdLayout& L, char* ws, cudaStream_t st) {
  const int nblk = L.nblk;
  const int qmax = p.q_len;
  const int nsub = (qmax + kInvRowsPerWarp - 1) / kInvRowsPerWarp;
  const int ctas_x = (nsub + kInvWarps - 1) / kInvWarps;
  const int nsub_pad = ctas_x * kInvWarps;
  const int64_t ncount = (int64_t)L.units * nblk * nsub_pad;
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.inv_cursor);
  int32_t* entries = reinterpret_cast<int32_t*>(ws + L.inv_entries);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + L.inv_offsets);
  const int64_t ntiles = (ncount + kScanTile - 1) / kScanTile;
  int32_t* tile_sums = counts + ncount;          // [ntiles]
  int32_t* total = tile_sums + ntiles;           // [1]
  size_t smem = sizeof(int32_t) * kInvWarps * nblk;
  cudaError_t e;
  e = cudaFuncSetAttribute(inv_pass_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(inv_pass_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * ncount, st);
  if (e != cudaSuccess) return e;
  dim3 grid(ctas_x, L.units);
  inv_pass_kernel<false><<<grid, kInvWarps * 32, smem, st>>>(p, nblk, nsub_pad, counts, entries);
  note_launch("index_count", st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  scan_tile_sums<<<(unsigned)ntiles, kScanThreads, 0, st>>>(counts, ncount, tile_sums);
  note_launch("index_scan_tiles", st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  scan_sums_single<<<1, 1024, 0, st>>>(tile_sums, (int)ntiles, total);
  note_launch("index_scan_sums", st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  scan_tiles<<<(unsigned)ntiles, kScanThreads, 0, st>>>(counts, ncount, tile_sums);
  note_launch("index_scan_apply", st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int64_t nlists = (int64_t)L.units * nblk;
  const int64_t gblocks = (nlists + 1 + 255) / 256;
  gather_offsets<<<(unsigned)(gblocks < 4096 ? gblocks : 4096), 256, 0, st>>>(
      counts, nlists, nsub_pad, total, offsets);
  note_launch("index_offsets", st);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  inv_pass_kernel<true><<<grid, kInvWarps * 32, smem, st>>>(p, nblk, nsub_pad, counts, entries);
  note_launch("index_fill", st);
  return cudaGetLastError();
}

}  // namespace sfa
