// sfa_general.cu — CUDA-core SFA kernels for every shape the tensor-core
// family does not cover (any head dims up to the shared-memory limit, any
// group size, any block size including token-level top-k, varlen).
//
// Forward: one CTA per (query row, kv head, group of up to 16 query heads).
// It walks the S*block_size expanded key slots in chunks of kKC keys, stages the
// gathered K/V rows in shared memory (fp32), and runs an online base-2 softmax —
// the arithmetic of `_inner_fwd` (SFA.py:309-480) without the Ascend
// cube/vector workspace round trips.
//
// Backward: the same decomposition recomputes scores, forms
// p = exp2(s*log2e - lse2) and ds = p*(dO.v - delta), accumulates dq in shared
// memory and scatters dk/dv through fp32 atomics — `_inner_dq`
// (SFA.py:613-716) and `_inner_dkv` (SFA.py:719-853) fused into one pass.
#include "sfa_common.cuh"
#include "sfa_internal.h"

#include <cuda_fp8.h>

namespace sfa {

constexpr int kGenThreads = 128;
constexpr int kKC = 16;

// one e4m3 byte as float (through the CUDA fp8 conversion)
static __device__ __forceinline__ float fp8_e4m3_to_float(uint8_t x) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)x, __NV_E4M3);
  return __half2float(__half(h));
}

static __device__ __forceinline__ const __nv_bfloat16* bfp(const void* p) {
  return reinterpret_cast<const __nv_bfloat16*>(p);
}

__device__ __forceinline__ int slot_key(const int32_t* idx, int lp, int bs, int topk, const Row& r, int causal) {
  if (lp >= topk * bs) return -1;
  int s = lp / bs, j = lp - s * bs;
  int e = __ldg(idx + s);
  int n = block_valid_keys(e, bs, r.kv_len, r.pos, causal);
  return j < n ? e * bs + j : -1;
}

__global__ void __launch_bounds__(kGenThreads) fwd_general_kernel(SfaParams p, int HG) {
  extern __shared__ float sm[];
  const int tid = threadIdx.x;
  const int row = blockIdx.x, hk = blockIdx.y, g0 = blockIdx.z * HG;
  const int G = p.h_q / p.h_kv;
  const int nh = min(HG, G - g0);
  const int Dq = p.d_qk, Dv = p.d_v;
  const Row r = row_info(p, row);
  const float qscale = p.scale * kLog2e;

  float* qs = sm;                       // [HG][Dq]
  float* ks = qs + HG * Dq;             // [KC][Dq]
  float* vs = ks + kKC * Dq;            // [KC][Dv]
  float* os = vs + kKC * Dv;            // [HG][Dv]
  float* sc = os + HG * Dv;             // [HG][KC]
  float* mrow = sc + HG * kKC;
  float* lrow = mrow + HG;
  float* arow = lrow + HG;
  int* keyid = reinterpret_cast<int*>(arow + HG);

  const __nv_bfloat16* q = bfp(p.q) + r.b * p.q_sb + r.tq * p.q_st + (int64_t)(hk * G + g0) * p.q_sh;
  for (int i = tid; i < nh * Dq; i += kGenThreads)
    qs[i] = bf2f(q[(i / Dq) * p.q_sh + i % Dq]) * qscale;
  for (int i = tid; i < nh * Dv; i += kGenThreads) os[i] = 0.f;
  if (tid < nh) { mrow[tid] = -INFINITY; lrow[tid] = 0.f; }

  const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
  const __nv_bfloat16* kb = bfp(p.k) + r.b * p.k_sb + (int64_t)hk * p.k_sh;
  const __nv_bfloat16* vb = bfp(p.v) + r.b * p.v_sb + (int64_t)hk * p.v_sh;
  const int L = p.topk * p.block_size;
  __syncthreads();

  for (int base = 0; base < L; base += kKC) {
    // keyid: the kv row of each slot's key (kv0 + key, or its row in a paged cache), -1 if invalid
    if (tid < kKC) {
      const int key = slot_key(idx, base + tid, p.block_size, p.topk, r, p.causal);
      keyid[tid] = key >= 0 ? (int)kv_row(p, r, key) : -1;
    }
    __syncthreads();
    int any = __syncthreads_or(tid < kKC && keyid[tid] >= 0);
    if (!any) continue;
    if (p.kv_dtype == SFA_KV_FP8_E4M3) {
      // e4m3 rows times their row scale (v is k's leading dims)
      const uint8_t* k8 = static_cast<const uint8_t*>(p.k) + r.b * p.k_sb + (int64_t)hk * p.k_sh;
      const float* sc = p.kv_scale + r.b * p.ks_sb + (int64_t)hk * p.ks_sh;
      for (int i = tid; i < kKC * Dq; i += kGenThreads) {
        int kk = i / Dq, d = i - kk * Dq, key = keyid[kk];
        ks[i] = key >= 0 ? fp8_e4m3_to_float(k8[(int64_t)key * p.k_st + d]) * __ldg(sc + (int64_t)key * p.ks_st) : 0.f;
      }
      for (int i = tid; i < kKC * Dv; i += kGenThreads) {
        int kk = i / Dv, d = i - kk * Dv, key = keyid[kk];
        vs[i] = key >= 0 ? fp8_e4m3_to_float(k8[(int64_t)key * p.k_st + d]) * __ldg(sc + (int64_t)key * p.ks_st) : 0.f;
      }
    } else {
      for (int i = tid; i < kKC * Dq; i += kGenThreads) {
        int kk = i / Dq, d = i - kk * Dq, key = keyid[kk];
        ks[i] = key >= 0 ? bf2f(kb[(int64_t)key * p.k_st + d]) : 0.f;
      }
      for (int i = tid; i < kKC * Dv; i += kGenThreads) {
        int kk = i / Dv, d = i - kk * Dv, key = keyid[kk];
        vs[i] = key >= 0 ? bf2f(vb[(int64_t)key * p.v_st + d]) : 0.f;
      }
    }
    __syncthreads();
    for (int i = tid; i < nh * kKC; i += kGenThreads) {
      int h = i / kKC, kk = i - h * kKC;
      float acc = -INFINITY;
      if (keyid[kk] >= 0) {
        acc = 0.f;
        const float* qh = qs + h * Dq;
        const float* kr = ks + kk * Dq;
        for (int d = 0; d < Dq; ++d) acc = fmaf(qh[d], kr[d], acc);
      }
      sc[i] = acc;
    }
    __syncthreads();
    if (tid < nh) {
      float* srow = sc + tid * kKC;
      float mold = mrow[tid], mx = mold;
      for (int kk = 0; kk < kKC; ++kk) mx = fmaxf(mx, srow[kk]);
      float alpha = (mx == -INFINITY) ? 1.f : exp2f(mold - mx);
      float lsum = 0.f;
      for (int kk = 0; kk < kKC; ++kk) {
        float pv = (srow[kk] == -INFINITY) ? 0.f : exp2f(srow[kk] - mx);
        lsum += pv;
        // the PV sum takes p at bf16 precision (the tensor-core kernels' operand),
        // or as the reference rounds it (fp16, then bf16) under SFA_COMPAT_REFERENCE_P
        srow[kk] = (p.compat & SFA_COMPAT_REFERENCE_P) ? bf2f(f2bf(ref_p(pv))) : pv;
      }
      lrow[tid] = lrow[tid] * alpha + lsum;
      mrow[tid] = mx;
      arow[tid] = alpha;
    }
    __syncthreads();
    for (int i = tid; i < nh * Dv; i += kGenThreads) {
      int h = i / Dv, d = i - h * Dv;
      float acc = os[i] * arow[h];
      const float* pr = sc + h * kKC;
      for (int kk = 0; kk < kKC; ++kk) acc = fmaf(pr[kk], vs[kk * Dv + d], acc);
      os[i] = acc;
    }
    __syncthreads();
  }

  if (tid < nh) {
    int h = hk * G + g0 + tid;
    float m = mrow[tid], l = lrow[tid];
    float s2 = p.attn_sink ? __ldg(p.attn_sink + h) * kLog2e : -INFINITY;
    float M = fmaxf(m, s2);
    float lse, so;
    if (M == -INFINITY) {
      lse = -INFINITY;
      so = 0.f;
    } else {
      float lt = l * exp2f(m - M) + exp2f(s2 - M);
      lse = (M + log2f(lt)) * kLn2;
      so = exp2f(m - M) / lt;
    }
    arow[tid] = so;
    p.lse[r.b * p.l_sb + r.tq * p.l_st + (int64_t)h * p.l_sh] = lse;
  }
  __syncthreads();
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.o) + r.b * p.o_sb + r.tq * p.o_st + (int64_t)(hk * G + g0) * p.o_sh;
  for (int i = tid; i < nh * Dv; i += kGenThreads) {
    int h = i / Dv, d = i - h * Dv;
    o[h * p.o_sh + d] = f2bf(os[i] * arow[h]);
  }
}

size_t fwd_general_smem(const SfaParams& p, int HG) {
  return sizeof(float) * ((size_t)HG * p.d_qk + (size_t)kKC * p.d_qk + (size_t)kKC * p.d_v + (size_t)HG * p.d_v +
                          (size_t)HG * kKC + 3 * HG) + sizeof(int) * kKC;
}

// ---------------------------------------------------------------------------
// backward (general): dq direct, dk/dv through fp32 atomics into `acc`
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kGenThreads)
bwd_general_kernel(SfaParams p, int HG, const float* __restrict__ delta, float* __restrict__ dk_acc,
                   float* __restrict__ dv_acc) {
  extern __shared__ float sm[];
  const int tid = threadIdx.x;
  const int row = blockIdx.x, hk = blockIdx.y, g0 = blockIdx.z * HG;
  const int G = p.h_q / p.h_kv;
  const int nh = min(HG, G - g0);
  const int Dq = p.d_qk, Dv = p.d_v;
  const Row r = row_info(p, row);
  const float qscale = p.scale * kLog2e;

  float* qs = sm;                       // [HG][Dq] raw q
  float* dos = qs + HG * Dq;            // [HG][Dv]
  float* ks = dos + HG * Dv;            // [KC][Dq]
  float* vs = ks + kKC * Dq;            // [KC][Dv]
  float* dqs = vs + kKC * Dv;           // [HG][Dq]
  float* ps = dqs + HG * Dq;            // [HG][KC]
  float* dss = ps + HG * kKC;           // [HG][KC]
  float* lse2 = dss + HG * kKC;         // [HG]
  float* dl = lse2 + HG;                // [HG]
  int* keyid = reinterpret_cast<int*>(dl + HG);

  const int h0 = hk * G + g0;
  const __nv_bfloat16* q = bfp(p.q) + r.b * p.q_sb + r.tq * p.q_st + (int64_t)h0 * p.q_sh;
  const __nv_bfloat16* dO = bfp(p.dout) + r.b * p.do_sb + r.tq * p.do_st + (int64_t)h0 * p.do_sh;
  for (int i = tid; i < nh * Dq; i += kGenThreads) {
    qs[i] = bf2f(q[(i / Dq) * p.q_sh + i % Dq]);
    dqs[i] = 0.f;
  }
  for (int i = tid; i < nh * Dv; i += kGenThreads) dos[i] = bf2f(dO[(i / Dv) * p.do_sh + i % Dv]);
  if (tid < nh) {
    lse2[tid] = p.lse[r.b * p.l_sb + r.tq * p.l_st + (int64_t)(h0 + tid) * p.l_sh] * kLog2e;
    dl[tid] = delta[(int64_t)row * p.h_q + h0 + tid];
  }
  const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
  const __nv_bfloat16* kb = bfp(p.k) + r.b * p.k_sb + (int64_t)hk * p.k_sh;
  const __nv_bfloat16* vb = bfp(p.v) + r.b * p.v_sb + (int64_t)hk * p.v_sh;
  const int64_t acc_row0 = (p.cu_seqlens_q == nullptr) ? (int64_t)r.b * p.kv_len : r.kv0;
  const int L = p.topk * p.block_size;
  __syncthreads();

  for (int base = 0; base < L; base += kKC) {
    if (tid < kKC) keyid[tid] = slot_key(idx, base + tid, p.block_size, p.topk, r, p.causal);
    __syncthreads();
    int any = __syncthreads_or(tid < kKC && keyid[tid] >= 0);
    if (!any) continue;
    for (int i = tid; i < kKC * Dq; i += kGenThreads) {
      int kk = i / Dq, d = i - kk * Dq, key = keyid[kk];
      ks[i] = key >= 0 ? bf2f(kb[(r.kv0 + key) * p.k_st + d]) : 0.f;
    }
    for (int i = tid; i < kKC * Dv; i += kGenThreads) {
      int kk = i / Dv, d = i - kk * Dv, key = keyid[kk];
      vs[i] = key >= 0 ? bf2f(vb[(r.kv0 + key) * p.v_st + d]) : 0.f;
    }
    __syncthreads();
    for (int i = tid; i < nh * kKC; i += kGenThreads) {
      int h = i / kKC, kk = i - h * kKC;
      float pv = 0.f, dsv = 0.f;
      if (keyid[kk] >= 0 && lse2[h] != -INFINITY) {
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < Dq; ++d) s = fmaf(qs[h * Dq + d], ks[kk * Dq + d], s);
        for (int d = 0; d < Dv; ++d) dp = fmaf(dos[h * Dv + d], vs[kk * Dv + d], dp);
        pv = exp2f(s * qscale - lse2[h]);
        dsv = pv * (dp - dl[h]);
      }
      ps[i] = pv;
      dss[i] = dsv;
    }
    __syncthreads();
    if (p.dq != nullptr) {
      for (int i = tid; i < nh * Dq; i += kGenThreads) {
        int h = i / Dq, d = i - h * Dq;
        float acc = dqs[i];
        for (int kk = 0; kk < kKC; ++kk) acc = fmaf(dss[h * kKC + kk], ks[kk * Dq + d], acc);
        dqs[i] = acc;
      }
    }
    for (int i = tid; i < kKC * Dq; i += kGenThreads) {
      int kk = i / Dq, d = i - kk * Dq, key = keyid[kk];
      if (key < 0) continue;
      float acc = 0.f;
      for (int h = 0; h < nh; ++h) acc = fmaf(dss[h * kKC + kk], qs[h * Dq + d], acc);
      atomicAdd(dk_acc + ((acc_row0 + key) * p.h_kv + hk) * Dq + d, acc * p.scale);
    }
    for (int i = tid; i < kKC * Dv; i += kGenThreads) {
      int kk = i / Dv, d = i - kk * Dv, key = keyid[kk];
      if (key < 0) continue;
      float acc = 0.f;
      for (int h = 0; h < nh; ++h) acc = fmaf(ps[h * kKC + kk], dos[h * Dv + d], acc);
      atomicAdd(dv_acc + ((acc_row0 + key) * p.h_kv + hk) * Dv + d, acc);
    }
    __syncthreads();
  }
  if (p.dq == nullptr) return;  // dq computed by another kernel; only the dk/dv atomics here
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(p.dq) + r.b * p.dq_sb + r.tq * p.dq_st + (int64_t)h0 * p.dq_sh;
  for (int i = tid; i < nh * Dq; i += kGenThreads) dq[(i / Dq) * p.dq_sh + i % Dq] = f2bf(dqs[i] * p.scale);
}

size_t bwd_general_smem(const SfaParams& p, int HG) {
  return sizeof(float) * ((size_t)HG * p.d_qk * 2 + (size_t)HG * p.d_v + (size_t)kKC * p.d_qk +
                          (size_t)kKC * p.d_v + 2 * (size_t)HG * kKC + 2 * HG) + sizeof(int) * kKC;
}

int general_head_group(const SfaParams& p) {
  int G = p.h_q / p.h_kv;
  return G < 16 ? G : 16;
}

cudaError_t launch_fwd_general(const SfaParams& p, cudaStream_t st) {
  int HG = general_head_group(p);
  int G = p.h_q / p.h_kv;
  size_t smem = fwd_general_smem(p, HG);
  cudaError_t e = cudaFuncSetAttribute(fwd_general_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(num_rows_host(p), p.h_kv, (G + HG - 1) / HG);
  if (grid.x == 0) return cudaSuccess;
  fwd_general_kernel<<<grid, kGenThreads, smem, st>>>(p, HG);
  note_launch("fwd_general", st);
  return cudaGetLastError();
}

cudaError_t launch_bwd_general(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc,
                               cudaStream_t st) {
  int HG = general_head_group(p);
  int G = p.h_q / p.h_kv;
  size_t smem = bwd_general_smem(p, HG);
  cudaError_t e = cudaFuncSetAttribute(bwd_general_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(num_rows_host(p), p.h_kv, (G + HG - 1) / HG);
  if (grid.x == 0) return cudaSuccess;
  bwd_general_kernel<<<grid, kGenThreads, smem, st>>>(p, HG, delta, dk_acc, dv_acc);
  note_launch("bwd_general", st);
  return cudaGetLastError();
}

}  // namespace sfa
