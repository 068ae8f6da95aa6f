// sfa_mla_bwd.cu — tensor-core SFA backward for token-level top-k at head dims
// above 256 (MLA: D_qk 576, D_v 512 with v = kv[..., :512], 128 query heads on
// one latent kv head), where the one-pass token-level backward does not fit:
// dQ of 128 heads x 576 dims is 288 KB of fp32 (TMEM holds 256 KB) and Q plus
// dO of 128 heads are 272 KB (shared memory holds 227 KB).
//
// Two passes over a workspace that holds P and dS' = scale * P * (dP - delta)
// as bf16, one row of topk slots per (query, head):
//
//  1. this file's kernel, per (query row, kv head, 64-head group): the
//     stacked product
//         [S ; dP] = [Q ; dO] . K_sel^T     (M = 128: Q rows 0-63, dO rows 64-127;
//                                           N = 128 keys; K = D_qk, dO zero past D_v)
//     valid because V is K's leading D_v dims, so one MMA chain over the
//     gathered K slabs yields S in TMEM lanes 0-63 and dP in lanes 64-127.
//     The S lanes form P = exp2(S*c - lse2), hand it to the dP lanes through
//     shared memory (fp32), and both write their bf16 rows to the workspace.
//  2. the token-level backward's gradient half (sfa_tok_bwd.cu, two-pass form),
//     per (row, kv head, 128-head tile, 192-dim part of the head dims): reads
//     the P and dS' tiles by TMA and forms dQ (TMEM), dK^T and dV^T (merged,
//     drained into the fp32 accumulators with one reduction per (key, 128 heads)).
//
// Rows go through in waves so the workspace stays bounded.  Formulas: S and
// dP SFA.py:678-679, P and dS SFA.py:688-700 (delta from the preprocess kernel).
//
// Warp roles of pass 1 (512 threads, one persistent CTA per SM):
//   warp 0        descriptor producer: validity masks of the item's 64-slot
//                 chunks, chunk descriptors, the stacked Q / dO loads (4-D TMA);
//   warp 1        MMA issuer: [S ; dP] per 128-key chunk, one 64-dim slab at a time
//                 (N = 128: a 64-key chunk's N = 64 MMAs run at half rate);
//   warps 4-5     P (thread = head row, TMEM lanes 0-63);
//   warps 6-7     dS' (thread = head row, TMEM lanes 64-127);
//   warps 8-15    gather pool: warps 8+2g, 9+2g own K ring stage g, keys 0-63 and
//                 64-127 of its 128-key slab (tile::gather4).
// Every wait is bounded (~2 s); on expiry the kernel records (6 << 16) | site in
// the status word and returns.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"
#include "sfa_tok_common.cuh"

#include <stdlib.h>

namespace sfa {
using namespace tc;
using namespace tok;

namespace mla {

constexpr int kThreads = 512;
constexpr int kKeys = 128;             // keys per chunk: [S ; dP] MMAs at N = 128 (full rate)
constexpr int kMaxTopk = 16 * kKeys;
constexpr int kJD = 3;
constexpr int kSlab = 128 * 128;       // 128 keys x 64 dims bf16
constexpr int kQSlab = 128 * 128;      // 128 stacked rows x 64 dims bf16
constexpr int kHalf = 64;              // heads per item (rows 0-63 Q, 64-127 dO)
constexpr int kMaxStages = 4;
constexpr uint32_t kTmemCols = 256;    // two [S ; dP] buffers of 128 columns
constexpr int kXBytes = kHalf * 64 * 4;  // P hand-over, 64 keys at a time

enum : int { kFirst = 1, kLast = 2, kSentinel = 8 };

struct Desc {
  uint32_t m[4];                       // valid keys of the chunk (bit i of m[q]: key 32 q + i)
  int flags;
  int wrow, hk, hh, b, tq, chunk;
  int64_t kbase;
  int keys[kKeys];
};

struct Args {
  SfaParams p;
  const float* delta;                  // [rows][h_q]
  __nv_bfloat16* pws;                  // P   [wave rows][h_q][ld]
  __nv_bfloat16* dsws;                 // dS' [wave rows][h_q][ld]
  int64_t ld;
  int r0;                              // first row of the wave
  int nitems, n_hh, HH, G, nq, nv, ks;
  uint32_t off_k, off_x, off_desc, off_bar;
  int64_t k_rs;
  int32_t* status;
};

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t sd_full[2], sd_empty[2];
  uint64_t x_full, x_empty;            // P hand-over from the S lanes to the dP lanes
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint64_t k_full[kMaxStages], k_empty[kMaxStages];
  uint32_t tmem_base;
  uint32_t pad;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (6 << 16) | site);
  return false;
}

__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

__device__ __forceinline__ void decode_item(const Args& a, int item, int& wrow, int& hk, int& hh) {
  hh = item % a.n_hh;
  const int r = item / a.n_hh;
  hk = r % a.p.h_kv;
  wrow = r / a.p.h_kv;
}

__global__ void __launch_bounds__(kThreads, 1)
sfa_mla_sdp_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaParams& p = args.p;
  uint8_t* sq = sbase;                                     // stacked [Q ; dO] slabs
  uint8_t* sk = sbase + args.off_k;                        // K ring (one 128-key slab per stage)
  float* xp = reinterpret_cast<float*>(sbase + args.off_x);
  Desc* jd = reinterpret_cast<Desc*>(sbase + args.off_desc);
  Bars& B = *reinterpret_cast<Bars*>(sbase + args.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* st = args.status;
  const int NQ = args.nq, NV = args.nv, KS = args.ks;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.sd_full[i], 1);
      mbar_init(&B.sd_empty[i], 4);
    }
    mbar_init(&B.x_full, 2);
    mbar_init(&B.x_empty, 2);
    // consumers of a descriptor: the MMA issuer, the gather pool (two warps a stage), the four P / dS' warps
    for (int i = 0; i < kJD; ++i) {
      mbar_init(&B.jd_full[i], 1);
      mbar_init(&B.jd_empty[i], 1 + 2 * KS + 4);
    }
    // a stage's two halves (keys 0-63, 64-127) arrive separately
    for (int i = 0; i < KS; ++i) {
      mbar_init(&B.k_full[i], 2);
      mbar_init(&B.k_empty[i], 1);
    }
    fence_barrier_init();
  }
  // rows no copy writes stay zero: heads past HH, and dO's rows of the slabs past D_v
  for (int i = threadIdx.x; i < NQ * kQSlab / 16; i += kThreads)
    reinterpret_cast<uint4*>(sq)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&B.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmdo);
    prefetch_tmap(&tmk);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;
  const int quad = lane & 15;

  if (warp == 0) {
    // ============================================================ descriptor producer
    int job = 0, item_i = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x) {
      int wrow, hk, hh;
      decode_item(args, item, wrow, hk, hh);
      const Row r = row_info(p, args.r0 + wrow);
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      const int nch = (p.topk + kKeys - 1) / kKeys;
      // lane c keeps the valid-key masks of chunk c
      uint32_t my_m[4] = {0u, 0u, 0u, 0u};
      for (int c = 0; c < nch; ++c) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int sl = c * kKeys + 32 * q + lane;
          const int e = sl < p.topk ? __ldg(idx + sl) : -1;
          const bool v = e >= 0 && e < r.kv_len && (!p.causal || e <= r.pos);
          const uint32_t m = __ballot_sync(0xffffffffu, v);
          if (lane == c) my_m[q] = m;
        }
      }
      // chunks without a valid key leave their workspace slots unwritten; the
      // gradient pass skips the same (64-key) chunks
      const uint32_t chunks = __ballot_sync(0xffffffffu, (my_m[0] | my_m[1] | my_m[2] | my_m[3]) != 0u);
      if (chunks == 0u) continue;
      const int64_t kbase = ((int64_t)r.b * p.k_sb + r.kv0 * p.k_st + (int64_t)hk * p.k_sh) / args.k_rs;
      if (lane == 0) {
        ok = wt(&B.q_empty, (item_i & 1) ^ 1, st, 1);
        if (ok) {
          mbar_arrive_expect_tx(&B.q_full, (uint32_t)(args.HH * 128 * (NQ + NV)));
          const int h0 = hk * args.G + hh * kHalf;
          for (int s = 0; s < NQ; ++s) tma_load_4d(sq + s * kQSlab, &tmq, &B.q_full, s * 64, h0, (int)r.tq, r.b);
          for (int s = 0; s < NV; ++s)
            tma_load_4d(sq + s * kQSlab + kQSlab / 2, &tmdo, &B.q_full, s * 64, h0, (int)r.tq, r.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++item_i;
      const int cfirst = __ffs(chunks) - 1, clast = 31 - __clz(chunks);
      for (uint32_t rem = chunks; rem && ok; rem &= rem - 1u, ++job) {
        const int c = __ffs(rem) - 1;
        uint32_t m[4];
        int e[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          m[q] = __shfl_sync(0xffffffffu, my_m[q], c);
          const int sl = c * kKeys + 32 * q + lane;
          e[q] = sl < p.topk ? __ldg(idx + sl) : -1;
        }
        // invalid slots gather the chunk's first valid key (in bounds); their P is 0
        const int fq = m[0] ? 0 : m[1] ? 1 : m[2] ? 2 : 3;
        const int fl = __ffs(m[fq]) - 1;
        int fk = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int f = __shfl_sync(0xffffffffu, e[q], fl);
          if (q == fq) fk = f;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (!((m[q] >> lane) & 1u)) e[q] = fk;
        const int js = job % kJD;
        if (lane == 0) ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 2);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        Desc& d = jd[js];
#pragma unroll
        for (int q = 0; q < 4; ++q) d.keys[32 * q + lane] = e[q];
        if (lane < 4) d.m[lane] = m[lane];
        if (lane == 0) {
          d.flags = (c == cfirst ? kFirst : 0) | (c == clast ? kLast : 0);
          d.wrow = wrow; d.hk = hk; d.hh = hh; d.b = r.b; d.tq = (int)r.tq; d.chunk = c;
          d.kbase = kbase;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.jd_full[js]);
      }
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 3)) {
        jd[js].flags = kSentinel;
        mbar_arrive(&B.jd_full[js]);
      }
    }
  } else if (warp >= 8) {
    // ============================================================ gather pool
    // Slab j of the kernel's sequence (chunk-major, NQ slabs a chunk) goes to
    // ring stage j % KS; warps 8 + 2g and 9 + 2g own stage g (keys 0-63 and
    // 64-127 of the slab) and serve every use of it in order.
    const int g = (warp - 8) >> 1, half = (warp - 8) & 1;
    if (g < KS) {
      const int64_t kstep = p.k_st / args.k_rs;
      int job = 0;
      int64_t j = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 4);
        if (!ok) break;
        const Desc& d = jd[js];
        const int flags = d.flags;
        if (flags & kSentinel) break;
        const int e0 = d.keys[64 * half + lane], e1 = d.keys[64 * half + 32 + lane];
        const int64_t kbase = d.kbase;
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.jd_empty[js]);
        int kq[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int src = (4 * quad + i) & 31;
          const int a = __shfl_sync(0xffffffffu, e0, src), bb = __shfl_sync(0xffffffffu, e1, src);
          kq[i] = quad < 8 ? a : bb;
        }
        for (int s = 0; s < NQ && ok; ++s, ++j) {
          const int stg = (int)(j % KS);
          if (stg != g) continue;
          const uint32_t use = (uint32_t)(j / KS);
          if (lane == 0) {
            ok = wt(&B.k_empty[stg], (use & 1) ^ 1, st, 5);
            if (ok) mbar_arrive_expect_tx(&B.k_full[stg], (uint32_t)(kSlab / 2));
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (ok && lane < 16)
            gather4(sk + stg * kSlab + half * (kSlab / 2) + quad * 512, &tmk, &B.k_full[stg], s * 64,
                    (int)(kbase + kq[0] * kstep), (int)(kbase + kq[1] * kstep), (int)(kbase + kq[2] * kstep),
                    (int)(kbase + kq[3] * kstep));
        }
        ++job;
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer: [S ; dP]
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, kKeys, false, false);
      int job = 0, item_i = 0, chunk = 0;
      int64_t j = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 6))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (flags & kFirst) {
          if (!(ok = wt(&B.q_full, item_i & 1, st, 7))) break;
          ++item_i;
        }
        const int buf = chunk & 1;
        if (!(ok = wt(&B.sd_empty[buf], ((chunk >> 1) & 1) ^ 1, st, 8))) break;
        tc_fence_after();
        for (int s = 0; s < NQ && ok; ++s, ++j) {
          const int stg = (int)(j % KS);
          if (!(ok = wt(&B.k_full[stg], (uint32_t)((j / KS) & 1), st, 9))) break;
          tc_fence_after();
          const uint64_t kd = smem_desc(smem_u32(sk + stg * kSlab), 16, 1024, kSw128);
          const uint64_t qd = smem_desc(smem_u32(sq + s * kQSlab), 16, 1024, kSw128);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tmem + buf * kKeys, qd + (uint64_t)((k * 32) >> 4), kd + (uint64_t)((k * 32) >> 4), id_s,
                        (s | k) != 0);
          mma_commit(&B.k_empty[stg]);
        }
        if (!ok) break;
        mma_commit(&B.sd_full[buf]);
        if (flags & kLast) mma_commit(&B.q_empty);
        ++chunk;
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp >= 4) {
    // ============================================================ P (warps 4-5) / dS' (warps 6-7)
    const int wq = warp & 3;
    const bool is_p = wq < 2;
    const int hm = (wq & 1) * 32 + lane;                  // head within the item's group
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    float ref = 0.f;                                      // lse2 (P lanes) or delta (dS' lanes)
    int job = 0, chunk = 0, xc = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 10))) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      const bool hv = hm < args.HH;
      const int h = d.hk * args.G + d.hh * kHalf + hm;
      uint32_t mk[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) mk[q] = d.m[q];
      const int64_t wsrow = ((int64_t)d.wrow * p.h_q + h) * args.ld + (int64_t)d.chunk * kKeys;
      const int row = args.r0 + d.wrow;
      if (flags & kFirst) {
        if (is_p) {
          ref = hv ? __ldg(p.lse + (int64_t)d.b * p.l_sb + (int64_t)d.tq * p.l_st + (int64_t)h * p.l_sh) * kLog2e
                   : INFINITY;
          if (!(ref > -INFINITY)) ref = INFINITY;          // a row with no mass: P = 0
        } else {
          ref = hv ? __ldg(args.delta + (int64_t)row * p.h_q + h) : 0.f;
        }
      }
      __syncwarp();
      warp_arrive(&B.jd_empty[js]);
      ++job;
      const int buf = chunk & 1;
      if (!(ok = wtw(&B.sd_full[buf], (chunk >> 1) & 1, st, 11))) break;
      tc_fence_after();
      // the chunk's 128 keys in two halves of 64 (one P hand-over each)
      for (int kh = 0; kh < 2 && ok; ++kh, ++xc) {
        float v[64];
        {
          float a[32];
          tmem_ld32(tl + buf * kKeys + 64 * kh, a);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = a[i];
          tmem_ld32(tl + buf * kKeys + 64 * kh + 32, a);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[32 + i] = a[i];
        }
        if (kh == 1) {
          tc_fence_before();
          warp_arrive(&B.sd_empty[buf]);
        }
        const uint32_t mlo = kh ? mk[2] : mk[0], mhi = kh ? mk[3] : mk[1];
        // row (head hm) of the exchange buffer, 16-byte groups rotated by the row
        float* xrow = xp + hm * 64;
        if (is_p) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const uint32_t m = i < 32 ? mlo : mhi;
            v[i] = (hv && ((m >> (i & 31)) & 1u)) ? ex2(fmaf(v[i], c2, -ref)) : 0.f;
          }
          // the dS' lanes have read the previous hand-over
          if (!(ok = wtw(&B.x_empty, (xc & 1) ^ 1, st, 12))) break;
#pragma unroll
          for (int g4 = 0; g4 < 16; ++g4)
            *reinterpret_cast<float4*>(xrow + 4 * ((g4 + hm) & 15)) =
                make_float4(v[4 * g4], v[4 * g4 + 1], v[4 * g4 + 2], v[4 * g4 + 3]);
          __syncwarp();
          warp_arrive(&B.x_full);
        } else {
          if (!(ok = wtw(&B.x_full, xc & 1, st, 13))) break;
#pragma unroll
          for (int g4 = 0; g4 < 16; ++g4) {
            const float4 t = *reinterpret_cast<const float4*>(xrow + 4 * ((g4 + hm) & 15));
            v[4 * g4] = p.scale * t.x * (v[4 * g4] - ref);
            v[4 * g4 + 1] = p.scale * t.y * (v[4 * g4 + 1] - ref);
            v[4 * g4 + 2] = p.scale * t.z * (v[4 * g4 + 2] - ref);
            v[4 * g4 + 3] = p.scale * t.w * (v[4 * g4 + 3] - ref);
          }
          __syncwarp();
          warp_arrive(&B.x_empty);
        }
        if (hv) {
          uint4* dst = reinterpret_cast<uint4*>((is_p ? args.pws : args.dsws) + wsrow + 64 * kh);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
        }
      }
      ++chunk;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

struct Plan {
  Args a;
  size_t smem;
};

static bool plan(const SfaParams& p, Plan* out, const char** why) {
  const int G = p.h_q / p.h_kv;
  Args& a = out->a;
  a = Args{};
  a.p = p;
  a.G = G;
  a.HH = G < kHalf ? G : kHalf;
  a.n_hh = (G + kHalf - 1) / kHalf;
  if (G > kHalf && G % kHalf) { *why = "query heads per kv head must be <= 64 or a multiple of 64"; return false; }
  a.nq = p.d_qk / 64;
  a.nv = p.d_v / 64;
  int64_t krows = 0;
  a.k_rs = gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  if (!a.k_rs) { *why = "k batch, token and head strides must fold into evenly spaced rows"; return false; }
  if (krows > INT32_MAX) { *why = "too many kv rows for 32-bit gather coordinates"; return false; }
  const size_t budget = 227 * 1024 - 1024;
  const size_t desc = ((sizeof(Desc) * kJD + 127) / 128) * 128;
  const size_t bars = ((sizeof(Bars) + 127) / 128) * 128;
  const size_t fixed = (size_t)a.nq * kQSlab + kXBytes + desc + bars;
  int ks = 0;
  while (ks < kMaxStages && fixed + (size_t)(ks + 1) * kSlab <= budget) ++ks;
  if (ks < 2) { *why = "head dims too large for shared memory"; return false; }
  a.ks = ks;
  a.off_k = (uint32_t)a.nq * kQSlab;
  a.off_x = a.off_k + (uint32_t)(ks * kSlab);
  a.off_desc = a.off_x + kXBytes;
  a.off_bar = a.off_desc + (uint32_t)desc;
  out->smem = a.off_bar + bars + 1024;
  return true;
}

}  // namespace mla

// ======================================================================
// Pass 2: gradients from the P / dS' workspace, 128-key chunks.
//
// Work item = (query row, kv head, head tile of <= 128 heads, part of 128
// head dims).  Per 128-key chunk the chunk's P and dS' tiles arrive by TMA
// (two 64-slot boxes each) and the part's K rows by tile::gather4; then
//     dQ[heads, part]   += dS' . K_part            (M = 128, N = 128, K = 128 keys)   issuer A
//     dKV^T[part, keys]  = Q_part^T . dS'^T (+ dO_part^T . P^T when the part has V dims)
//                                                   (M = 128, N = 128, K = heads)      issuer B
// dQ stays in TMEM for the item; the dKV^T tile (double-buffered) is drained
// into the fp32 accumulator by eight warps (keys 0-63 / 64-127), one 128-byte
// line per (key, 32 dims) and reduction.
//
// Warp roles (512 threads): 0 descriptors, Q / dO of the part, the P / dS'
// tiles; 1 issuer A; 2 issuer B; 8-11 gather (warp 8+g: slab g >> 1, keys
// 64 (g & 1) .. + 63 of each stage); 4-7 drain (keys 64-127) and the dq
// epilogue; 12-15 drain (keys 0-63).  Status (8 << 16) | site.
namespace mlag {

constexpr int kThreads = 512;
constexpr int kKeys = 128;
constexpr int kJD = 4;
constexpr int kPD = 128;                       // head dims a part
constexpr int kSlab = 128 * 128;               // 128 keys x 64 dims bf16
constexpr int kQSlab = 128 * 128;              // 128 heads x 64 dims bf16
constexpr int kTile = 2 * 128 * 128;           // P or dS' of a chunk: 128 heads x 128 slots (two 64-slot boxes)
constexpr int kStages = 2;
constexpr int kGatherWarps = 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColDQ = 0, kColKV = 128;   // dKV^T buffers at 128 and 256

enum : int { kFirst = 1, kLast = 2, kEmpty = 4, kSentinel = 8 };

struct Desc {
  uint32_t m[4];
  int flags;
  int row, hk, hg, b, tq, part, nqi, nvi, chunk, wrow;
  int64_t kbase, accrow;
  int keys[kKeys];
};

struct Args {
  SfaParams p;
  float* dk_acc;                       // fp32 [kv rows][h_kv][d_qk]: dk + dv of the one latent tensor
  int r0;
  int nitems, n_hg, HG, G, parts, nq_all, nv_all;
  int64_t k_rs;
  uint32_t off_do, off_k, off_t, off_desc, off_bar;
  int32_t* status;
};

struct Bars {
  uint64_t q_full, q_empty, t_full, t_empty;
  uint64_t dq_full, dq_empty;
  uint64_t kv_full[2], kv_empty[2];
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint64_t k_full[kStages], k_empty[kStages];
  uint32_t tmem_base;
  uint32_t pad;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (8 << 16) | site);
  return false;
}

__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

__device__ __forceinline__ void decode_item(const Args& a, int item, int& row, int& hk, int& hg, int& part) {
  part = item % a.parts;               // a row's parts run side by side: its P / dS' rows stay in L2
  item /= a.parts;
  hg = item % a.n_hg;
  const int r = item / a.n_hg;
  hk = r % a.p.h_kv;
  row = a.r0 + r / a.p.h_kv;
}

__global__ void __launch_bounds__(kThreads, 1)
sfa_mla_grad_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                    const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmp, const __grid_constant__ CUtensorMap tmds) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaParams& p = args.p;
  uint8_t* sq = sbase;                          // Q of the part: 2 slabs of 128 heads x 64 dims
  uint8_t* sdo = sbase + args.off_do;           // dO of the part: 2 slabs
  uint8_t* sk = sbase + args.off_k;             // K ring: stages of 2 slabs x 128 keys
  uint8_t* sp = sbase + args.off_t;             // P tile (2 x 64 slots), then the dS' tile
  uint8_t* sds = sp + kTile;
  Desc* jd = reinterpret_cast<Desc*>(sbase + args.off_desc);
  Bars& B = *reinterpret_cast<Bars*>(sbase + args.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* st = args.status;
  constexpr int kStageBytes = 2 * kSlab;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    mbar_init(&B.t_full, 1);
    mbar_init(&B.t_empty, 2);                  // both issuers read the tiles
    mbar_init(&B.dq_full, 1);
    mbar_init(&B.dq_empty, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.kv_full[i], 1);
      mbar_init(&B.kv_empty[i], 8);
    }
    // descriptor consumers: two issuers, the gather warps, eight drain warps
    for (int i = 0; i < kJD; ++i) {
      mbar_init(&B.jd_full[i], 1);
      mbar_init(&B.jd_empty[i], 2 + kGatherWarps + 8);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&B.k_full[i], kGatherWarps);
      mbar_init(&B.k_empty[i], 1);
    }
    fence_barrier_init();
  }
  // head rows past HG stay zero in Q, dO and the tiles (TMA writes HG rows)
  if (args.HG < 128) {
    for (int i = threadIdx.x; i < 4 * kQSlab / 16; i += kThreads) reinterpret_cast<uint4*>(sq)[i] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < 2 * kTile / 16; i += kThreads) reinterpret_cast<uint4*>(sp)[i] = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&B.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmdo);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmp);
    prefetch_tmap(&tmds);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;
  const int quad = lane & 15;

  if (warp == 0) {
    // ============================================================ descriptors, Q / dO, tiles
    int job = 0, item_i = 0, tile = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x) {
      int row, hk, hg, part;
      decode_item(args, item, row, hk, hg, part);
      const Row r = row_info(p, row);
      const int s0q = part * 2;
      const int nqi = min(2, args.nq_all - s0q), nvi = max(0, min(2, args.nv_all - s0q));
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      const int nch = (p.topk + kKeys - 1) / kKeys;
      uint32_t my_m[4] = {0u, 0u, 0u, 0u};
      for (int c = 0; c < nch; ++c) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int sl = c * kKeys + 32 * q + lane;
          const int e = sl < p.topk ? __ldg(idx + sl) : -1;
          const bool v = e >= 0 && e < r.kv_len && (!p.causal || e <= r.pos);
          const uint32_t m = __ballot_sync(0xffffffffu, v);
          if (lane == c) my_m[q] = m;
        }
      }
      const uint32_t chunks = __ballot_sync(0xffffffffu, (my_m[0] | my_m[1] | my_m[2] | my_m[3]) != 0u);
      const int64_t kbase = ((int64_t)r.b * p.k_sb + r.kv0 * p.k_st + (int64_t)hk * p.k_sh) / args.k_rs;
      const int64_t accrow = p.cu_seqlens_q == nullptr ? (int64_t)r.b * p.kv_len : r.kv0;
      if (chunks == 0u) {
        // nothing selected: dq of the part is zero, nothing reaches dk / dv
        if (lane == 0) {
          const int js = job % kJD;
          ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 1);
          if (ok) {
            Desc& d = jd[js];
            d.flags = kFirst | kLast | kEmpty;
            d.row = row; d.hk = hk; d.hg = hg; d.b = r.b; d.tq = (int)r.tq; d.part = part; d.nqi = nqi; d.nvi = nvi;
            mbar_arrive(&B.jd_full[js]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        ++job;
        continue;
      }
      ok = wtw(&B.q_empty, (item_i & 1) ^ 1, st, 2);
      // a part with one dO slab beside two Q slabs: the dV^T product reads the
      // second slab for dims that do hold dK, so it must be zero
      if (ok && nvi == 1 && nqi == 2) {
        for (int i = lane; i < kQSlab / 16; i += 32) reinterpret_cast<uint4*>(sdo + kQSlab)[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        if (ok) {
          mbar_arrive_expect_tx(&B.q_full, (uint32_t)(args.HG * 128 * (nqi + nvi)));
          for (int sl = 0; sl < nqi; ++sl)
            tma_load_4d(sq + sl * kQSlab, &tmq, &B.q_full, (s0q + sl) * 64, hk * args.G + hg * 128, (int)r.tq, r.b);
          for (int sl = 0; sl < nvi; ++sl)
            tma_load_4d(sdo + sl * kQSlab, &tmdo, &B.q_full, (s0q + sl) * 64, hk * args.G + hg * 128, (int)r.tq, r.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++item_i;
      const int cfirst = __ffs(chunks) - 1, clast = 31 - __clz(chunks);
      for (uint32_t rem = chunks; rem && ok; rem &= rem - 1u, ++job) {
        const int c = __ffs(rem) - 1;
        uint32_t m[4];
        int e[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          m[q] = __shfl_sync(0xffffffffu, my_m[q], c);
          const int sl = c * kKeys + 32 * q + lane;
          e[q] = sl < p.topk ? __ldg(idx + sl) : -1;
        }
        const int fq = m[0] ? 0 : m[1] ? 1 : m[2] ? 2 : 3;
        const int fl = __ffs(m[fq]) - 1;
        int fk = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int f = __shfl_sync(0xffffffffu, e[q], fl);
          if (q == fq) fk = f;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (!((m[q] >> lane) & 1u)) e[q] = fk;
        const int js = job % kJD;
        if (lane == 0) ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 3);
        // this chunk's P and dS' tiles (one buffer: the issuers of the previous chunk release it)
        if (lane == 0 && ok) {
          ok = wt(&B.t_empty, (tile & 1) ^ 1, st, 4);
          if (ok) {
            mbar_arrive_expect_tx(&B.t_full, (uint32_t)(4 * args.HG * 128));
            const int wrow = row - args.r0, h0 = hk * args.G + hg * 128;
            for (int hb = 0; hb < 2; ++hb) {
              tma_load_4d(sp + hb * kQSlab, &tmp, &B.t_full, c * kKeys + 64 * hb, h0, wrow, 0);
              tma_load_4d(sds + hb * kQSlab, &tmds, &B.t_full, c * kKeys + 64 * hb, h0, wrow, 0);
            }
          }
        }
        ++tile;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        Desc& d = jd[js];
#pragma unroll
        for (int q = 0; q < 4; ++q) d.keys[32 * q + lane] = e[q];
        if (lane < 4) d.m[lane] = m[lane];
        if (lane == 0) {
          d.flags = (c == cfirst ? kFirst : 0) | (c == clast ? kLast : 0);
          d.row = row; d.hk = hk; d.hg = hg; d.b = r.b; d.tq = (int)r.tq;
          d.part = part; d.nqi = nqi; d.nvi = nvi; d.chunk = c;
          d.kbase = kbase; d.accrow = accrow;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.jd_full[js]);
      }
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 5)) {
        jd[js].flags = kSentinel;
        mbar_arrive(&B.jd_full[js]);
      }
    }
  } else if (warp >= 8 && warp < 8 + kGatherWarps) {
    // ============================================================ gather: K rows of the part
    // warp 8 + g fills slab g >> 1, keys 64 (g & 1) .. + 63, of every stage use in order
    const int g = warp - 8, sl = g >> 1, half = g & 1;
    const int64_t kstep = p.k_st / args.k_rs;
    int job = 0, use = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 6);
      if (!ok) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      if (flags & kEmpty) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.jd_empty[js]);
        ++job;
        continue;
      }
      const int e0 = d.keys[64 * half + lane], e1 = d.keys[64 * half + 32 + lane];
      const int64_t kbase = d.kbase;
      const bool real = sl < d.nqi;
      const int col = (d.part * 2 + sl) * 64;
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.jd_empty[js]);
      int kq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int src = (4 * quad + i) & 31;
        const int a = __shfl_sync(0xffffffffu, e0, src), bb = __shfl_sync(0xffffffffu, e1, src);
        kq[i] = quad < 8 ? a : bb;
      }
      const int s_ = use % kStages;
      uint64_t* full = &B.k_full[s_];
      if (lane == 0) {
        ok = wt(&B.k_empty[s_], ((use / kStages) & 1) ^ 1, st, 7);
        if (ok) {
          if (real) mbar_arrive_expect_tx(full, (uint32_t)(kSlab / 2));
          else mbar_arrive(full);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (ok && real && lane < 16)
        gather4(sk + s_ * kStageBytes + sl * kSlab + half * (kSlab / 2) + quad * 512, &tmk, full, col,
                (int)(kbase + kq[0] * kstep), (int)(kbase + kq[1] * kstep), (int)(kbase + kq[2] * kstep),
                (int)(kbase + kq[3] * kstep));
      ++use;
      ++job;
    }
  } else if (warp == 1) {
    // ============================================================ issuer A: dQ += dS' . K_part
    if (lane == 0) {
      int job = 0, use = 0, chunk = 0, item_i = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 8))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          const int nqi = jd[js].nqi;
          const uint32_t id_q = idesc_bf16(128, (uint32_t)(nqi * 64), false, true);
          if (flags & kFirst)
            if (!(ok = wt(&B.dq_empty, (item_i & 1) ^ 1, st, 9))) break;
          if (!(ok = wt(&B.t_full, chunk & 1, st, 10))) break;
          const int s_ = use % kStages;
          if (!(ok = wt(&B.k_full[s_], (use / kStages) & 1, st, 11))) break;
          tc_fence_after();
          // A: dS' [heads][keys], K-major, keys in two 64-slot boxes 16 KB apart;
          // B: the K stage MN-major (dims: 64-dim slabs 32 KB apart; keys: 16-row steps of 2 KB)
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = smem_desc(smem_u32(sds + (k >> 2) * kQSlab), 16, 1024, kSw128) +
                                (uint64_t)(((k & 3) * 32) >> 4);
            const uint64_t bd = smem_desc(smem_u32(sk + s_ * kStageBytes + k * 2048), kSlab, 1024, kSw128);
            mma_bf16_ss(tmem + kColDQ, ad, bd, id_q, !((flags & kFirst) && k == 0));
          }
          mma_commit(&B.k_empty[s_]);
          mma_commit(&B.t_empty);
          if (flags & kLast) {
            mma_commit(&B.dq_full);
            ++item_i;
          }
          ++use;
          ++chunk;
        }
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp == 2) {
    // ============================================================ issuer B: dKV^T tile
    if (lane == 0) {
      const uint32_t id_kv = idesc_bf16(128, kKeys, true, true);
      int job = 0, chunk = 0, item_i = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 12))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          const int nvi = jd[js].nvi;
          if (flags & kFirst)
            if (!(ok = wt(&B.q_full, item_i & 1, st, 13))) break;
          if (!(ok = wt(&B.t_full, chunk & 1, st, 14))) break;
          const int kb = chunk & 1;
          if (!(ok = wt(&B.kv_empty[kb], ((chunk >> 1) & 1) ^ 1, st, 15))) break;
          tc_fence_after();
          const uint32_t dcol = tmem + kColKV + kb * 128;
          // A: Q^T (dims: two 64-dim slabs 16 KB apart; heads: 16-row steps of 2 KB), MN-major;
          // B: dS'^T (keys: two 64-slot boxes 16 KB apart; heads: 16-row steps), MN-major
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = smem_desc(smem_u32(sq + k * 2048), kQSlab, 1024, kSw128);
            const uint64_t bd = smem_desc(smem_u32(sds + k * 2048), kQSlab, 1024, kSw128);
            mma_bf16_ss(dcol, ad, bd, id_kv, k != 0);
          }
          if (nvi > 0) {
            for (int k = 0; k < 8; ++k) {
              const uint64_t ad = smem_desc(smem_u32(sdo + k * 2048), kQSlab, 1024, kSw128);
              const uint64_t bd = smem_desc(smem_u32(sp + k * 2048), kQSlab, 1024, kSw128);
              mma_bf16_ss(dcol, ad, bd, id_kv, 1);
            }
          }
          mma_commit(&B.t_empty);
          mma_commit(&B.kv_full[kb]);
          if (flags & kLast) {
            mma_commit(&B.q_empty);
            ++item_i;
          }
          ++chunk;
        }
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else if ((warp >= 4 && warp < 8) || warp >= 12) {
    // ============================================================ drain (+ dq epilogue in warps 4-7)
    const int wq = warp & 3;
    const int kh = warp < 8 ? 1 : 0;            // keys 64 kh .. + 63 of each chunk
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    int job = 0, chunk = 0, item_i = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 16))) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      const int d0 = d.part * kPD, nk = d.nqi * 64;
      if (!(flags & kEmpty)) {
        const uint32_t m0 = d.m[2 * kh], m1 = d.m[2 * kh + 1];
        const int r0 = (int)((d.accrow + d.keys[64 * kh + lane]) * p.h_kv + d.hk);
        const int r1 = (int)((d.accrow + d.keys[64 * kh + 32 + lane]) * p.h_kv + d.hk);
        const int kb = chunk & 1;
        if (!(ok = wtw(&B.kv_full[kb], (chunk >> 1) & 1, st, 17))) break;
        tc_fence_after();
        const int dim = 32 * wq + lane;                 // TMEM lane = dim of the part
        // one latent gradient buffer: dK and dV share the tile
        float* acc = args.dk_acc + d0 + dim;
        const bool dim_ok = dim < nk;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v[32];
          tmem_ld32(tl + kColKV + kb * 128 + 64 * kh + 32 * hh, v);
          tmem_ld_wait();
          const uint32_t msk = hh ? m1 : m0;
          const int rr = hh ? r1 : r0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int ri = __shfl_sync(0xffffffffu, rr, i);
            if (((msk >> i) & 1u) && dim_ok) atomicAdd(acc + (int64_t)ri * p.d_qk, v[i]);
          }
        }
        tc_fence_before();
        warp_arrive(&B.kv_empty[kb]);
        ++chunk;
      }
      // dq of the part: warps 4-7 (thread = head row), after the item's last chunk
      if (kh == 1 && (flags & kLast)) {
        const int m = wq * 32 + lane;
        const int h = d.hk * args.G + d.hg * 128 + m;
        const bool hv = d.hg * 128 + m < args.G;
        __nv_bfloat16* dqrow = reinterpret_cast<__nv_bfloat16*>(p.dq) + (int64_t)d.b * p.dq_sb +
                               (int64_t)d.tq * p.dq_st + (int64_t)h * p.dq_sh + d0;
        if (flags & kEmpty) {
          if (hv)
            for (int i = 0; i < nk; i += 8) *reinterpret_cast<uint4*>(dqrow + i) = make_uint4(0, 0, 0, 0);
        } else {
          if (!(ok = wtw(&B.dq_full, item_i & 1, st, 18))) break;
          tc_fence_after();
          for (int c0 = 0; c0 < nk; c0 += 32) {
            float o[32];
            tmem_ld32(tl + kColDQ + c0, o);
            tmem_ld_wait();
            if (hv) {
#pragma unroll
              for (int i = 0; i < 32; i += 8)
                *reinterpret_cast<uint4*>(dqrow + c0 + i) =
                    make_uint4(pack_bf16x2(o[i], o[i + 1]), pack_bf16x2(o[i + 2], o[i + 3]),
                               pack_bf16x2(o[i + 4], o[i + 5]), pack_bf16x2(o[i + 6], o[i + 7]));
            }
          }
          tc_fence_before();
          warp_arrive(&B.dq_empty);
          ++item_i;
        }
      }
      warp_arrive(&B.jd_empty[js]);
      ++job;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace mlag

// ------------------------------------------------------------------ host side

bool mla_bwd_supported(const SfaParams& p, const char** why) {
  if (device_cc() != 100) { *why = "needs an sm_100 device"; return false; }
  if (p.block_size != 1) { *why = "two-pass token-level backward: block_size must be 1"; return false; }
  if (p.topk > mla::kMaxTopk) { *why = "two-pass token-level backward: topk must be <= 2048"; return false; }
  if (p.d_qk % 64 || p.d_v % 64 || p.d_qk > 576 || p.d_v > p.d_qk) {
    *why = "two-pass token-level backward: head dims must be multiples of 64, d_v <= d_qk <= 576";
    return false;
  }
  // the stacked [S ; dP] product needs V to be K's leading dims
  const bool v_leading = p.v == p.k && p.v_sb == p.k_sb && p.v_st == p.k_st && p.v_sh == p.k_sh;
  if (!v_leading) { *why = "two-pass token-level backward: v must be k or k's leading dims"; return false; }
  if (!(p.scale > 0.f)) { *why = "needs a positive softmax scale"; return false; }
  if (!tma_compatible(p.q, p.q_sb, p.q_st, p.q_sh) || !tma_compatible(p.k, p.k_sb, p.k_st, p.k_sh) ||
      !tma_compatible(p.dout, p.do_sb, p.do_st, p.do_sh)) {
    *why = "q/k/dout need 16-byte aligned base and strides";
    return false;
  }
  if ((p.dq_sh % 8) || (p.dq_st % 8) || (p.dq_sb % 8) || (reinterpret_cast<uintptr_t>(p.dq) & 15)) {
    *why = "dq needs a 16-byte aligned base and strides";
    return false;
  }
  mla::Plan pl;
  if (!mla::plan(p, &pl, why)) return false;
  return tok_bwd_parts_supported(p, why);
}

namespace mlag {

struct Plan {
  Args a;
  size_t smem;
};

static bool plan(const SfaParams& p, Plan* out, const char** why) {
  const int G = p.h_q / p.h_kv;
  Args& a = out->a;
  a = Args{};
  a.p = p;
  a.G = G;
  a.HG = G < 128 ? G : 128;
  a.n_hg = (G + 127) / 128;
  if (G > 128 && G % 128) { *why = "query heads per kv head must be <= 128 or a multiple of 128"; return false; }
  if (p.dk != p.dv) { *why = "the 128-key gradient pass needs one gradient buffer (dk == dv)"; return false; }
  a.nq_all = p.d_qk / 64;
  a.nv_all = p.d_v / 64;
  a.parts = (a.nq_all + 1) / 2;
  int64_t krows = 0;
  a.k_rs = gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  if (!a.k_rs) { *why = "k batch, token and head strides must fold into evenly spaced rows"; return false; }
  if (krows > INT32_MAX) { *why = "too many kv rows for 32-bit gather coordinates"; return false; }
  const size_t desc = ((sizeof(Desc) * kJD + 127) / 128) * 128;
  const size_t bars = ((sizeof(Bars) + 127) / 128) * 128;
  a.off_do = 2 * kQSlab;
  a.off_k = a.off_do + 2 * kQSlab;
  a.off_t = a.off_k + kStages * 2 * kSlab;
  a.off_desc = a.off_t + 2 * kTile;
  a.off_bar = a.off_desc + (uint32_t)desc;
  out->smem = a.off_bar + bars + 1024;
  if (out->smem > 227 * 1024) { *why = "shared memory"; return false; }
  return true;
}

}  // namespace mlag

// workspace row length: whole 128-key chunks of the first pass
int64_t mla_ws_ld(const SfaParams& p) { return (int64_t)((p.topk + mla::kKeys - 1) / mla::kKeys) * mla::kKeys; }

// Rows per wave: the P and dS' workspace of one wave stays within 4 GiB
// (SFA_MLA_WAVE_ROWS overrides, for tests of the wave loop).
int64_t mla_wave_rows(const SfaParams& p) {
  const int64_t rows = num_rows_host(p);
  const int64_t per_row = 2 * (int64_t)p.h_q * mla_ws_ld(p) * 2;
  int64_t w = ((int64_t)4 << 30) / (per_row > 0 ? per_row : 1);
  if (const char* e = getenv("SFA_MLA_WAVE_ROWS")) {
    const long long v = atoll(e);
    if (v > 0) w = v;
  }
  if (w < 1) w = 1;
  return w < rows ? w : rows;
}

size_t mla_ws_bytes(const SfaParams& p) {
  return (size_t)(2 * mla_wave_rows(p) * (int64_t)p.h_q * mla_ws_ld(p) * 2);
}

cudaError_t launch_bwd_mla(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc, void* pd,
                           cudaStream_t stream) {
  mla::Plan pl;
  const char* why = "";
  if (!mla::plan(p, &pl, &why)) return cudaErrorInvalidValue;
  mla::Args& a = pl.a;
  const int64_t rows = num_rows_host(p);
  if (rows == 0) return cudaSuccess;
  const int64_t wave = mla_wave_rows(p);
  const int64_t ld = mla_ws_ld(p);
  a.delta = delta;
  a.ld = ld;
  a.pws = reinterpret_cast<__nv_bfloat16*>(pd);
  a.dsws = a.pws + wave * p.h_q * ld;
  a.status = device_status_ptr();
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len;
  const int64_t nb = vl ? 1 : p.batch;
  CUtensorMap tq, tdo, tk;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)p.d_qk, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)a.HH, 1u, 1u});
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_4d(&tdo, p.dout, {(uint64_t)p.d_v, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                        {p.do_sh, p.do_st, p.do_sb}, {64u, (uint32_t)a.HH, 1u, 1u});
  if (e != cudaSuccess) return e;
  int64_t krows = 0;
  gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  if ((e = make_tmap_rows(&tk, p.k, (uint64_t)p.d_qk, (uint64_t)krows, a.k_rs)) != cudaSuccess) return e;
  e = cudaFuncSetAttribute(mla::sfa_mla_sdp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  // the 128-key gradient pass (one latent gradient buffer) and its maps
  mlag::Plan gp;
  const char* gwhy = "";
  const bool grad_ok = mlag::plan(p, &gp, &gwhy);
  CUtensorMap tgq, tgdo;
  if (grad_ok) {
    gp.a.dk_acc = dk_acc;
    gp.a.status = device_status_ptr();
    e = make_tmap_bf16_4d(&tgq, p.q, {(uint64_t)p.d_qk, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                          {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)gp.a.HG, 1u, 1u});
    if (e == cudaSuccess)
      e = make_tmap_bf16_4d(&tgdo, p.dout, {(uint64_t)p.d_v, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                            {p.do_sh, p.do_st, p.do_sb}, {64u, (uint32_t)gp.a.HG, 1u, 1u});
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(mlag::sfa_mla_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gp.smem);
    if (e != cudaSuccess) return e;
  }
  for (int64_t r0 = 0; r0 < rows; r0 += wave) {
    const int64_t r1 = r0 + wave < rows ? r0 + wave : rows;
    a.r0 = (int)r0;
    a.nitems = (int)((r1 - r0) * p.h_kv * a.n_hh);
    const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
    mla::sfa_mla_sdp_kernel<<<grid, mla::kThreads, pl.smem, stream>>>(a, tq, tdo, tk);
    note_launch("bwd_mla_sdp", stream);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (grad_ok) {
      mlag::Args& g = gp.a;
      g.r0 = (int)r0;
      g.nitems = (int)((r1 - r0) * p.h_kv * g.n_hg * g.parts);
      CUtensorMap tp, tds;
      const uint64_t wr = (uint64_t)(r1 - r0);
      e = make_tmap_bf16_4d(&tp, a.pws, {(uint64_t)ld, (uint64_t)p.h_q, wr, 1u}, {ld, ld * p.h_q, ld * p.h_q * (int64_t)wr},
                            {64u, (uint32_t)g.HG, 1u, 1u});
      if (e == cudaSuccess)
        e = make_tmap_bf16_4d(&tds, a.dsws, {(uint64_t)ld, (uint64_t)p.h_q, wr, 1u},
                              {ld, ld * p.h_q, ld * p.h_q * (int64_t)wr}, {64u, (uint32_t)g.HG, 1u, 1u});
      if (e != cudaSuccess) return e;
      const int ggrid = g.nitems < device_sm_count() ? g.nitems : device_sm_count();
      mlag::sfa_mla_grad_kernel<<<ggrid, mlag::kThreads, gp.smem, stream>>>(g, tgq, tgdo, tk, tp, tds);
      note_launch("bwd_mla_grad", stream);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    } else {
      // separate dk / dv buffers: the token-level backward's two-pass form
      e = launch_bwd_tok_parts(p, dk_acc, dv_acc, a.pws, a.dsws, ld, (int)r0, (int)r1, stream);
      if (e != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

}  // namespace sfa
