// sfa_tc_fwd.cu — tensor-core SFA forward for sm_100a (tcgen05 + TMA + TMEM).
//
// Work item = (query row, kv head): the G <= 16 query heads of one kv group
// against that row's selected 64-key blocks.  G is too small for an MMA M
// dimension, so the kernel computes the transposed problem ("swap AB"):
//     S^T[keys, heads]  = K_sel[keys, D] . Q^T[D, heads]        (M = 128 keys, N = 16)
//     O^T[D, heads]    += V_sel^T[D, keys] . P^T[keys, heads]   (M = 128 dims, N = 16)
// with both accumulators in TMEM.  A segment of up to 1024 selected keys is
// scored completely before its softmax (so the max/sum need one cross-thread
// reduction per segment instead of per tile); segments of one row are merged in
// registers with the usual log-sum-exp rescale.
//
// Warp roles (192 threads, one persistent CTA per SM):
//   warp 0      TMA producer: compacts the row's valid block ids, loads Q and
//               gathers 64-key K/V blocks (one 4-D box per block and 64-dim
//               slab, 128B swizzle) into a ring of 128-key stages;
//   warp 1      MMA issuer (one thread): S^T for job j, then PV for job j-1;
//   warps 2-5   softmax (thread = key lane of a 128-key tile) and epilogue
//               (thread = dim lane of O^T): writes o (bf16) and lse (fp32).
// Hand-offs: mbarriers (TMA complete_tx, tcgen05.commit, thread arrivals).
// Every wait is bounded (~2 s); on expiry the kernel records a status word
// and returns.
//
// Replaces `_attn_fwd` / `_inner_fwd` (SFA.py:309-587): same math, no
// per-program global-memory workspaces, one gather per selected block per
// (row, kv head) instead of one per 32-head tile.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"

namespace sfa {
using namespace tc;

namespace fwd {

constexpr int kThreads = 192;
constexpr int kSegBlocks = 16;      // 64-key blocks per segment (1024 keys)
constexpr int kJD = 4;              // job descriptor ring depth
constexpr int kNH = 16;             // MMA N: query heads padded to 16
constexpr int kMaxTopk = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;       // 2 buffers x 8 tiles x 16 columns
constexpr uint32_t kColO = 256;     // 2 buffers x 16 columns

enum : int { kFirst = 1, kLast = 2, kSentinel = 4 };

struct JobDesc {
  int row, hk, b, tq, kv0, kv_len, pos, nblk, flags;
  int blocks[kSegBlocks];
};

template <int D>
struct Smem {
  static constexpr int kStages = D == 128 ? 4 : 8;
  static constexpr int kStageBytes = 128 * D * 2;   // 128 keys x D bf16
  static constexpr int kQBytes = kNH * D * 2;
  static constexpr int kPBytes = kSegBlocks * 64 * kNH * 2;
  alignas(1024) uint8_t stage[kStages][kStageBytes];
  alignas(1024) uint8_t q[2][kQBytes];
  alignas(1024) uint8_t p[2][kPBytes];
  JobDesc jd[kJD];
  float red[4][16];
  float ml[2][2][16];
  int plist[kMaxTopk];
  uint64_t stage_full[kStages], stage_empty[kStages];
  uint64_t q_full[2], q_empty[2];
  uint64_t s_full[2], s_empty[2], p_full[2], p_empty[2], o_full[2], o_empty[2];
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint32_t tmem_base;
  int abort_flag;
};

struct Args {
  SfaParams p;
  int nitems;
  int nrows;
  int oob_row;       // a kv row coordinate past the tensor map: zero-filled loads
  int32_t* status;
};

template <int D>
__device__ __forceinline__ bool wait_or_abort(Smem<D>& sm, uint64_t* bar, uint32_t parity, int32_t* status,
                                              int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (1 << 16) | site);
  atomicExch(&sm.abort_flag, 1);
  return false;
}

// Reduce 16 per-thread values over the 128 threads of warps 2-5; result for
// head h is written to out[h] (shared) and returned in v.
template <bool kMax, int D>
__device__ __forceinline__ void wg_reduce16(Smem<D>& sm, float (&v)[16], float* out, int wq, int lane, int tid) {
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    float x = v[h];
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      float y = __shfl_xor_sync(0xffffffffu, x, off);
      x = kMax ? fmaxf(x, y) : x + y;
    }
    v[h] = x;
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 16; ++h) sm.red[wq][h] = v[h];
  }
  named_barrier(1, 128);
  if (tid < 16) {
    float a = sm.red[0][tid], b = sm.red[1][tid], c = sm.red[2][tid], d = sm.red[3][tid];
    out[tid] = kMax ? fmaxf(fmaxf(a, b), fmaxf(c, d)) : (a + b) + (c + d);
  }
  named_barrier(1, 128);
#pragma unroll
  for (int h = 0; h < 16; ++h) v[h] = out[h];
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
sfa_fwd_tc_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                  const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int S = Smem<D>::kStages;
  const SfaParams& p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.h_q / p.h_kv;

  // ---------------------------------------------------------------- setup
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) { mbar_init(&sm.stage_full[i], 1); mbar_init(&sm.stage_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], 128);
      mbar_init(&sm.p_full[i], 128);
      mbar_init(&sm.p_empty[i], 1);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], 128);
    }
    for (int i = 0; i < kJD; ++i) { mbar_init(&sm.jd_full[i], 1); mbar_init(&sm.jd_empty[i], 1 + 128); }
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  // padded query rows (G..15) stay zero for the whole kernel
  for (int i = threadIdx.x; i < 2 * Smem<D>::kQBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(&sm.q[0][0])[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ============================================================ producer
    int job = 0, item_i = 0, use = 0;
    const uint32_t chunk_bytes = 128u * D * 2u;
    auto load_chunk = [&](const CUtensorMap* map, const JobDesc& d, int c) -> bool {
      const int s = use % S;
      if (!wait_or_abort(sm, &sm.stage_empty[s], ((use / S) & 1) ^ 1, args.status, 1)) return false;
      mbar_arrive_expect_tx(&sm.stage_full[s], chunk_bytes);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int bi = 2 * c + half;
        const int row = bi < d.nblk ? d.kv0 + d.blocks[bi] * 64 : args.oob_row;
#pragma unroll
        for (int cd = 0; cd < D / 64; ++cd)
          tma_load_4d(&sm.stage[s][cd * 128 * 128 + half * 64 * 128], map, &sm.stage_full[s], cd * 64, d.hk, row,
                      d.b);
      }
      ++use;
      return true;
    };
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x, ++item_i) {
      const int hk = item / args.nrows, row = item - hk * args.nrows;
      const Row r = row_info(p, row);
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      int n = 0;
      for (int s0 = 0; s0 < p.topk; s0 += 32) {
        const int s = s0 + lane;
        int e = -1;
        bool valid = false;
        if (s < p.topk) {
          e = __ldg(idx + s);
          valid = block_valid_keys(e, 64, r.kv_len, r.pos, p.causal) > 0;
        }
        const unsigned m = __ballot_sync(0xffffffffu, valid);
        if (valid) sm.plist[n + __popc(m & ((1u << lane) - 1u))] = e;
        n += __popc(m);
      }
      __syncwarp();
      const int nseg = n == 0 ? 1 : (n + kSegBlocks - 1) / kSegBlocks;
      if (lane == 0) {
        const int qs = item_i & 1;
        ok = wait_or_abort(sm, &sm.q_empty[qs], ((item_i >> 1) & 1) ^ 1, args.status, 2);
        if (ok) {
          mbar_arrive_expect_tx(&sm.q_full[qs], (uint32_t)(G * D * 2));
#pragma unroll
          for (int cd = 0; cd < D / 64; ++cd)
            tma_load_4d(&sm.q[qs][cd * kNH * 128], &tmq, &sm.q_full[qs], cd * 64, hk * G, (int)r.tq, r.b);
        }
        for (int seg = 0; seg < nseg && ok; ++seg, ++job) {
          const int js = job % kJD;
          ok = wait_or_abort(sm, &sm.jd_empty[js], ((job / kJD) & 1) ^ 1, args.status, 3);
          if (!ok) break;
          JobDesc& d = sm.jd[js];
          const int nb = n == 0 ? 0 : min(kSegBlocks, n - seg * kSegBlocks);
          d.row = row;
          d.hk = hk;
          d.b = r.b;
          d.tq = (int)r.tq;
          d.kv0 = (int)r.kv0;
          d.kv_len = r.kv_len;
          d.pos = r.pos;
          d.nblk = nb;
          d.flags = (seg == 0 ? kFirst : 0) | (seg == nseg - 1 ? kLast : 0);
          for (int i = 0; i < nb; ++i) d.blocks[i] = sm.plist[seg * kSegBlocks + i];
          mbar_arrive(&sm.jd_full[js]);
          for (int c = 0; c < (nb + 1) / 2 && ok; ++c) ok = load_chunk(&tmk, d, c);
          if (job > 0 && ok) {
            const JobDesc& pd = sm.jd[(job - 1) % kJD];
            for (int c = 0; c < (pd.nblk + 1) / 2 && ok; ++c) ok = load_chunk(&tmv, pd, c);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      job = __shfl_sync(0xffffffffu, job, 0);
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wait_or_abort(sm, &sm.jd_empty[js], ((job / kJD) & 1) ^ 1, args.status, 4)) {
        sm.jd[js].flags = kSentinel;
        mbar_arrive(&sm.jd_full[js]);
        if (job > 0) {
          const JobDesc& pd = sm.jd[(job - 1) % kJD];
          for (int c = 0; c < (pd.nblk + 1) / 2 && ok; ++c) ok = load_chunk(&tmv, pd, c);
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, kNH, false, false);
      const uint32_t id_o = idesc_bf16(128, kNH, true, true);
      // A = V tile as MN-major: 64-dim slabs LBO apart (D = 64 repeats the slab;
      // rows 64-127 of O^T are then ignored), 8-key groups 1024 B apart.
      const uint32_t lbo_v = D == 128 ? 128u * 128u : 0u;
      int job = 0, item_i = 0, use = 0;
      bool ok = true;
      auto pv = [&](int jj) -> bool {
        const JobDesc& d = sm.jd[jj % kJD];
        const int sb = jj & 1;
        if (!wait_or_abort(sm, &sm.p_full[sb], (jj >> 1) & 1, args.status, 10)) return false;
        if (!wait_or_abort(sm, &sm.o_empty[sb], ((jj >> 1) & 1) ^ 1, args.status, 11)) return false;
        tc_fence_after();
        const uint32_t dcol = tmem + kColO + sb * kNH;
        const uint32_t pbase = smem_u32(&sm.p[sb][0]);
        const int nch = (d.nblk + 1) / 2;
        for (int c = 0; c < nch; ++c) {
          const int s = use % S;
          if (!wait_or_abort(sm, &sm.stage_full[s], (use / S) & 1, args.status, 12)) return false;
          tc_fence_after();
          const uint32_t vbase = smem_u32(&sm.stage[s][0]);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = smem_desc(vbase + kk * 2048, lbo_v, 1024, kSw128);
            const uint64_t b = smem_desc(pbase + (c * 128 + kk * 16) * (kNH * 2), 0, 256, kSw32);
            mma_bf16_ss(dcol, a, b, id_o, (c | kk) != 0);
          }
          mma_commit(&sm.stage_empty[s]);
          ++use;
        }
        mma_commit(&sm.p_empty[sb]);
        mma_commit(&sm.o_full[sb]);
        mbar_arrive(&sm.jd_empty[jj % kJD]);
        return true;
      };
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wait_or_abort(sm, &sm.jd_full[js], (job / kJD) & 1, args.status, 13))) break;
        const JobDesc& d = sm.jd[js];
        if (d.flags & kSentinel) break;
        const int qs = item_i & 1;
        if (d.flags & kFirst)
          if (!(ok = wait_or_abort(sm, &sm.q_full[qs], (item_i >> 1) & 1, args.status, 14))) break;
        const int sb = job & 1;
        if (!(ok = wait_or_abort(sm, &sm.s_empty[sb], ((job >> 1) & 1) ^ 1, args.status, 15))) break;
        tc_fence_after();
        const uint32_t qbase = smem_u32(&sm.q[qs][0]);
        const int nch = (d.nblk + 1) / 2;
        for (int c = 0; c < nch && ok; ++c) {
          const int s = use % S;
          if (!(ok = wait_or_abort(sm, &sm.stage_full[s], (use / S) & 1, args.status, 16))) break;
          tc_fence_after();
          const uint32_t kbase = smem_u32(&sm.stage[s][0]);
          const uint32_t dcol = tmem + kColS + sb * 128 + c * kNH;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t a = smem_desc(kbase + (k >> 2) * (128 * 128) + (k & 3) * 32, 16, 1024, kSw128);
            const uint64_t b = smem_desc(qbase + (k >> 2) * (kNH * 128) + (k & 3) * 32, 16, 1024, kSw128);
            mma_bf16_ss(dcol, a, b, id_s, k != 0);
          }
          mma_commit(&sm.stage_empty[s]);
          ++use;
        }
        if (!ok) break;
        mma_commit(&sm.s_full[sb]);
        if (d.flags & kLast) {
          mma_commit(&sm.q_empty[qs]);
          ++item_i;
        }
        if (job > 0 && !(ok = pv(job - 1))) break;
        ++job;
      }
      if (ok && job > 0) pv(job - 1);
    }
  } else {
    // ============================================================ softmax / epilogue
    const int wq = warp & 3;             // TMEM lane quadrant of this warp
    const int tid = threadIdx.x - 64;    // 0..127
    const int lrow = wq * 32 + lane;     // TMEM lane: key (softmax) or dim (epilogue)
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    float acc[16], mrun[16], lrun[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) { acc[h] = 0.f; mrun[h] = -INFINITY; lrun[h] = 0.f; }
    bool ok = true;
    auto key_valid = [&](const JobDesc& d, int c) -> bool {
      const int bi = 2 * c + (lrow >> 6);
      if (bi >= d.nblk) return false;
      const int key = d.blocks[bi] * 64 + (lrow & 63);
      return key < d.kv_len && (!p.causal || key <= d.pos);
    };
    auto softmax = [&](int j) -> bool {
      const JobDesc& d = sm.jd[j % kJD];
      const int sb = j & 1;
      if (!wait_or_abort(sm, &sm.s_full[sb], (j >> 1) & 1, args.status, 20)) return false;
      tc_fence_after();
      const int nch = (d.nblk + 1) / 2;
      const uint32_t ts = tl + kColS + sb * 128;
      float m[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) m[h] = -INFINITY;
      for (int c = 0; c < nch; ++c) {
        float s[16];
        tmem_ld16(ts + c * kNH, s);
        tmem_ld_wait();
        if (key_valid(d, c)) {
#pragma unroll
          for (int h = 0; h < 16; ++h) m[h] = fmaxf(m[h], s[h] * c2);
        }
      }
      wg_reduce16<true>(sm, m, sm.ml[sb][0], wq, lane, tid);
      if (!wait_or_abort(sm, &sm.p_empty[sb], ((j >> 1) & 1) ^ 1, args.status, 21)) return false;
      float l[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) l[h] = 0.f;
      const uint32_t pbase = smem_u32(&sm.p[sb][0]);
      for (int c = 0; c < nch; ++c) {
        float s[16];
        tmem_ld16(ts + c * kNH, s);
        tmem_ld_wait();
        const bool v = key_valid(d, c);
        float pr[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          pr[h] = v ? exp2f(s[h] * c2 - m[h]) : 0.f;
          l[h] += pr[h];
        }
        // row = key within the segment; 32-byte rows, 32B swizzle (16-byte halves
        // swap when bit 2 of the row is set)
        const int rowk = c * 128 + lrow;
        const uint32_t off = pbase + rowk * 32;
        const uint32_t sw = ((rowk >> 2) & 1) << 4;
        st_shared_v4(off + sw, pack_bf16x2(pr[0], pr[1]), pack_bf16x2(pr[2], pr[3]), pack_bf16x2(pr[4], pr[5]),
                     pack_bf16x2(pr[6], pr[7]));
        st_shared_v4(off + (16 - sw), pack_bf16x2(pr[8], pr[9]), pack_bf16x2(pr[10], pr[11]),
                     pack_bf16x2(pr[12], pr[13]), pack_bf16x2(pr[14], pr[15]));
      }
      tc_fence_before();
      mbar_arrive(&sm.s_empty[sb]);
      fence_proxy_async_smem();
      mbar_arrive(&sm.p_full[sb]);
      wg_reduce16<false>(sm, l, sm.ml[sb][1], wq, lane, tid);
      return true;
    };
    auto epilogue = [&](int jj) -> bool {
      const JobDesc& d = sm.jd[jj % kJD];
      const int sb = jj & 1;
      if (d.flags & kFirst) {
#pragma unroll
        for (int h = 0; h < 16; ++h) { acc[h] = 0.f; mrun[h] = -INFINITY; lrun[h] = 0.f; }
      }
      if (!wait_or_abort(sm, &sm.o_full[sb], (jj >> 1) & 1, args.status, 22)) return false;
      tc_fence_after();
      if (d.nblk > 0) {
        float o[16];
        tmem_ld16(tl + kColO + sb * kNH, o);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float ms = sm.ml[sb][0][h], ls = sm.ml[sb][1][h];
          const float M = fmaxf(mrun[h], ms);
          const float a = exp2f(mrun[h] - M), bb = exp2f(ms - M);
          acc[h] = acc[h] * a + o[h] * bb;
          lrun[h] = lrun[h] * a + ls * bb;
          mrun[h] = M;
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.o_empty[sb]);
      if (d.flags & kLast) {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.o) + d.b * p.o_sb + (int64_t)d.tq * p.o_st +
                           (int64_t)(d.hk * G) * p.o_sh;
        float* lse = p.lse + d.b * p.l_sb + (int64_t)d.tq * p.l_st + (int64_t)(d.hk * G) * p.l_sh;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          if (h < G) {
            const float s2 = p.attn_sink ? __ldg(p.attn_sink + d.hk * G + h) * kLog2e : -INFINITY;
            const float M = fmaxf(mrun[h], s2);
            float outv = 0.f, lv = -INFINITY;
            if (M != -INFINITY) {
              const float lt = lrun[h] * exp2f(mrun[h] - M) + exp2f(s2 - M);
              outv = acc[h] * exp2f(mrun[h] - M) / lt;
              lv = (M + log2f(lt)) * kLn2;
            }
            if (lrow < D) o[h * p.o_sh + lrow] = f2bf(outv);
            if (lrow == h) lse[h * p.l_sh] = lv;
          }
        }
      }
      mbar_arrive(&sm.jd_empty[jj % kJD]);
      return true;
    };
    int job = 0;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wait_or_abort(sm, &sm.jd_full[js], (job / kJD) & 1, args.status, 23))) break;
      if (sm.jd[js].flags & kSentinel) break;
      if (!(ok = softmax(job))) break;
      if (job > 0 && !(ok = epilogue(job - 1))) break;
      ++job;
    }
    if (ok && job > 0) epilogue(job - 1);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int D>
cudaError_t launch(const SfaParams& p, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  const int G = p.h_q / p.h_kv;
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len, krows = vl ? p.total_kv : p.kv_len;
  const int64_t nb = vl ? 1 : p.batch;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)D, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)G, 1u, 1u});
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_4d(&tk, p.k, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                        {p.k_sh, p.k_st, p.k_sb}, {64u, 1u, 64u, 1u});
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_4d(&tv, p.v, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                        {p.v_sh, p.v_st, p.v_sb}, {64u, 1u, 64u, 1u});
  if (e != cudaSuccess) return e;
  Args a;
  a.p = p;
  a.nrows = num_rows_host(p);
  a.nitems = a.nrows * p.h_kv;
  a.oob_row = (int)krows;
  a.status = device_status_ptr();
  if (a.nitems == 0) return cudaSuccess;
  static_assert(sizeof(Smem<D>) + 1024 <= 227 * 1024, "shared memory budget");
  const size_t smem = sizeof(Smem<D>) + 1024;
  e = cudaFuncSetAttribute(sfa_fwd_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  sfa_fwd_tc_kernel<D><<<grid, kThreads, smem, st>>>(a, tq, tk, tv);
  note_launch();
  return cudaGetLastError();
}

}  // namespace fwd

bool tc_fwd_supported(const SfaParams& p, const char** why) {
  const int G = p.h_q / p.h_kv;
  if (device_cc() != 100) { *why = "needs an sm_100 device"; return false; }
  if (p.block_size != 64) { *why = "block_size must be 64"; return false; }
  if (p.topk > fwd::kMaxTopk) { *why = "topk must be <= 64"; return false; }
  if (p.d_qk != p.d_v || (p.d_qk != 64 && p.d_qk != 128)) { *why = "head dim must be 64 or 128 (D_qk == D_v)"; return false; }
  if (G > fwd::kNH) { *why = "query heads per kv head must be <= 16"; return false; }
  if (!tma_compatible(p.q, p.q_sb, p.q_st, p.q_sh) || !tma_compatible(p.k, p.k_sb, p.k_st, p.k_sh) ||
      !tma_compatible(p.v, p.v_sb, p.v_st, p.v_sh)) {
    *why = "q/k/v need 16-byte aligned base and strides";
    return false;
  }
  return true;
}

cudaError_t launch_fwd_tc(const SfaParams& p, cudaStream_t st) {
  return p.d_qk == 128 ? fwd::launch<128>(p, st) : fwd::launch<64>(p, st);
}

}  // namespace sfa
