// sfa_tc_bwd.cu — tensor-core SFA backward for sm_100a.
//
// dQ pass (query-centric, swap-AB like the forward).  Work item = (query row,
// kv head).  For every 128-key tile of the row's selected blocks:
//     S^T  = K . Q^T        dP^T = V . dO^T          (M = 128 keys, N = 16 heads)
//     dS^T = P^T o (dP^T - delta),  P^T = exp2(S^T*scale*log2e - lse2)
//     dQ^T += K^T . dS^T                              (M = 128 dims, N = 16 heads)
// lse comes from the forward, so no online softmax: every tile is independent
// and dQ^T accumulates in TMEM across all tiles of the row.  The K tile is used
// twice (K-major for S^T, MN-major for dQ^T) and held until the dQ MMA retires.
// Replaces `_attn_bwd_dq_dsink` / `_inner_dq` (SFA.py:613-716, 856-1002).
//
// dK/dV pass (key-centric).  Work item = (sequence, kv head, 64-key block e),
// taken from an atomic work counter; its query rows come from the inverted
// block->query index.  Rows are processed 8 queries x 16 heads = 128 at a time:
//     S  = Qb . K_e^T        dP = dOb . V_e^T         (M = 128 rows, N = 64 keys)
//     P = exp2(S*scale*log2e - lse2),  dS = P o (dP - delta)
//     dV^T += dOb^T . P      dK^T += Qb^T . dS        (M = 128 dims, N = 64 keys)
// dK^T/dV^T stay in TMEM for the whole block; each key block is written once,
// in a fixed order (no atomics): deterministic.  Replaces `_attn_bwd_dk_dv` /
// `_inner_dkv` (SFA.py:719-853, 1005-1145) and its fp32 atomics (SFA.py:853).
//
// Fused dQ (SFA_DQ_FUSED): the same pass also forms
//     dQ^T += K_e^T . dS^T                            (M = 128 dims, N = 128 rows)
// per batch and adds it to an fp32 [rows][h_q][d_qk] accumulator with
// coalesced fp32 reductions (a warp covers 32 dims of one row); the dQ pass
// above, which recomputes S and dP at N = 16, is then not run.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"

namespace sfa {
using namespace tc;

namespace bwd {

constexpr int kNH = 16;
constexpr int kMaxTopk = 64;
constexpr int kJD = 4;
enum : int { kSentinel = 4 };

// =========================================================================
// dQ
// =========================================================================
namespace dq {

constexpr int kThreads = 256;   // K producer, S/dP issuer, 4 dS warps, dQ issuer, V producer
constexpr int kR = 4;            // S/dP TMEM slots and dS smem slots
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColSdP = 0;  // kR x (16 S + 16 dP)
constexpr uint32_t kColDQ = 128; // 2 x 16

static_assert(kR >= 4, "stage-reuse waits on ds_empty/sdp_full assume kR > KS and kR > VS + 1");

struct JobDesc {
  int row, hk, b, tq, kv0, kv_len, pos, nblk, flags;
  int blocks[kMaxTopk];
  alignas(16) float lse2[kNH];   // lse * log2(e) of the row's heads (-inf past G); read as float4
  alignas(16) float dl[kNH];     // delta of the row's heads
};
static_assert(offsetof(JobDesc, lse2) % 16 == 0 && offsetof(JobDesc, dl) % 16 == 0, "float4 reads");

template <int D>
struct Smem {
  static constexpr int kKS = 3, kVS = 2;
  static constexpr int kStageBytes = 128 * D * 2;
  static constexpr int kQBytes = kNH * D * 2;
  alignas(1024) uint8_t kst[kKS][kStageBytes];
  alignas(1024) uint8_t vst[kVS][kStageBytes];
  alignas(1024) uint8_t q[2][kQBytes];
  alignas(1024) uint8_t dO[2][kQBytes];
  alignas(1024) uint8_t ds[kR][128 * kNH * 2];
  JobDesc jd[kJD];
  uint64_t k_full[kKS], v_full[kVS];
  uint64_t qdo_full[2], qdo_empty[2];
  uint64_t sdp_full[kR], sdp_empty[kR], ds_full[kR], ds_empty[kR];
  uint64_t dq_full[2], dq_empty[2];
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint32_t tmem_base;
};

struct Args {
  SfaParams p;
  const float* delta;
  int nitems, nrows, oob_row;
  int32_t* status;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (2 << 16) | site);
  return false;
}

// The same wait for a whole warp: every lane gets one verdict, so a warp that
// gives up leaves its later warp-wide instructions together.
__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
sfa_bwd_dq_tc_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                     const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KS = Smem<D>::kKS, VS = Smem<D>::kVS;
  const SfaParams& p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.h_q / p.h_kv;
  int32_t* st = args.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < KS; ++i) mbar_init(&sm.k_full[i], 1);
    for (int i = 0; i < VS; ++i) mbar_init(&sm.v_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.qdo_full[i], 1);
      mbar_init(&sm.qdo_empty[i], 1);
      mbar_init(&sm.dq_full[i], 1);
      mbar_init(&sm.dq_empty[i], 4);
    }
    for (int i = 0; i < kR; ++i) {
      mbar_init(&sm.sdp_full[i], 1);
      mbar_init(&sm.sdp_empty[i], 4);
      mbar_init(&sm.ds_full[i], 4);
      mbar_init(&sm.ds_empty[i], 1);
    }
    // consumers of a job descriptor: the two issuers, the V producer and the
    // 4 dS/epilogue warps (one arrival per warp)
    for (int i = 0; i < kJD; ++i) { mbar_init(&sm.jd_full[i], 1); mbar_init(&sm.jd_empty[i], 3 + 4); }
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 2 * Smem<D>::kQBytes / 16; i += kThreads) {
    reinterpret_cast<uint4*>(&sm.q[0][0])[i] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(&sm.dO[0][0])[i] = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmdo);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  const uint32_t chunk_bytes = 128u * D * 2u;
  // one 128-key stage = blocks row0 / row1 (a row past the tensor map reads
  // zeros) x D/64 slabs; coordinates in registers, so no shared-memory load
  // sits between two TMA issues
  auto load_chunk = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* full, int row0, int row1, int hk, int b) {
    mbar_arrive_expect_tx(full, chunk_bytes);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int cd = 0; cd < D / 64; ++cd)
        tma_load_4d(dst + cd * 128 * 128 + half * 64 * 128, map, full, cd * 64, hk, half ? row1 : row0, b);
    }
  };
  if (warp == 0) {
    // ============================================================ K producer
    int job = 0, g = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x, ++job) {
      const int hk = item / args.nrows, row = item - hk * args.nrows;
      const Row r = row_info(p, row);
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      const int js = job % kJD;
      if (lane == 0) ok = wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 1);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      JobDesc& d = sm.jd[js];
      // compact the valid block ids into d.blocks
      int n = 0;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int s = h2 * 32 + lane;
        int e = -1;
        bool valid = false;
        if (s < p.topk) {
          e = __ldg(idx + s);
          valid = block_valid_keys(e, 64, r.kv_len, r.pos, p.causal) > 0;
        }
        const unsigned m = __ballot_sync(0xffffffffu, valid);
        if (valid) d.blocks[n + __popc(m & ((1u << lane) - 1u))] = e;
        n += __popc(m);
      }
      __syncwarp();
      if (lane < kNH) {
        float l2 = -INFINITY, dlv = 0.f;
        if (lane < G) {
          l2 = p.lse[r.b * p.l_sb + r.tq * p.l_st + (int64_t)(hk * G + lane) * p.l_sh] * kLog2e;
          dlv = args.delta[(int64_t)row * p.h_q + hk * G + lane];
        }
        d.lse2[lane] = l2;
        d.dl[lane] = dlv;
      }
      if (lane == 0) {
        d.row = row;
        d.hk = hk;
        d.b = r.b;
        d.tq = (int)r.tq;
        d.kv0 = (int)r.kv0;
        d.kv_len = r.kv_len;
        d.pos = r.pos;
        d.nblk = n;
        d.flags = 0;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.jd_full[js]);
        const int ib = job & 1;
        ok = wt(&sm.qdo_empty[ib], ((job >> 1) & 1) ^ 1, st, 2);
        if (ok) {
          mbar_arrive_expect_tx(&sm.qdo_full[ib], (uint32_t)(2 * G * D * 2));
#pragma unroll
          for (int cd = 0; cd < D / 64; ++cd) {
            tma_load_4d(&sm.q[ib][cd * kNH * 128], &tmq, &sm.qdo_full[ib], cd * 64, hk * G, (int)r.tq, r.b);
            tma_load_4d(&sm.dO[ib][cd * kNH * 128], &tmdo, &sm.qdo_full[ib], cd * 64, hk * G, (int)r.tq, r.b);
          }
        }
      }
      if (lane == 0 && ok) {
        // block ids come from shared memory one tile ahead, so no load sits
        // between two TMA issues
        const int nch = (n + 1) / 2;
        int e0 = n > 0 ? d.blocks[0] : 0, e1 = n > 1 ? d.blocks[1] : 0;
        for (int c = 0; c < nch && ok; ++c, ++g) {
          const int row0 = (int)r.kv0 + e0 * 64;
          const int row1 = 2 * c + 1 < n ? (int)r.kv0 + e1 * 64 : args.oob_row;
          if (c + 1 < nch) {
            e0 = d.blocks[2 * c + 2];
            e1 = d.blocks[2 * c + 3];   // past n: never used
          }
          const int ks = g % KS;
          // a K stage is free once the dQ MMAs of tile g-KS retired (the same
          // commit that frees its dS slot); that barrier cannot complete its
          // next phase before this thread loads tile g+1
          if (g >= KS) ok = wt(&sm.ds_empty[(g - KS) % kR], ((g - KS) / kR) & 1, st, 3);
          if (ok) load_chunk(&tmk, sm.kst[ks], &sm.k_full[ks], row0, row1, hk, r.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      g = __shfl_sync(0xffffffffu, g, 0);
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 5)) {
        sm.jd[js].flags = kSentinel;
        mbar_arrive(&sm.jd_full[js]);
      }
    }
  } else if (warp == 7) {
    // ============================================================ V producer
    // Its own thread: one TMA-issuing thread alone limits the gather rate.
    if (lane == 0) {
      int job = 0, g = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 6))) break;
        const JobDesc& d = sm.jd[js];
        const int flags = d.flags;
        if (flags & kSentinel) break;
        const int n = d.nblk, kv0 = d.kv0, hk = d.hk, b = d.b;
        const int nch = (n + 1) / 2;
        int e0 = n > 0 ? d.blocks[0] : 0, e1 = n > 1 ? d.blocks[1] : 0;
        for (int c = 0; c < nch && ok; ++c, ++g) {
          const int row0 = kv0 + e0 * 64;
          const int row1 = 2 * c + 1 < n ? kv0 + e1 * 64 : args.oob_row;
          if (c + 1 < nch) {
            e0 = d.blocks[2 * c + 2];
            e1 = d.blocks[2 * c + 3];   // past n: never used
          }
          const int vs = g % VS;
          // a V stage is free once dP of tile g-VS retired (the commit that
          // hands S/dP to the dS warps); that barrier cannot complete its next
          // phase before this thread loads tile g+1
          if (g >= VS) ok = wt(&sm.sdp_full[(g - VS) % kR], ((g - VS) / kR) & 1, st, 4);
          if (ok) load_chunk(&tmv, sm.vst[vs], &sm.v_full[vs], row0, row1, hk, b);
        }
        if (!ok) break;
        mbar_arrive(&sm.jd_empty[js]);   // after the last read of the descriptor
        ++job;
      }
    }
  } else if (warp == 1) {
    // ============================================================ S/dP issuer
    if (lane == 0) {
      const uint32_t id_sdp = idesc_bf16(128, kNH, false, false);
      bool ok = true;
      int job = 0, g = 0;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 12))) break;
        // job fields go to registers once: a shared-memory load between MMAs
        // stalls this thread and leaves the tensor pipe without work
        const int flags = sm.jd[js].flags, nblk = sm.jd[js].nblk;
        if (flags & kSentinel) break;
        mbar_arrive(&sm.jd_empty[js]);
        const int ib = job & 1;
        if (!(ok = wt(&sm.qdo_full[ib], (job >> 1) & 1, st, 13))) break;
        const int nch = (nblk + 1) / 2;
        if (nch == 0) {
          mma_commit(&sm.qdo_empty[ib]);
          ++job;
          continue;
        }
        const uint64_t qdesc = smem_desc(smem_u32(&sm.q[ib][0]), 16, 1024, kSw128);
        const uint64_t odesc = smem_desc(smem_u32(&sm.dO[ib][0]), 16, 1024, kSw128);
        for (int c = 0; c < nch && ok; ++c, ++g) {
          const int slot = g % kR, ks = g % KS, vs = g % VS;
          if (!(ok = wt(&sm.sdp_empty[slot], ((g / kR) & 1) ^ 1, st, 15))) break;
          tc_fence_after();
          // TMA-filled stages: their mbarriers' complete_tx order them for the tensor core
          if (!(ok = wt(&sm.k_full[ks], (g / KS) & 1, st, 16))) break;
          if (!(ok = wt(&sm.v_full[vs], (g / VS) & 1, st, 17))) break;
          const uint64_t kdesc = smem_desc(smem_u32(&sm.kst[ks][0]), 16, 1024, kSw128);
          const uint64_t vdesc = smem_desc(smem_u32(&sm.vst[vs][0]), 16, 1024, kSw128);
          const uint32_t scol = tmem + kColSdP + slot * 32;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ko = (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4);
            const uint64_t qo = (uint64_t)(((k >> 2) * (kNH * 128) + (k & 3) * 32) >> 4);
            mma_bf16_ss(scol, kdesc + ko, qdesc + qo, id_sdp, k != 0);
          }
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t vo = (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4);
            const uint64_t oo = (uint64_t)(((k >> 2) * (kNH * 128) + (k & 3) * 32) >> 4);
            mma_bf16_ss(scol + 16, vdesc + vo, odesc + oo, id_sdp, k != 0);
          }
          mma_commit(&sm.sdp_full[slot]);   // also frees V stage vs
          if (c == nch - 1) mma_commit(&sm.qdo_empty[ib]);
        }
        ++job;
      }
    }
  } else if (warp == 6) {
    // ============================================================ dQ issuer
    // A second issuing thread: while one waits, the other's MMAs keep the
    // tensor pipe busy.
    if (lane == 0) {
      const uint32_t id_dq = idesc_bf16(128, kNH, true, true);
      const uint32_t lbo_k = D == 128 ? 128u * 128u : 0u;
      bool ok = true;
      int job = 0, g = 0;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 18))) break;
        const int flags = sm.jd[js].flags, nblk = sm.jd[js].nblk;
        if (flags & kSentinel) break;
        mbar_arrive(&sm.jd_empty[js]);
        const int ib = job & 1;
        if (!(ok = wt(&sm.dq_empty[ib], ((job >> 1) & 1) ^ 1, st, 11))) break;
        tc_fence_after();
        const int nch = (nblk + 1) / 2;
        const uint32_t dcol = tmem + kColDQ + ib * kNH;
        for (int c = 0; c < nch && ok; ++c, ++g) {
          const int slot = g % kR, ks = g % KS;
          if (!(ok = wt(&sm.ds_full[slot], (g / kR) & 1, st, 10))) break;
          tc_fence_after();
          const uint64_t a0 = smem_desc(smem_u32(&sm.kst[ks][0]), lbo_k, 1024, kSw128);
          const uint64_t b0 = smem_desc(smem_u32(&sm.ds[slot][0]), 0, 256, kSw32);
          // descriptors advance by adding the byte offset / 16 to the start-address field
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ss(dcol, a0 + (uint64_t)(kk * 2048 >> 4), b0 + (uint64_t)(kk * 16 * (kNH * 2) >> 4), id_dq,
                        (c == 0 && kk == 0) ? 0u : 1u);
          mma_commit(&sm.ds_empty[slot]);   // also frees K stage ks
        }
        if (!ok) break;
        mma_commit(&sm.dq_full[ib]);   // with no tiles this hands the epilogue an unwritten dQ: it writes zeros
        ++job;
      }
    }
  } else {
    // ============================================================ dS / epilogue
    const int wq = warp & 3;
    const int lrow = wq * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    int job = 0, g = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&sm.jd_full[js], (job / kJD) & 1, st, 20))) break;
      const JobDesc& d = sm.jd[js];
      if (d.flags & kSentinel) break;
      const int ib = job & 1;
      float lse2[16], dl[16];
#pragma unroll
      for (int h4 = 0; h4 < 4; ++h4) {
        const float4 a = reinterpret_cast<const float4*>(d.lse2)[h4];
        const float4 b = reinterpret_cast<const float4*>(d.dl)[h4];
        lse2[4 * h4] = a.x; lse2[4 * h4 + 1] = a.y; lse2[4 * h4 + 2] = a.z; lse2[4 * h4 + 3] = a.w;
        dl[4 * h4] = b.x; dl[4 * h4 + 1] = b.y; dl[4 * h4 + 2] = b.z; dl[4 * h4 + 3] = b.w;
      }
      const int nch = (d.nblk + 1) / 2;
      for (int c = 0; c < nch && ok; ++c, ++g) {
        const int slot = g % kR;
        if (!(ok = wtw(&sm.sdp_full[slot], (g / kR) & 1, st, 21))) break;
        tc_fence_after();
        float s[16], dp[16];
        tmem_ld16(tl + kColSdP + slot * 32, s);
        tmem_ld16(tl + kColSdP + slot * 32 + 16, dp);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(&sm.sdp_empty[slot]);
        const int bi = 2 * c + (lrow >> 6);
        bool valid = bi < d.nblk;
        if (valid) {
          const int key = d.blocks[bi] * 64 + (lrow & 63);
          valid = key < d.kv_len && (!p.causal || key <= d.pos);
        }
        float ds[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float pr = (valid && lse2[h] != -INFINITY) ? ex2(s[h] * c2 - lse2[h]) : 0.f;
          ds[h] = pr * (dp[h] - dl[h]);
        }
        if (!(ok = wtw(&sm.ds_empty[slot], ((g / kR) & 1) ^ 1, st, 22))) break;
        const uint32_t off = smem_u32(&sm.ds[slot][0]) + lrow * 32;
        const uint32_t sw = ((lrow >> 2) & 1) << 4;
        st_shared_v4(off + sw, pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]), pack_bf16x2(ds[4], ds[5]),
                     pack_bf16x2(ds[6], ds[7]));
        st_shared_v4(off + (16 - sw), pack_bf16x2(ds[8], ds[9]), pack_bf16x2(ds[10], ds[11]),
                     pack_bf16x2(ds[12], ds[13]), pack_bf16x2(ds[14], ds[15]));
        fence_proxy_async_smem();
        warp_arrive(&sm.ds_full[slot]);
      }
      if (!ok) break;
      // epilogue: dq = scale * dQ^T (thread = dim)
      if (!(ok = wtw(&sm.dq_full[ib], (job >> 1) & 1, st, 23))) break;
      tc_fence_after();
      float acc[16];
      if (nch > 0) {
        tmem_ld16(tl + kColDQ + ib * kNH, acc);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) acc[h] = 0.f;
      }
      tc_fence_before();
      warp_arrive(&sm.dq_empty[ib]);
      if (lrow < D) {
        __nv_bfloat16* dqp = reinterpret_cast<__nv_bfloat16*>(p.dq) + d.b * p.dq_sb + (int64_t)d.tq * p.dq_st +
                             (int64_t)(d.hk * G) * p.dq_sh + lrow;
#pragma unroll
        for (int h = 0; h < 16; ++h)
          if (h < G) dqp[h * p.dq_sh] = f2bf(acc[h] * p.scale);
      }
      warp_arrive(&sm.jd_empty[js]);
      ++job;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int D>
cudaError_t launch(const SfaParams& p, const float* delta, cudaStream_t stream) {
  CUtensorMap tq, tdo, tk, tv;
  const int G = p.h_q / p.h_kv;
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len, krows = vl ? p.total_kv : p.kv_len;
  const int64_t nb = vl ? 1 : p.batch;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)D, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)G, 1u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tdo, p.dout, {(uint64_t)D, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                          {p.do_sh, p.do_st, p.do_sb}, {64u, (uint32_t)G, 1u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tk, p.k, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                          {p.k_sh, p.k_st, p.k_sb}, {64u, 1u, 64u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tv, p.v, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                          {p.v_sh, p.v_st, p.v_sb}, {64u, 1u, 64u, 1u});
  if (e != cudaSuccess) return e;
  Args a;
  a.p = p;
  a.delta = delta;
  a.nrows = num_rows_host(p);
  a.nitems = a.nrows * p.h_kv;
  a.oob_row = (int)krows;
  a.status = device_status_ptr();
  if (a.nitems == 0) return cudaSuccess;
  static_assert(sizeof(Smem<D>) + 1024 <= 227 * 1024, "shared memory budget");
  const size_t smem = sizeof(Smem<D>) + 1024;
  e = cudaFuncSetAttribute(sfa_bwd_dq_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  sfa_bwd_dq_tc_kernel<D><<<grid, kThreads, smem, stream>>>(a, tq, tdo, tk, tv);
  note_launch("bwd_dq_tc", stream);
  return cudaGetLastError();
}

}  // namespace dq

// =========================================================================
// dK / dV (key-centric over the inverted index)
// =========================================================================
namespace dkdv {

constexpr int kThreads = 384;       // warp 0 metadata, 1 S/dP issuer, 2-9 P/dS + epilogue, 10 loads,
                                    // 11 dV/dK issuer
constexpr int kThreadsDQ = 640;     // + warps 12-19: fused-dQ reducers (two per TMEM lane quadrant);
                                    // 20 warps leave 96 registers a thread (21 would leave 80)
constexpr int kWG = 256;            // P/dS threads: 2 warpgroups, each takes 32 of the 64 keys
constexpr int kQB = 8;              // queries per batch (x 16 heads = 128 MMA rows)
constexpr int kMeta = 6;            // batch metadata ring depth
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColSdP = 0;     // 2 slots x (64 S + 64 dP)
constexpr uint32_t kColAcc = 256;   // 2 buffers x (64 dV^T + 64 dK^T); 1 buffer with the fused dQ
constexpr uint32_t kColDQ = 384;    // fused dQ: dQ^T partial of one batch (128 dims x 128 rows)

struct JobDesc {
  int e, b, hk, kv0, kv_len, n, list0, flags;
  int64_t part;   // row-range split: this job's fp32 dK/dV partial slot, else -1
};

// Per-batch metadata of the queries of one batch, written by the metadata warp
// ahead of the loads: TMA coordinates of each query, its causal position and
// its row id (lse and delta are fetched by the P/dS threads themselves).
struct BatchMeta {
  int tq[kQB], b[kQB], pos[kQB], rowid[kQB];
  int m;                  // queries in the batch
};

template <int D>
struct Smem {
  static constexpr int kBatchBytes = 128 * D * 2;   // 128 rows x D bf16
  static constexpr int kKVBytes = 64 * D * 2;       // 64 keys x D bf16
  alignas(1024) uint8_t qb[2][kBatchBytes];
  alignas(1024) uint8_t dob[2][kBatchBytes];
  alignas(1024) uint8_t ke[kKVBytes];
  alignas(1024) uint8_t ve[kKVBytes];
  alignas(1024) uint8_t pbuf[128 * 64 * 2];
  alignas(1024) uint8_t dsbuf[128 * 64 * 2];
  JobDesc jd[kJD];
  alignas(16) BatchMeta meta[kMeta];
  uint64_t bq_full[2], bdo_full[2], b_empty[2], kv_full, kv_empty;
  uint64_t meta_full[kMeta], meta_empty[kMeta];
  // S and dP of a batch land separately (s_full, dp_full), and P and dS go
  // back separately (p_full, ds_full): P's exponentials overlap the dP MMAs
  // and the dV MMAs overlap the dS math
  uint64_t s_full[2], dp_full[2], sdp_empty[2], p_full, p_empty, ds_full, ds_empty;
  uint64_t acc_full[2], acc_empty[2];
  uint64_t dq_full, dq_empty;         // fused dQ partial (TMEM) hand-off
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint32_t tmem_base;
};

struct Args {
  SfaParams p;
  const float* delta;
  float* dq_acc;            // fused dQ: fp32 [rows][h_q][d_qk] accumulator (zeroed by the host), else null
  const int32_t* offsets;   // [units * nblk + 1]
  const int32_t* entries;   // query rows
  // Row ranges: with nranges > 1 a job is (range, unit, block) and covers the
  // block's queries in rows [r*range_rows, (r+1)*range_rows) of its sequence;
  // starts[] (the index builder's scanned sub-chunk counts) gives where each
  // range starts in the list; the job writes an fp32 dK/dV partial to
  // part[(unit*nblk + block)*nranges + r] and a reduction sums the ranges.
  const int32_t* starts;    // [units * nblk * nsub] list position of each 128-row sub-chunk
  float* part;              // [units * nblk * nranges][2][64][D] (dK then dV), or null
  int nsub, sub_per_range, nranges;
  int* sched;               // work counter (zeroed by the host)
  int units, nblk, nitems;
  int32_t* status;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (3 << 16) | site);
  return false;
}

// The same wait for a whole warp: every lane gets one verdict, so a warp that
// gives up leaves its later warp-wide instructions together.
__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

template <int D, bool kDQ>
__global__ void __launch_bounds__(kDQ ? kThreadsDQ : kThreads, 1)
sfa_bwd_dkdv_tc_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                       const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaParams& p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.h_q / p.h_kv;
  int32_t* st = args.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.bq_full[i], 1);
      mbar_init(&sm.bdo_full[i], 1);
      mbar_init(&sm.b_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.dp_full[i], 1);
      mbar_init(&sm.sdp_empty[i], kWG / 32);
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], kWG / 32);
    }
    // counts in warps for the P/dS warps (one arrival per warp)
    for (int i = 0; i < kMeta; ++i) {
      mbar_init(&sm.meta_full[i], 1);
      mbar_init(&sm.meta_empty[i], 1 + kWG / 32 + (kDQ ? 8 : 0));   // loader warp, P/dS warps, reducers
    }
    mbar_init(&sm.kv_full, 1);
    mbar_init(&sm.kv_empty, 1);
    mbar_init(&sm.p_full, kWG / 32);
    mbar_init(&sm.p_empty, 1);
    mbar_init(&sm.ds_full, kWG / 32);
    mbar_init(&sm.ds_empty, 1);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_empty, 8);   // the 8 reducer warps
    // consumers of a job descriptor: the two issuers, the loader warp, the
    // P/dS warps and (fused dQ) the reducer warps
    for (int i = 0; i < kJD; ++i) {
      mbar_init(&sm.jd_full[i], 1);
      mbar_init(&sm.jd_empty[i], 3 + kWG / 32 + (kDQ ? 8 : 0));
    }
    fence_barrier_init();
  }
  // padded head rows (G..15 of every query) stay zero
  for (int i = threadIdx.x; i < 2 * Smem<D>::kBatchBytes / 16; i += blockDim.x) {
    reinterpret_cast<uint4*>(&sm.qb[0][0])[i] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(&sm.dob[0][0])[i] = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 10 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmdo);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ============================================================ scheduler + metadata
    // Items run unit-major (all blocks of one (sequence, kv head) before the
    // next), so the CTAs working at one time share that unit's Q/dO in L2; the
    // lowest blocks, which have the longest query lists, start first.
    int job = 0, gb = 0;
    bool ok = true;
    while (ok) {
      int item = 0;
      if (lane == 0) item = atomicAdd(args.sched, 1);
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item >= args.nitems) break;
      const int per_range = args.units * args.nblk;
      const int r = item / per_range, ue = item - r * per_range;
      const int u = ue / args.nblk, e = ue - u * args.nblk;
      const int seq = u / p.h_kv, hk = u - seq * p.h_kv;
      int kv0 = 0, kv_len = p.kv_len, b = seq;
      if (p.cu_seqlens_q != nullptr) {
        kv0 = __ldg(p.cu_seqlens_k + seq);
        kv_len = __ldg(p.cu_seqlens_k + seq + 1) - kv0;
        b = 0;
      }
      if (e * 64 >= kv_len) continue;   // past this sequence's last block
      int list0, n;
      if (args.nranges > 1) {
        // [start of range r, start of range r+1) inside the block's list
        const int64_t sb = ((int64_t)u * args.nblk + e) * args.nsub;
        const int s0 = r * args.sub_per_range, s1 = s0 + args.sub_per_range;
        list0 = __ldg(args.starts + sb + s0);
        const int end = s1 < args.nsub ? __ldg(args.starts + sb + s1)
                                        : __ldg(args.offsets + (int64_t)u * args.nblk + e + 1);
        n = end - list0;
        if (n == 0) continue;   // no query of this range: no partial (the reduction skips it)
      } else {
        list0 = __ldg(args.offsets + (int64_t)u * args.nblk + e);
        n = __ldg(args.offsets + (int64_t)u * args.nblk + e + 1) - list0;
      }
      const int js = job % kJD;
      if (lane == 0) {
        ok = wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 1);
        if (ok) {
          JobDesc& d = sm.jd[js];
          d.e = e;
          d.b = b;
          d.hk = hk;
          d.kv0 = kv0;
          d.kv_len = kv_len;
          d.n = n;
          d.list0 = list0;
          d.flags = 0;
          d.part = args.nranges > 1 ? ((int64_t)u * args.nblk + e) * args.nranges + r : -1;
          mbar_arrive(&sm.jd_full[js]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      const int nb = (n + kQB - 1) / kQB;
      for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
        const int slot = gb % kMeta;
        if (lane == 0) ok = wt(&sm.meta_empty[slot], ((gb / kMeta) & 1) ^ 1, st, 2);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        const int m = min(kQB, n - jb * kQB);
        int tq = 0, bb = 0, rowid = 0, pos = 0;
        if (lane < m) {
          rowid = __ldg(args.entries + list0 + jb * kQB + lane);
          const Row r = row_info(p, rowid);
          tq = (int)r.tq;
          bb = r.b;
          pos = r.pos;
        }
        BatchMeta& mt = sm.meta[slot];
        if (lane < kQB) {
          mt.tq[lane] = tq;
          mt.b[lane] = bb;
          mt.pos[lane] = pos;
          mt.rowid[lane] = rowid;
        }
        if (lane == 0) mt.m = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.meta_full[slot]);
      }
      ++job;
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 4)) {
        sm.jd[js].flags = kSentinel;
        mbar_arrive(&sm.jd_full[js]);
      }
    }
  } else if (warp == 10) {
    // ============================================================ TMA loads
    // One loader warp: lane 0 gathers K_e / V_e, lanes 0-7 the batch's Q rows
    // (query = lane) and lanes 8-15 its dO rows (query = lane - 8).  Each
    // 16-head row is a 2 KB box and one thread issues about one box per 100
    // cycles, so the batch's 32 boxes leave from 16 lanes at once.
    const bool is_q = lane < kQB;
    const int qj = lane & (kQB - 1);
    const CUtensorMap* map = is_q ? &tmq : &tmdo;
    int job = 0, gb = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&sm.jd_full[js], (job / kJD) & 1, st, 5))) break;
      const JobDesc& d = sm.jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      const int hk = d.hk, n = d.n, krow = d.kv0 + d.e * 64, kb = d.b;
      warp_arrive(&sm.jd_empty[js]);
      if (lane == 0) {
        ok = wt(&sm.kv_empty, (job & 1) ^ 1, st, 6);
        if (ok) {
          mbar_arrive_expect_tx(&sm.kv_full, 2u * 64u * D * 2u);
#pragma unroll
          for (int cd = 0; cd < D / 64; ++cd) {
            tma_load_4d(&sm.ke[cd * 64 * 128], &tmk, &sm.kv_full, cd * 64, hk, krow, kb);
            tma_load_4d(&sm.ve[cd * 64 * 128], &tmv, &sm.kv_full, cd * 64, hk, krow, kb);
          }
        }
      }
      if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
      const int nb = (n + kQB - 1) / kQB;
      for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
        const int slot = gb % kMeta, s = gb & 1;
        if (!(ok = wtw(&sm.meta_full[slot], (gb / kMeta) & 1, st, 7))) break;
        const BatchMeta& mt = sm.meta[slot];
        const int m = mt.m;
        const int tq = mt.tq[qj], bq = mt.b[qj];
        warp_arrive(&sm.meta_empty[slot]);
        if (!(ok = wtw(&sm.b_empty[s], ((gb >> 1) & 1) ^ 1, st, 3))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&sm.bq_full[s], (uint32_t)(m * G * D * 2));
          mbar_arrive_expect_tx(&sm.bdo_full[s], (uint32_t)(m * G * D * 2));
        }
        __syncwarp();
        if (lane < 2 * kQB && qj < m) {
          uint64_t* full = is_q ? &sm.bq_full[s] : &sm.bdo_full[s];
          uint8_t* buf = is_q ? sm.qb[s] : sm.dob[s];
#pragma unroll
          for (int cd = 0; cd < D / 64; ++cd)
            tma_load_4d(buf + cd * 128 * 128 + qj * 16 * 128, map, full, cd * 64, hk * G, tq, bq);
        }
      }
      ++job;
    }
  } else if (warp == 1) {
    // ============================================================ S/dP issuer
    if (lane == 0) {
      const uint32_t id_sdp = idesc_bf16(128, 64, false, false);
      bool ok = true;
      int job = 0, gb = 0;
      const uint64_t kd = smem_desc(smem_u32(&sm.ke[0]), 16, 1024, kSw128);
      const uint64_t vd = smem_desc(smem_u32(&sm.ve[0]), 16, 1024, kSw128);
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 12))) break;
        // job fields go to registers once: a shared-memory load between MMAs
        // stalls this thread and leaves the tensor pipe without work
        const int flags = sm.jd[js].flags, n = sm.jd[js].n;
        if (flags & kSentinel) break;
        mbar_arrive(&sm.jd_empty[js]);
        // K_e / V_e are TMA-filled: the mbarrier's complete_tx orders them for the tensor core
        if (!(ok = wt(&sm.kv_full, job & 1, st, 13))) break;
        const int nb = (n + kQB - 1) / kQB;
        for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
          const int s = gb & 1;
          if (!(ok = wt(&sm.sdp_empty[s], ((gb >> 1) & 1) ^ 1, st, 15))) break;
          tc_fence_after();
          const uint64_t qd = smem_desc(smem_u32(&sm.qb[s][0]), 16, 1024, kSw128);
          const uint64_t od = smem_desc(smem_u32(&sm.dob[s][0]), 16, 1024, kSw128);
          const uint32_t scol = tmem + kColSdP + s * 128;
          if (!(ok = wt(&sm.bq_full[s], (gb >> 1) & 1, st, 16))) break;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ro = (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4);
            const uint64_t ko = (uint64_t)(((k >> 2) * (64 * 128) + (k & 3) * 32) >> 4);
            mma_bf16_ss(scol, qd + ro, kd + ko, id_sdp, k != 0);
          }
          mma_commit(&sm.s_full[s]);
          if (!(ok = wt(&sm.bdo_full[s], (gb >> 1) & 1, st, 18))) break;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint64_t ro = (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4);
            const uint64_t ko = (uint64_t)(((k >> 2) * (64 * 128) + (k & 3) * 32) >> 4);
            mma_bf16_ss(scol + 64, od + ro, vd + ko, id_sdp, k != 0);
          }
          mma_commit(&sm.dp_full[s]);
        }
        if (!ok) break;
        // K_e / V_e are free once their last reader retires: these S/dP MMAs,
        // or with the fused dQ the dQ MMAs of the job's last batch (the other
        // issuer commits then)
        if (!kDQ || nb == 0) mma_commit(&sm.kv_empty);
        ++job;
      }
    }
  } else if (warp == 11) {
    // ============================================================ dV/dK (and dQ) issuer
    // A second issuing thread: while one waits, the other's MMAs keep the
    // tensor pipe busy.
    if (lane == 0) {
      const uint32_t id_acc = idesc_bf16(128, 64, true, true);
      // fused dQ: dQ^T[dims, rows] = K_e^T[dims, keys] . dS^T[keys, rows]
      // (A = K_e read MN-major: 64-dim slabs 8 KB apart, 8-key groups 1 KB
      // apart; B = dS read K-major: 8-row groups 1 KB apart)
      const uint32_t id_dq = idesc_bf16(128, 128, true, false);
      const uint32_t lbo_rows = D == 128 ? 128u * 128u : 0u;   // 64-dim slabs of the 128-row buffers
      const uint64_t pdsc = smem_desc(smem_u32(&sm.pbuf[0]), 0, 1024, kSw128);
      const uint64_t dd = smem_desc(smem_u32(&sm.dsbuf[0]), 0, 1024, kSw128);
      const uint64_t kdq = smem_desc(smem_u32(&sm.ke[0]), D == 128 ? 64u * 128u : 0u, 1024, kSw128);
      const uint64_t ddq = smem_desc(smem_u32(&sm.dsbuf[0]), 16, 1024, kSw128);
      constexpr int kNAcc = kDQ ? 1 : 2;   // accumulator buffers
      bool ok = true;
      int job = 0, gb = 0;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 17))) break;
        const int flags = sm.jd[js].flags, n = sm.jd[js].n;
        if (flags & kSentinel) break;
        mbar_arrive(&sm.jd_empty[js]);
        const int ab = job % kNAcc, use = job / kNAcc;
        if (!(ok = wt(&sm.acc_empty[ab], (use & 1) ^ 1, st, 11))) break;
        tc_fence_after();
        const int nb = (n + kQB - 1) / kQB;
        const uint32_t acc = tmem + kColAcc + ab * 128;
        for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
          const int s = gb & 1;
          const uint64_t od = smem_desc(smem_u32(&sm.dob[s][0]), lbo_rows, 1024, kSw128);
          const uint64_t qd = smem_desc(smem_u32(&sm.qb[s][0]), lbo_rows, 1024, kSw128);
          // dV^T += dOb^T . P as soon as P is in (16 rows per K-step: +2048
          // bytes = +128 in the start-address field).  P is made from S
          // alone, so p_full says nothing about the batch's dO rows: wait for
          // their copy here (the slot cannot refill before this batch's dK
          // MMAs retire, so the parity is unambiguous).
          if (!(ok = wt(&sm.p_full, gb & 1, st, 10))) break;
          if (!(ok = wt(&sm.bdo_full[s], (gb >> 1) & 1, st, 30))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ss(acc, od + (uint64_t)(kk * 128), pdsc + (uint64_t)(kk * 128), id_acc, (jb | kk) != 0);
          mma_commit(&sm.p_empty);
          // dK^T += Qb^T . dS
          if (!(ok = wt(&sm.ds_full, gb & 1, st, 9))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ss(acc + 64, qd + (uint64_t)(kk * 128), dd + (uint64_t)(kk * 128), id_acc, (jb | kk) != 0);
          // the last readers of the batch's Q / dO rows (the S/dP MMAs retired
          // before its P/dS were written): the slot goes back to the loader
          // now, not after the dQ MMAs below
          mma_commit(&sm.b_empty[s]);
          if (kDQ) {
            // the reducer warps have read the previous batch's partial out of TMEM
            if (!(ok = wt(&sm.dq_empty, (gb & 1) ^ 1, st, 19))) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)   // 16 keys per step: +2048 B of K_e, +32 B of dS rows
              mma_bf16_ss(tmem + kColDQ, kdq + (uint64_t)(kk * 128), ddq + (uint64_t)(kk * 2), id_dq, kk != 0);
            mma_commit(&sm.dq_full);   // also: dS read by the dK and dQ MMAs (the P/dS warps wait on it)
          } else {
            mma_commit(&sm.ds_empty);   // dS read by the dK MMAs
          }
        }
        if (!ok) break;
        if (kDQ && nb > 0) mma_commit(&sm.kv_empty);   // the dQ MMAs read K_e
        mma_commit(&sm.acc_full[ab]);   // with no batches the epilogue writes zeros
        ++job;
      }
    }
  } else if (kDQ && warp >= 12) {
    // ============================================================ fused-dQ reducers (warps 12-19)
    // thread = dim (TMEM lane); per batch the dQ^T partial's 128 columns are
    // the batch's 8 queries x 16 heads, and each quadrant has two reducer
    // warps: warps 12-15 take queries 0-3, warps 16-19 queries 4-7.  A warp
    // reads its 64 columns at once and releases the partial before issuing
    // its reductions, so the next batch's dQ MMAs need not wait for them; each
    // reduction adds 32 dims of one (query, head) row: coalesced 128 bytes.
    const int wq = warp & 3;
    const int q0 = ((warp - 12) >> 2) * 4;   // first query of this warp's half
    const int dim = wq * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    int job = 0, gb = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&sm.jd_full[js], (job / kJD) & 1, st, 26))) break;
      const JobDesc& d = sm.jd[js];
      if (d.flags & kSentinel) break;
      const int hk = d.hk, nb = (d.n + kQB - 1) / kQB;
      warp_arrive(&sm.jd_empty[js]);
      for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
        const int slot = gb % kMeta;
        if (!(ok = wtw(&sm.meta_full[slot], (gb / kMeta) & 1, st, 27))) break;
        const BatchMeta& mt = sm.meta[slot];
        const int m = mt.m;
        int rid[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) rid[j] = q0 + j < m ? mt.rowid[q0 + j] : -1;
        warp_arrive(&sm.meta_empty[slot]);
        if (!(ok = wtw(&sm.dq_full, gb & 1, st, 25))) break;
        tc_fence_after();
        float part[4][16];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_ld16(tl + kColDQ + (q0 + j) * 16, part[j]);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(&sm.dq_empty);
        if (dim < D) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (rid[j] >= 0) {
              float* dst = args.dq_acc + ((int64_t)rid[j] * p.h_q + hk * G) * D + dim;
#pragma unroll
              for (int hh = 0; hh < 16; ++hh)
                if (hh < G) atomicAdd(dst + hh * D, part[j][hh]);
            }
          }
        }
      }
      ++job;
    }
  } else {
    // ============================================================ P/dS and epilogue (warps 2-9)
    // thread = TMEM lane (row = (query j, head h)); warpgroup wg takes keys
    // 32*wg .. 32*wg+31 of the block (columns of S/dP, 64-byte halves of the
    // P/dS rows); in the epilogue thread = dim and wg takes the same keys.
    const int wg = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int lrow = wq * 32 + lane;
    const int jq = lrow >> 4, h = lrow & 15;
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    const bool shared_kv = p.dk == p.dv;
    constexpr int kNAcc = kDQ ? 1 : 2;
    int job = 0, gb = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&sm.jd_full[js], (job / kJD) & 1, st, 20))) break;
      const JobDesc& d = sm.jd[js];
      if (d.flags & kSentinel) break;
      const int ab = job % kNAcc, use = job / kNAcc;
      const int nb = (d.n + kQB - 1) / kQB;
      const int key_base = d.e * 64 + wg * 32;
      const int kv_len = d.kv_len;
      for (int jb = 0; jb < nb && ok; ++jb, ++gb) {
        const int s = gb & 1, slot = gb % kMeta;
        if (!(ok = wtw(&sm.meta_full[slot], (gb / kMeta) & 1, st, 24))) break;
        const BatchMeta& mt = sm.meta[slot];
        // this thread's (query, head) row: lse and delta straight from global
        // memory, issued after the slot is released (the arrive's release
        // would otherwise wait for them), so their latency overlaps the wait
        // for S/dP below
        const int pos = mt.pos[jq], qb_ = mt.b[jq], qtq = mt.tq[jq], qrow = mt.rowid[jq];
        const bool live = jq < mt.m && h < G;
        warp_arrive(&sm.meta_empty[slot]);
        float lse2 = -INFINITY, dl = 0.f;
        if (live) {
          const int hh = d.hk * G + h;
          lse2 = __ldg(p.lse + qb_ * p.l_sb + (int64_t)qtq * p.l_st + (int64_t)hh * p.l_sh) * kLog2e;
          dl = __ldg(args.delta + (int64_t)qrow * p.h_q + hh);
        }
        // S first: P = exp2(S*scale*log2e - lse2) goes out while dP is computed
        if (!(ok = wtw(&sm.s_full[s], (gb >> 1) & 1, st, 21))) break;
        tc_fence_after();
        const uint32_t col = tl + kColSdP + s * 128 + wg * 32;
        float pv[32];
        tmem_ld16(col, *reinterpret_cast<float(*)[16]>(&pv[0]));
        tmem_ld16(col + 16, *reinterpret_cast<float(*)[16]>(&pv[16]));
        tmem_ld_wait();
        // keys of this warpgroup valid for this row: key_base + i < lim
        const int lim = lse2 != -INFINITY ? min(kv_len, p.causal ? pos + 1 : kv_len) - key_base : 0;
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          pv[i] = i < lim ? ex2(pv[i] * c2 - lse2) : 0.f;
          pv[i + 1] = i + 1 < lim ? ex2(pv[i + 1] * c2 - lse2) : 0.f;
          pk[i / 2] = pack_bf16x2(pv[i], pv[i + 1]);
        }
        // row lrow: 64 keys = 8 chunks of 16 bytes, 128B swizzle (chunk ^= row & 7);
        // this warpgroup writes chunks 4*wg .. 4*wg+3
        const uint32_t prow = smem_u32(&sm.pbuf[0]) + lrow * 128;
        const uint32_t drow = smem_u32(&sm.dsbuf[0]) + lrow * 128;
        if (!(ok = wtw(&sm.p_empty, (gb & 1) ^ 1, st, 22))) break;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t off = (uint32_t)(((wg * 4 + c) ^ (lrow & 7)) * 16);
          st_shared_v4(prow + off, pk[c * 4], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
        }
        fence_proxy_async_smem();
        warp_arrive(&sm.p_full);
        // then dP: dS = P o (dP - delta)
        if (!(ok = wtw(&sm.dp_full[s], (gb >> 1) & 1, st, 28))) break;
        tc_fence_after();
        float dp[32];
        tmem_ld16(col + 64, *reinterpret_cast<float(*)[16]>(&dp[0]));
        tmem_ld16(col + 80, *reinterpret_cast<float(*)[16]>(&dp[16]));
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(&sm.sdp_empty[s]);
        uint32_t dk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          dk[i / 2] = pack_bf16x2(pv[i] * (dp[i] - dl), pv[i + 1] * (dp[i + 1] - dl));
        // the previous batch's dS has been read: with the fused dQ its dQ MMAs
        // were the last readers and their commit (dq_full) says so, which
        // saves the issuing thread a second commit per batch
        if (!(ok = wtw(kDQ ? &sm.dq_full : &sm.ds_empty, (gb & 1) ^ 1, st, 29))) break;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t off = (uint32_t)(((wg * 4 + c) ^ (lrow & 7)) * 16);
          st_shared_v4(drow + off, dk[c * 4], dk[c * 4 + 1], dk[c * 4 + 2], dk[c * 4 + 3]);
        }
        fence_proxy_async_smem();
        warp_arrive(&sm.ds_full);
      }
      if (!ok) break;
      // epilogue: thread = dim; this warpgroup's 32 keys of dV^T and dK^T
      if (!(ok = wtw(&sm.acc_full[ab], use & 1, st, 23))) break;
      tc_fence_after();
      const bool has = nb > 0;
      __nv_bfloat16* dkp = reinterpret_cast<__nv_bfloat16*>(p.dk) + d.b * p.dk_sb + (int64_t)d.hk * p.dk_sh + lrow;
      __nv_bfloat16* dvp = reinterpret_cast<__nv_bfloat16*>(p.dv) + d.b * p.dv_sb + (int64_t)d.hk * p.dv_sh + lrow;
#pragma unroll
      for (int q2 = 0; q2 < 2; ++q2) {
        float vv[16], kv[16];
        if (has) {
          tmem_ld16(tl + kColAcc + ab * 128 + wg * 32 + q2 * 16, vv);
          tmem_ld16(tl + kColAcc + ab * 128 + 64 + wg * 32 + q2 * 16, kv);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) { vv[i] = 0.f; kv[i] = 0.f; }
        }
        if (lrow < D && d.part >= 0) {
          // one row range's partial, fp32 [dK|dV][key][dim]: a warp writes 32
          // consecutive dims of one key per store
          float* pk = args.part + d.part * (2 * 64 * D) + lrow;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int key = wg * 32 + q2 * 16 + i;
            pk[key * D] = kv[i];
            pk[(64 + key) * D] = vv[i];
          }
        } else if (lrow < D) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int key = key_base + q2 * 16 + i;
            if (key < kv_len) {
              const int64_t t = (int64_t)d.kv0 + key;
              if (shared_kv) {
                dkp[t * p.dk_st] = f2bf(kv[i] * p.scale + vv[i]);
              } else {
                dkp[t * p.dk_st] = f2bf(kv[i] * p.scale);
                dvp[t * p.dv_st] = f2bf(vv[i]);
              }
            }
          }
        }
      }
      tc_fence_before();
      warp_arrive(&sm.acc_empty[ab]);
      warp_arrive(&sm.jd_empty[js]);
      ++job;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int D, bool kDQ>
cudaError_t launch(const SfaParams& p, const BwdLayout& L, char* ws, const float* delta, float* dq_acc,
                   cudaStream_t stream) {
  CUtensorMap tq, tdo, tk, tv;
  const int G = p.h_q / p.h_kv;
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len, krows = vl ? p.total_kv : p.kv_len;
  const int64_t nb = vl ? 1 : p.batch;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)D, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)G, 1u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tdo, p.dout, {(uint64_t)D, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                          {p.do_sh, p.do_st, p.do_sb}, {64u, (uint32_t)G, 1u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tk, p.k, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                          {p.k_sh, p.k_st, p.k_sb}, {64u, 1u, 64u, 1u});
  if (e == cudaSuccess)
    e = make_tmap_bf16_4d(&tv, p.v, {(uint64_t)D, (uint64_t)p.h_kv, (uint64_t)krows, (uint64_t)nb},
                          {p.v_sh, p.v_st, p.v_sb}, {64u, 1u, 64u, 1u});
  if (e != cudaSuccess) return e;
  Args a;
  a.p = p;
  a.delta = delta;
  a.dq_acc = dq_acc;
  a.offsets = reinterpret_cast<const int32_t*>(ws + L.inv_offsets);
  a.entries = reinterpret_cast<const int32_t*>(ws + L.inv_entries);
  a.sched = reinterpret_cast<int*>(ws + L.sched);
  a.units = L.units;
  a.nblk = L.nblk;
  a.starts = reinterpret_cast<const int32_t*>(ws + L.inv_cursor);
  a.nsub = L.inv_nsub;
  a.nranges = L.nranges;
  a.sub_per_range = L.sub_per_range;
  a.part = L.nranges > 1 ? reinterpret_cast<float*>(ws + L.dkv_part) : nullptr;
  a.nitems = L.nranges * L.units * L.nblk;
  a.status = device_status_ptr();
  if (a.nitems == 0) return cudaSuccess;
  e = cudaMemsetAsync(a.sched, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  static_assert(sizeof(Smem<D>) + 1024 <= 227 * 1024, "shared memory budget");
  const size_t smem = sizeof(Smem<D>) + 1024;
  e = cudaFuncSetAttribute(sfa_bwd_dkdv_tc_kernel<D, kDQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  sfa_bwd_dkdv_tc_kernel<D, kDQ><<<grid, kDQ ? kThreadsDQ : kThreads, smem, stream>>>(a, tq, tdo, tk, tv);
  note_launch("bwd_dkdv_tc", stream);
  return cudaGetLastError();
}

}  // namespace dkdv
}  // namespace bwd

bool tc_bwd_supported(const SfaParams& p, const char** why) {
  if (!tc_fwd_supported(p, why)) return false;
  if (!tma_compatible(p.dout, p.do_sb, p.do_st, p.do_sh)) { *why = "dout needs 16-byte alignment"; return false; }
  return true;
}

bool tc_dkdv_available() { return true; }

cudaError_t launch_bwd_dq_tc(const SfaParams& p, const float* delta, cudaStream_t st) {
  return p.d_qk == 128 ? bwd::dq::launch<128>(p, delta, st) : bwd::dq::launch<64>(p, delta, st);
}

cudaError_t launch_bwd_dkdv_tc(const SfaParams& p, const BwdLayout& L, char* ws, const float* delta, float* dq_acc,
                               cudaStream_t st) {
  if (dq_acc)
    return p.d_qk == 128 ? bwd::dkdv::launch<128, true>(p, L, ws, delta, dq_acc, st)
                         : bwd::dkdv::launch<64, true>(p, L, ws, delta, dq_acc, st);
  return p.d_qk == 128 ? bwd::dkdv::launch<128, false>(p, L, ws, delta, nullptr, st)
                       : bwd::dkdv::launch<64, false>(p, L, ws, delta, nullptr, st);
}

}  // namespace sfa
