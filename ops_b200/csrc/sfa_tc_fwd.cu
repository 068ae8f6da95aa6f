// sfa_tc_fwd.cu — tensor-core SFA forward for sm_100a (tcgen05 + TMA + TMEM).
//
// Work item = (query row, kv head): the G <= 16 query heads of one kv group
// against that row's selected 64-key blocks.  G is too small for an MMA M
// dimension, so the kernel computes the transposed problem ("swap AB"):
//     S^T[keys, heads]  = K_sel[keys, D] . Q^T[D, heads]        (M = 128 keys, N = 16)
//     O^T[D, heads]    += V_sel^T[D, keys] . P^T[keys, heads]   (M = 128 dims, N = 16)
// with both accumulators in TMEM.  A segment of up to 1024 selected keys is
// scored completely before its softmax, so the max and the sum need one
// cross-thread reduction per segment; segments of one row merge in registers
// with the usual log-sum-exp rescale.
//
// Cost model (measured on B200): an M=128, K=16 tcgen05 MMA with N = 16 takes
// 40-60 cycles — its A operand (4 KB) is read from shared memory — and the
// MMA queue behind one issuing thread is shallow: anything that thread does
// between MMAs (a shared-memory load ~140 cycles, a commit ~90, an mbarrier
// test ~40) leaves the tensor pipe idle.  So two threads issue: one the S^T
// tiles, one the PV tiles; each one's waits are covered by the other's MMAs
// (one issuer: 11.7K cycles per 1024-key job with the kernel's commits and
// waits; two: 6.6K).  K and V stream through separate rings fed by separate
// producer warps, and the softmax runs on two warpgroups with S held in
// registers (one TMEM read per score).
//
// Every gathered K/V byte crosses shared memory twice (TMA write, MMA operand
// read): ~1.1 MB per 1024-key job with Q and P.  Measured at c2 that is 45% of
// the tensor-core shared-memory read rate and ~22% of the bank write rate, so
// the kernel is bound by latency along the softmax chain, not by bandwidth; a
// shared-memory round trip there costs ~0.5-1K cycles under the gathers'
// traffic, so the softmax keeps job fields, maxima and sums in registers and
// uses one barrier per job.
//
// Warp roles (384 threads, one persistent CTA per SM):
//   warp 0      K producer: compacts the row's valid block ids into a job
//               descriptor, loads Q, gathers 64-key K blocks (4-D TMA box per
//               block and 64-dim slab, 128B swizzle) into 128-key stages;
//   warp 10     V producer: the same gathers for V;
//   warp 1      S issuer (one thread): S^T tiles of each job;
//   warp 11     PV issuer (one thread): O^T += V^T P^T tiles of each job;
//   warps 2-9   two softmax warpgroups (thread = key lane of a 128-key tile,
//               warpgroup w takes tiles 4w..4w+3) and the epilogue
//               (thread = dim lane of O^T, warpgroup w takes heads 8w..8w+7):
//               writes o (bf16) and lse (fp32, natural log).
// Every wait is bounded (~2 s); on expiry the kernel records a status word and
// returns.
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

constexpr int kThreads = 384;
constexpr int kSoftmaxThreads = 256;
constexpr int kSegBlocks = 16;      // 64-key blocks per segment (1024 keys, 8 tiles)
constexpr int kJD = 4;              // job descriptor ring depth
constexpr int kNH = 16;             // MMA N: query heads padded to 16
constexpr int kMaxTopk = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;       // 2 buffers x 8 tiles x 16 columns
constexpr uint32_t kColO = 256;     // 2 buffers x 16 columns

enum : int { kFirst = 1, kLast = 2, kSentinel = 4 };

struct JobDesc {
  int row, hk, b, tq, kv0, kv_len, pos, nblk, flags;
  int blocks[kSegBlocks];   // block ids (the softmax's key positions)
  int prow[kSegBlocks];     // kv row of each block's first key (kv0 + 64 e, or its page's rows)
};

template <int D>
struct Smem {
  // K ring stages (128 keys each) and V ring stages.  D = 128: one K stage
  // less and one V stage more measured 4.61 vs 4.91 ms (c2) in the same space:
  // PV starts when the softmax hands over P, so its V must already be in flight.
  static constexpr int kKS = D == 128 ? 2 : 6;
  static constexpr int kVS = D == 128 ? 3 : 4;
  static constexpr int kStageBytes = 128 * D * 2;
  static constexpr int kQBytes = kNH * D * 2;
  static constexpr int kPBytes = kSegBlocks * 64 * kNH * 2;
  alignas(1024) uint8_t kst[kKS][kStageBytes];
  alignas(1024) uint8_t vst[kVS][kStageBytes];
  alignas(1024) uint8_t q[2][kQBytes];
  alignas(1024) uint8_t p[kPBytes];
  JobDesc jd[kJD];
  alignas(16) int bmax[4][16];        // row max of job j in buffer j % 4 (order-preserving ints)
  alignas(16) float bsum[2][16][8];   // row-sum partials of job j-1 in buffer j & 1: [head][warp]
  int plist[kMaxTopk];
  uint64_t k_full[kKS], k_empty[kKS], v_full[kVS], v_empty[kVS];
  uint64_t q_full[2], q_empty[2];
  uint64_t s_full[2], s_empty[2], o_full[2], o_empty[2];
  uint64_t p_full[2], p_empty[2];     // P tiles 0-3 (warpgroup 0) and 4-7 (warpgroup 1)
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint64_t sm_bar;                    // barrier among the softmax threads
  uint32_t tmem_base;
};

struct Args {
  SfaParams p;
  int nitems;
  int nrows;
  int oob_row;       // a kv row coordinate past the tensor map: zero-filled loads
  int32_t* status;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (1 << 16) | site);
  return false;
}

// The same wait for a whole warp: every lane gets one verdict, so a warp that
// gives up leaves its later warp-wide instructions together.
__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

// Sum (kMax = false) or max of v[h] over the 32 lanes of a warp, 16 heads at
// once with 16 shuffles: halve the head set at each butterfly step.  The result
// for head (lane >> 1) & 15 is returned (lanes 2h and 2h+1 hold head h).
template <bool kMax>
__device__ __forceinline__ float warp_reduce16(const float (&v)[16], int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  float a[8], b[4], c[2];
  const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4, h1 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = h4 ? v[i] : v[i + 8], keep = h4 ? v[i + 8] : v[i];
    a[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h3 ? a[i] : a[i + 4], keep = h3 ? a[i + 4] : a[i];
    b[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h2 ? b[i] : b[i + 2], keep = h2 ? b[i + 2] : b[i];
    c[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  float d = op(h1 ? c[1] : c[0], __shfl_xor_sync(0xffffffffu, h1 ? c[0] : c[1], 2));
  return op(d, __shfl_xor_sync(0xffffffffu, d, 1));
}

// Barrier among the softmax threads on an mbarrier, with the same bounded wait
// as every other hand-off (a bar.sync could not give up if a peer stopped).
// `use` counts this thread's barrier uses; all softmax threads make the same
// sequence of uses.
__device__ __forceinline__ bool softmax_barrier(uint64_t* bar, uint32_t& use, int32_t* status) {
  warp_arrive(bar);
  return wtw(bar, (use++) & 1, status, 30);
}

// Floats as ints with the same order, so that a shared-memory integer max
// reduces them (no NaNs here).
__device__ __forceinline__ int f2ord(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

__device__ __forceinline__ void red_max_shared(const int* addr, int v) {
  asm volatile("red.shared.max.s32 [%0], %1;" ::"r"(smem_u32(addr)), "r"(v) : "memory");
}

// Four ordered ints of a max row back to floats (16-byte aligned).
__device__ __forceinline__ void load_max4(const int* src, float* v) {
  const int4 x = *reinterpret_cast<const int4*>(src);
  v[0] = ord2f(x.x);
  v[1] = ord2f(x.y);
  v[2] = ord2f(x.z);
  v[3] = ord2f(x.w);
}

// Eight consecutive floats (16-byte aligned).
__device__ __forceinline__ void load8(const float* src, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(src)[0], b = reinterpret_cast<const float4*>(src)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// One reduction round over the 256 softmax threads, with a single barrier:
// the row max of job j (v: all 16 heads in; the maxima over all threads out)
// by shared-memory integer max into bmax[j % 4], and this warp's row-sum
// partial of job j-1 (lw, for head (lane >> 1) & 15) into bsum[j & 1][head][warp].
// Buffer lifetimes (every thread reads a buffer before it arrives at the
// barrier of the round that recycles it):
//   bmax[j % 4]  written in round j, read after its barrier and again at the
//                end of softmax(j+1) (for the epilogue of j); the first warp
//                resets it after the barrier of round j+2, and round j+4
//                writes it after the barrier of round j+3;
//   bsum[j & 1]  written in round j, read at the end of softmax(j) (for the
//                epilogue of j-1); round j+2 rewrites it.
// kMax = false: the sum partials only (the last job's).
template <bool kMax>
__device__ __forceinline__ bool reduce_round(float (&v)[16], float lw, int j, int (*bmax)[16], float (*bsum)[16][8],
                                             int w8, int lane, int tid, uint64_t* bar, uint32_t& use,
                                             int32_t* status) {
  if constexpr (kMax) {
    const float r = warp_reduce16<true>(v, lane);
    if ((lane & 1) == 0) red_max_shared(&bmax[j % 4][(lane >> 1) & 15], f2ord(r));
  }
  if ((lane & 1) == 0) bsum[j & 1][(lane >> 1) & 15][w8] = lw;
  if (!softmax_barrier(bar, use, status)) return false;
  if constexpr (kMax) {
    if (tid < 16) bmax[(j + 2) % 4][tid] = f2ord(-INFINITY);
#pragma unroll
    for (int h4 = 0; h4 < 4; ++h4) load_max4(&bmax[j % 4][4 * h4], &v[4 * h4]);
  }
  return true;
}

// PAGED: the kv cache is a page pool reached through the block table (the
// unpaged instantiation keeps block ids, not rows, in its registers)
template <int D, bool PAGED>
__global__ void __launch_bounds__(kThreads, 1)
sfa_fwd_tc_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                  const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KS = Smem<D>::kKS, VS = Smem<D>::kVS;
  const SfaParams& p = args.p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.h_q / p.h_kv;
  int32_t* st = args.status;
  const uint32_t chunk_bytes = 128u * D * 2u;

  // ---------------------------------------------------------------- setup
  if (threadIdx.x == 0) {
    for (int i = 0; i < KS; ++i) { mbar_init(&sm.k_full[i], 1); mbar_init(&sm.k_empty[i], 1); }
    for (int i = 0; i < VS; ++i) { mbar_init(&sm.v_full[i], 1); mbar_init(&sm.v_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_empty[i], kSoftmaxThreads / 32);
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], kSoftmaxThreads / 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.p_full[i], kSoftmaxThreads / 64);
      mbar_init(&sm.p_empty[i], 1);
    }
    mbar_init(&sm.sm_bar, kSoftmaxThreads / 32);
    // consumers of a job descriptor: S issuer, PV issuer, V producer, softmax warps
    for (int i = 0; i < kJD; ++i) { mbar_init(&sm.jd_full[i], 1); mbar_init(&sm.jd_empty[i], 3 + kSoftmaxThreads / 32); }
    fence_barrier_init();
  }
  if (threadIdx.x < 64) sm.bmax[threadIdx.x / 16][threadIdx.x % 16] = f2ord(-INFINITY);
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

  // the same copy with its coordinates read from a job descriptor
  auto load_tile = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* full, const JobDesc& d, int c) {
    mbar_arrive_expect_tx(full, chunk_bytes);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int bi = 2 * c + half;
      const int row = bi >= d.nblk ? args.oob_row : PAGED ? d.prow[bi] : d.kv0 + d.blocks[bi] * 64;
#pragma unroll
      for (int cd = 0; cd < D / 64; ++cd)
        tma_load_4d(dst + cd * 128 * 128 + half * 64 * 128, map, full, cd * 64, d.hk, row, d.b);
    }
  };

  // One 128-key stage = two 64-key blocks (TMA rows row0 / row1; a row past the
  // tensor map reads zeros) x D/64 slabs.  All coordinates are in registers: a
  // shared-memory load between two TMA issues would stall the producer.
  auto load_chunk = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* full, int row0, int row1, int hk, int b) {
    mbar_arrive_expect_tx(full, chunk_bytes);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int cd = 0; cd < D / 64; ++cd)
        tma_load_4d(dst + cd * 128 * 128 + half * 64 * 128, map, full, cd * 64, hk, half ? row1 : row0, b);
    }
  };
  // TMA row of block slot i of a segment (block ids in registers; a missing
  // block reads rows past the tensor map, i.e. zeros)
  // (rb holds block ids, or with a paged cache the blocks' rows)
  auto blk_row = [&](const int (&rb)[kSegBlocks], int i, int nb, int kv0) {
    return i >= nb ? args.oob_row : PAGED ? rb[i] : kv0 + rb[i] * 64;
  };

  if (warp == 0) {
    // ============================================================ K producer
    int job = 0, item_i = 0, use = 0;
    bool ok = true;
    // the index slots of the next item are loaded one item ahead (lane s holds
    // slots s and s + 32), so their latency overlaps this item's loads
    auto fetch = [&](int item, int& e0, int& e1, Row& r) {
      const int hk = item / args.nrows, row = item - hk * args.nrows;
      r = row_info(p, row);
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      e0 = lane < p.topk ? __ldg(idx + lane) : -1;
      e1 = lane + 32 < p.topk ? __ldg(idx + lane + 32) : -1;
    };
    int nx0 = -1, nx1 = -1;
    Row nr{};
    if (blockIdx.x < args.nitems) fetch(blockIdx.x, nx0, nx1, nr);
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x, ++item_i) {
      const int hk = item / args.nrows, row = item - hk * args.nrows;
      const Row r = nr;
      const int cur0 = nx0, cur1 = nx1;
      if (item + (int)gridDim.x < args.nitems) fetch(item + gridDim.x, nx0, nx1, nr);
      // compact the valid block ids: position i of the list lives in lane i & 31
      // of pl0 (i < 32) or pl1 (i >= 32)
      int n = 0, pl0 = -1, pl1 = -1;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int e = half ? cur1 : cur0;
        const bool valid = block_valid_keys(e, 64, r.kv_len, r.pos, p.causal) > 0;
        const unsigned m = __ballot_sync(0xffffffffu, valid);
        if (valid) sm.plist[n + __popc(m & ((1u << lane) - 1u))] = e;
        n += __popc(m);
      }
      __syncwarp();
      if (lane < n) pl0 = sm.plist[lane];
      if (lane + 32 < n) pl1 = sm.plist[lane + 32];
      const int nseg = n == 0 ? 1 : (n + kSegBlocks - 1) / kSegBlocks;
      if (lane == 0) {
        const int qs = item_i & 1;
        ok = wt(&sm.q_empty[qs], ((item_i >> 1) & 1) ^ 1, st, 2);
        if (ok) {
          mbar_arrive_expect_tx(&sm.q_full[qs], (uint32_t)(G * D * 2));
#pragma unroll
          for (int cd = 0; cd < D / 64; ++cd)
            tma_load_4d(&sm.q[qs][cd * kNH * 128], &tmq, &sm.q_full[qs], cd * 64, hk * G, (int)r.tq, r.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      for (int seg = 0; seg < nseg && ok; ++seg, ++job) {
        const int js = job % kJD;
        if (lane == 0) ok = wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 3);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        JobDesc& d = sm.jd[js];
        const int nb = n == 0 ? 0 : min(kSegBlocks, n - seg * kSegBlocks);
        // lane i < nb: block i of this segment (list position seg * 16 + i)
        const int gi = seg * kSegBlocks + (lane & (kSegBlocks - 1));
        const int v0 = __shfl_sync(0xffffffffu, pl0, gi & 31);
        const int v1 = __shfl_sync(0xffffffffu, pl1, gi & 31);
        const int blk = gi < 32 ? v0 : v1;
        // a paged cache: the block's first row in the page pool
        constexpr bool paged = PAGED;
        const int prow = paged && lane < nb ? (int)kv_row(p, r, blk * 64) : 0;
        if (lane < nb) {
          d.blocks[lane] = blk;
          if (paged) d.prow[lane] = prow;
        }
        if (lane == 0) {
          d.row = row;
          d.hk = hk;
          d.b = r.b;
          d.tq = (int)r.tq;
          d.kv0 = (int)r.kv0;
          d.kv_len = r.kv_len;
          d.pos = r.pos;
          d.nblk = nb;
          d.flags = (seg == 0 ? kFirst : 0) | (seg == nseg - 1 ? kLast : 0);
        }
        // the segment's block ids (rows, when paged) into lane 0's registers
        int rb[kSegBlocks];
#pragma unroll
        for (int i = 0; i < kSegBlocks; ++i) rb[i] = __shfl_sync(0xffffffffu, paged ? prow : blk, i);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sm.jd_full[js]);
          const int nch = (nb + 1) / 2;
#pragma unroll
          for (int c = 0; c < kSegBlocks / 2; ++c) {
            if (c < nch && ok) {
              const int s = use % KS;
              ok = wt(&sm.k_empty[s], ((use / KS) & 1) ^ 1, st, 1);
              if (ok)
                load_chunk(&tmk, sm.kst[s], &sm.k_full[s], blk_row(rb, 2 * c, nb, (int)r.kv0),
                           blk_row(rb, 2 * c + 1, nb, (int)r.kv0), hk, r.b);
              ++use;
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        use = __shfl_sync(0xffffffffu, use, 0);
      }
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&sm.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 4)) {
        sm.jd[js].flags = kSentinel;
        mbar_arrive(&sm.jd_full[js]);
      }
    }
  } else if (warp == 10) {
    // ============================================================ V producer
    // Reads each copy's coordinates from the descriptor.  A V producer with
    // register-resident coordinates issues faster, but together with the K
    // producer below it measured slower overall (c2: 6.42 vs 5.47 ms): the
    // extra V gathers in flight delay the K gathers that S^T waits on.
    if (lane == 0) {
      int job = 0, use = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 5))) break;
        const JobDesc& d = sm.jd[js];
        if (d.flags & kSentinel) break;
        for (int c = 0; c < (d.nblk + 1) / 2 && ok; ++c, ++use) {
          const int s = use % VS;
          if (!(ok = wt(&sm.v_empty[s], ((use / VS) & 1) ^ 1, st, 6))) break;
          load_tile(&tmv, sm.vst[s], &sm.v_full[s], d, c);
        }
        mbar_arrive(&sm.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp == 1) {
    // ============================================================ S issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, kNH, false, false);
      int job = 0, item_i = 0, kuse = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 13))) break;
        // job fields go to registers once: a shared-memory load between MMAs
        // stalls this thread and leaves the tensor pipe without work
        const int flags = sm.jd[js].flags, nblk = sm.jd[js].nblk;
        if (flags & kSentinel) break;
        const int qs = item_i & 1;
        if (flags & kFirst)
          if (!(ok = wt(&sm.q_full[qs], (item_i >> 1) & 1, st, 14))) break;
        const int sb = job & 1;
        if (!(ok = wt(&sm.s_empty[sb], ((job >> 1) & 1) ^ 1, st, 15))) break;
        tc_fence_after();
        const uint64_t qdesc = smem_desc(smem_u32(&sm.q[qs][0]), 16, 1024, kSw128);
        const int nch = (nblk + 1) / 2;
        for (int c = 0; c < nch && ok; ++c, ++kuse) {
          const int s = kuse % KS;
          // TMA-filled stage: the mbarrier's complete_tx orders it for the
          // tensor core (no tcgen05 fence needed)
          if (!(ok = wt(&sm.k_full[s], (kuse / KS) & 1, st, 16))) break;
          const uint64_t kdesc = smem_desc(smem_u32(&sm.kst[s][0]), 16, 1024, kSw128);
          const uint32_t dcol = tmem + kColS + sb * 128 + c * kNH;
#pragma unroll
          for (int k = 0; k < D / 16; ++k)
            mma_bf16_ss(dcol, kdesc + (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4),
                        qdesc + (uint64_t)(((k >> 2) * (kNH * 128) + (k & 3) * 32) >> 4), id_s, k != 0);
          mma_commit(&sm.k_empty[s]);
        }
        if (!ok) break;
        mma_commit(&sm.s_full[sb]);
        if (flags & kLast) {
          mma_commit(&sm.q_empty[qs]);
          ++item_i;
        }
        mbar_arrive(&sm.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp == 11) {
    // ============================================================ PV issuer
    // A second issuing thread: while one waits (on P, a stage, a barrier) the
    // other's MMAs keep the tensor pipe busy.
    if (lane == 0) {
      const uint32_t id_o = idesc_bf16(128, kNH, true, true);
      // A = V tile as MN-major: 64-dim slabs LBO apart (D = 64 repeats the slab;
      // rows 64-127 of O^T are then ignored), 8-key groups 1024 B apart.
      const uint32_t lbo_v = D == 128 ? 128u * 128u : 0u;
      const uint64_t pdesc = smem_desc(smem_u32(&sm.p[0]), 0, 256, kSw32);
      int job = 0, vuse = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&sm.jd_full[js], (job / kJD) & 1, st, 17))) break;
        const int flags = sm.jd[js].flags, nblk = sm.jd[js].nblk;
        if (flags & kSentinel) break;
        const int sb = job & 1;
        if (!(ok = wt(&sm.o_empty[sb], ((job >> 1) & 1) ^ 1, st, 11))) break;
        const uint32_t dcol = tmem + kColO + sb * kNH;
        const int nch = (nblk + 1) / 2;
        for (int c = 0; c < 8 && ok; ++c) {
          // tiles 0-3 come from softmax warpgroup 0, tiles 4-7 from group 1
          if (c == 0 || c == 4) {
            if (!(ok = wt(&sm.p_full[c >> 2], job & 1, st, 10))) break;
            tc_fence_after();
          }
          if (c < nch) {
            const int s = vuse % VS;
            if (!(ok = wt(&sm.v_full[s], (vuse / VS) & 1, st, 12))) break;
            // descriptors advance by adding the byte offset / 16 to the start-address field
            const uint64_t a0 = smem_desc(smem_u32(&sm.vst[s][0]), lbo_v, 1024, kSw128);
            const uint64_t b0 = pdesc + (uint64_t)(c * 128 * (kNH * 2) >> 4);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_bf16_ss(dcol, a0 + (uint64_t)(kk * 2048 >> 4), b0 + (uint64_t)(kk * 16 * (kNH * 2) >> 4), id_o,
                          (c | kk) != 0);
            mma_commit(&sm.v_empty[s]);
            ++vuse;
          }
          if (c == 3 || c == 7) mma_commit(&sm.p_empty[c >> 2]);
        }
        if (!ok) break;
        mma_commit(&sm.o_full[sb]);
        mbar_arrive(&sm.jd_empty[js]);
        ++job;
      }
    }
  } else {
    // ============================================================ softmax / epilogue
    const int w8 = warp - 2;             // 0..7
    const int wg = w8 >> 2;              // warpgroup 0 / 1
    const int wq = warp & 3;             // TMEM lane quadrant of this warp
    const int tid = threadIdx.x - 64;    // 0..255
    const int lrow = wq * 32 + lane;     // TMEM lane: key (softmax) or dim (epilogue)
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    uint32_t bar_use = 0;
    float acc[8], mrun[8];               // epilogue state for heads 8*wg .. 8*wg+7
#pragma unroll
    for (int h = 0; h < 8; ++h) { acc[h] = 0.f; mrun[h] = -INFINITY; }
    // What this thread needs of a job, copied out of its descriptor one job
    // ahead: under the gathers' shared-memory traffic one load round trip costs
    // ~2K cycles, so none may sit on the softmax -> epilogue chain.
    // w: flags (bits 0-2), vmask (4-7: bit i set when this thread's key of
    // tile 4*wg + i is selected), nblk (8-15), kv head (16-31)
    struct JobRegs {
      uint32_t w;
      int b, tq;
      __device__ int flags() const { return (int)(w & 7u); }
      __device__ uint32_t vmask() const { return (w >> 4) & 15u; }
      __device__ int nblk() const { return (int)((w >> 8) & 255u); }
      __device__ int hk() const { return (int)(w >> 16); }
    };
    auto load_job = [&](int j, JobRegs& r) {
      const JobDesc& d = sm.jd[j % kJD];
      const int nblk = d.nblk, kv_len = d.kv_len, pos = d.pos;
      uint32_t vm = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int bi = 2 * (wg * 4 + i) + (lrow >> 6);
        // slots past nblk hold stale ids: unsigned arithmetic, and bi < nblk decides
        const int key = (int)((uint32_t)d.blocks[bi] * 64u) + (lrow & 63);
        if (bi < nblk && key < kv_len && (!p.causal || key <= pos)) vm |= 1u << i;
      }
      r.w = (uint32_t)d.flags | (vm << 4) | ((uint32_t)nblk << 8) | ((uint32_t)d.hk << 16);
      r.b = d.b;
      r.tq = d.tq;
    };
    bool ok = true;
    float lw_prev = 0.f;                 // this warp's row-sum partial of the previous job
    const int hl = wg * 8 + (lane & 7);  // lane l finishes head 8*wg + (l & 7) in the epilogue
    float lrun_l = 0.f;                  // running row sum of head hl
    // softmax of job j: P tiles to shared memory; returns this warp's row-sum
    // partial of job j (lw_out) and, loaded last so that their latency hides
    // behind what follows, this warpgroup's 8 row maxima of job j-1 (raw
    // scores) and the 8 warp partials of its row sum for head hl (lprev)
    auto softmax = [&](int j, const JobRegs& r, float& lw_out, float (&mprev)[8], float (&lprev)[8]) -> bool {
      const int sb = j & 1;
      if (!wtw(&sm.s_full[sb], (j >> 1) & 1, st, 20)) return false;
      tc_fence_after();
      const int nch = (r.nblk() + 1) / 2;
      const uint32_t ts = tl + kColS + sb * 128;
      float s[4][16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = wg * 4 + i;
        if (c < nch) tmem_ld16(ts + c * kNH, s[i]);
      }
      tmem_ld_wait();
      tc_fence_before();
      warp_arrive(&sm.s_empty[sb]);
      // the max of the raw scores (c2 > 0); the scale folds into the exponent's FMA
      float m[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) m[h] = -INFINITY;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if ((r.vmask() >> i) & 1u) {
#pragma unroll
          for (int h = 0; h < 16; ++h) m[h] = fmaxf(m[h], s[i][h]);
        }
      }
      if (!reduce_round<true>(m, lw_prev, j, sm.bmax, sm.bsum, w8, lane, tid, &sm.sm_bar, bar_use, st)) return false;
      float l[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        l[h] = 0.f;
        m[h] *= -c2;                     // finite for every head once a key is selected
      }
      // this warpgroup's half of the P buffer is free once PV(j-1) read it
      if (!wtw(&sm.p_empty[wg], (j & 1) ^ 1, st, 21)) return false;
      const uint32_t pbase = smem_u32(&sm.p[0]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = wg * 4 + i;
        if (c < nch) {
          const bool valid = (r.vmask() >> i) & 1u;
          float pr[16];
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            pr[h] = valid ? ex2(fmaf(s[i][h], c2, m[h])) : 0.f;
            l[h] += pr[h];
          }
          if (p.compat & SFA_COMPAT_REFERENCE_P) {
#pragma unroll
            for (int h = 0; h < 16; ++h) pr[h] = ref_p(pr[h]);
          }
          // row = key within the segment; 32-byte rows, 32B swizzle (16-byte
          // halves swap when bit 2 of the row is set)
          const int rowk = c * 128 + lrow;
          const uint32_t off = pbase + rowk * 32;
          const uint32_t sw = ((rowk >> 2) & 1) << 4;
          st_shared_v4(off + sw, pack_bf16x2(pr[0], pr[1]), pack_bf16x2(pr[2], pr[3]), pack_bf16x2(pr[4], pr[5]),
                       pack_bf16x2(pr[6], pr[7]));
          st_shared_v4(off + (16 - sw), pack_bf16x2(pr[8], pr[9]), pack_bf16x2(pr[10], pr[11]),
                       pack_bf16x2(pr[12], pr[13]), pack_bf16x2(pr[14], pr[15]));
        }
      }
      fence_proxy_async_smem();
      warp_arrive(&sm.p_full[wg]);
      load_max4(&sm.bmax[(j + 3) % 4][wg * 8], &mprev[0]);      // job j-1
      load_max4(&sm.bmax[(j + 3) % 4][wg * 8 + 4], &mprev[4]);
      load8(&sm.bsum[j & 1][hl][0], lprev);
      lw_out = warp_reduce16<false>(l, lane);
      return true;
    };
    // mj: the raw-score maxima of job jj (scaled here); lsj: the 8 warp
    // partials of its row sum for head hl, added in a fixed order
    auto epilogue = [&](int jj, const JobRegs& r, const float (&mj)[8], const float (&lsj)[8]) -> bool {
      const int sb = jj & 1;
      const int flags = r.flags(), hk = r.hk();
      float s2 = -INFINITY;              // sink logit, log2 units (L1-resident)
      if ((flags & kLast) && p.attn_sink && hl < G) s2 = __ldg(p.attn_sink + hk * G + hl) * kLog2e;
      if (!wtw(&sm.o_full[sb], (jj >> 1) & 1, st, 22)) return false;
      tc_fence_after();
      if (r.nblk() > 0) {
        float o[16];
        tmem_ld16(tl + kColO + sb * kNH, o);   // all 16 heads; this warpgroup keeps 8
        tmem_ld_wait();
        float ls = lsj[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) ls += lsj[w];
        if (flags & kFirst) {
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            acc[h] = wg ? o[8 + h] : o[h];
            mrun[h] = mj[h] * c2;
          }
          lrun_l = ls;
        } else {
          float al = 0.f, bl = 0.f;
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const float ov = wg ? o[8 + h] : o[h];
            const float ms = mj[h] * c2;
            const float M = fmaxf(mrun[h], ms);
            const float a = ex2(mrun[h] - M), bb = ex2(ms - M);
            acc[h] = acc[h] * a + ov * bb;
            mrun[h] = M;
            if ((lane & 7) == h) { al = a; bl = bb; }
          }
          lrun_l = lrun_l * al + ls * bl;
        }
      } else if (flags & kFirst) {
#pragma unroll
        for (int h = 0; h < 8; ++h) { acc[h] = 0.f; mrun[h] = -INFINITY; }
        lrun_l = 0.f;
      }
      tc_fence_before();
      warp_arrive(&sm.o_empty[sb]);
      if (flags & kLast) {
        // the head's running max / sum are the same in every thread: each lane
        // finishes one head and the scale goes out by shuffle
        float mh = mrun[0];
        const float lh = lrun_l;
#pragma unroll
        for (int h = 1; h < 8; ++h)
          if ((lane & 7) == h) mh = mrun[h];
        const float M = fmaxf(mh, s2);
        float inv = 0.f, lv = -INFINITY;
        if (M != -INFINITY) {
          const float w = ex2(mh - M);
          const float lt = lh * w + ex2(s2 - M);
          inv = __fdividef(w, lt);
          lv = (M + lg2(lt)) * kLn2;
        }
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.o) + r.b * p.o_sb + (int64_t)r.tq * p.o_st +
                           (int64_t)(hk * G) * p.o_sh;
        float* lse = p.lse + r.b * p.l_sb + (int64_t)r.tq * p.l_st + (int64_t)(hk * G) * p.l_sh;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const int hh = wg * 8 + h;
          const float sc = __shfl_sync(0xffffffffu, inv, h);
          if (hh < G && lrow < D) o[hh * p.o_sh + lrow] = f2bf(acc[h] * sc);
        }
        if (wq == 0 && lane < 8 && hl < G) lse[hl * p.l_sh] = lv;
      }
      warp_arrive(&sm.jd_empty[jj % kJD]);
      return true;
    };
    // job j's softmax, then the next descriptor's copy, then job j-1's epilogue
    // (its O^T accumulates meanwhile)
    JobRegs cur{}, prev{};
    int job = 0;
    if ((ok = wtw(&sm.jd_full[0], 0, st, 23))) load_job(0, cur);
    while (ok && !(cur.flags() & kSentinel)) {
      float lw, mprev[8], lprev[8];
      if (!(ok = softmax(job, cur, lw, mprev, lprev))) break;
      const int jn = job + 1;
      JobRegs nxt;
      if (!(ok = wtw(&sm.jd_full[jn % kJD], (jn / kJD) & 1, st, 23))) break;
      load_job(jn, nxt);
      if (job > 0 && !(ok = epilogue(job - 1, prev, mprev, lprev))) break;
      prev = cur;
      cur = nxt;
      lw_prev = lw;
      ++job;
    }
    // the last job's row sums still need their reduction round
    if (ok && job > 0) {
      float unused[16], mlast[8], llast[8];
      if (reduce_round<false>(unused, lw_prev, job, sm.bmax, sm.bsum, w8, lane, tid, &sm.sm_bar, bar_use, st)) {
        load_max4(&sm.bmax[(job + 3) % 4][wg * 8], &mlast[0]);
        load_max4(&sm.bmax[(job + 3) % 4][wg * 8 + 4], &mlast[4]);
        load8(&sm.bsum[job & 1][hl][0], llast);
        epilogue(job - 1, prev, mlast, llast);
      }
    }
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
  const bool paged = p.block_table != nullptr;
  e = cudaFuncSetAttribute(paged ? sfa_fwd_tc_kernel<D, true> : sfa_fwd_tc_kernel<D, false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  if (paged)
    sfa_fwd_tc_kernel<D, true><<<grid, kThreads, smem, st>>>(a, tq, tk, tv);
  else
    sfa_fwd_tc_kernel<D, false><<<grid, kThreads, smem, st>>>(a, tq, tk, tv);
  note_launch("fwd_tc", st);
  return cudaGetLastError();
}

}  // namespace fwd

bool tc_fwd_supported(const SfaParams& p, const char** why) {
  const int G = p.h_q / p.h_kv;
  if (device_cc() != 100) { *why = "needs an sm_100 device"; return false; }
  if (p.block_size != 64) { *why = "block_size must be 64"; return false; }
  if (p.kv_dtype != SFA_KV_BF16) { *why = "fp8 kv: the token-level and CUDA-core kernels read it"; return false; }
  if (p.topk > fwd::kMaxTopk) { *why = "topk must be <= 64"; return false; }
  if (p.d_qk != p.d_v || (p.d_qk != 64 && p.d_qk != 128)) { *why = "head dim must be 64 or 128 (D_qk == D_v)"; return false; }
  if (G > fwd::kNH) { *why = "query heads per kv head must be <= 16"; return false; }
  if (p.h_kv > 65535) { *why = "at most 65535 kv heads"; return false; }
  if (!(p.scale > 0.f)) { *why = "needs a positive softmax scale"; return false; }
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
