// sfa_tok_fwd.cu — tensor-core SFA forward for token-level top-k (block_size 1)
// on sm_100a: the reference's native operating mode (one kv row per index,
// SFA.py:399-415) and the MLA shape (128 query heads on one latent kv head,
// D_qk 576 / D_v 512).
//
// Work item = (query row, kv head, head tile of up to 128 heads, V part).
// Normal orientation: the head tile is the MMA's M dimension,
//     S[heads, keys]  = Q[heads, D_qk] . K_sel[keys, D_qk]^T   (M = 128, N = 64)
//     O[heads, dims] += P[heads, keys] . V_sel[keys, dims]     (M = 128, N <= 128 per stage)
// Q stays in shared memory for the whole item; the selected rows stream in
// 64-key chunks gathered with TMA `tile::gather4` (four kv rows per copy,
// 128B-swizzled 64-dim slabs) — K slabs for S, then the V slabs of this
// item's part.  O for one part (at most 256 dims = 256 TMEM columns), two
// S buffers (2 x 64 columns) and P (bf16, 32 columns) fit the 512 TMEM
// columns; D_v beyond 256 (MLA: 512) is split into parts computed by separate
// work items, each recomputing S.  P stays in TMEM as the PV MMA's A operand,
// so shared memory holds only Q and the K / V rings (MLA: three K stages
// where a shared-memory P left room for two).
//
// Softmax: one thread per head row (the row is thread-local in TMEM, so the
// max and the sum need no cross-thread reduction).  P = exp2(S*c - m) uses a
// reference maximum m that is raised only when a chunk's max exceeds it by
// more than 8 (log2 units), so P <= 2^8 and O is rescaled in TMEM only on
// those rare chunks (before that chunk's PV is issued; the previous chunk's
// PV has completed because P's buffer is single).
//
// Row gathers are issue-bound: a warp's gather4 copies leave one after another
// (~100 cycles each, so ~5 B/clk per issuing warp, measured on B200), while
// warps issue in parallel.  A pool of nine gather warps therefore shares the
// K and V rings: every (stage slot, slab half) position has a fixed owner.
//
// Warp roles (512 threads, one persistent CTA per SM):
//   warp 0      descriptor producer: index validity masks of the item's 64-slot
//               chunks, chunk descriptors (mask, key ids), Q loads;
//   warp 1      S issuer (one thread);
//   warp 2      PV issuer (one thread);
//   warps 3, 8-15  gather pool: K and V slabs of each chunk (tile::gather4);
//   warps 4-7   softmax + epilogue, thread = head row (TMEM lane).
// Every wait is bounded (~2 s); on expiry the kernel records (4 << 16) | site in
// the status word and returns.
//
// Replaces `_attn_fwd` / `_inner_fwd` (SFA.py:309-587) for token-level indices:
// the same math (scores SFA.py:425, online softmax SFA.py:432-446, PV SFA.py:456,
// sink and lse SFA.py:469-480), one gather per selected row per item instead of
// one per 32-head tile, no global-memory workspaces.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"
#include "sfa_tok_common.cuh"

#include <cuda_fp8.h>

namespace sfa {
using namespace tc;
using namespace tok;

namespace tokf {

constexpr int kThreads = 512;
constexpr int kGatherWarps = 9;        // warps 3 and 8-15
constexpr int kKeys = 64;            // keys per chunk
constexpr int kMaxTopk = 32 * kKeys;  // one chunk per producer lane
constexpr int kJD = 4;               // descriptor ring
constexpr int kSlab = 64 * 128;      // bytes of one 64-row x 64-dim bf16 slab
constexpr int kQSlab = 128 * 128;    // bytes of one 128-row x 64-dim Q slab
constexpr float kRescaleLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 256;      // two S buffers of 64 columns after O's 256
constexpr uint32_t kColP = 384;      // P of one chunk: 64 keys as bf16 pairs, 32 columns

enum : int { kFirst = 1, kLast = 2, kEmpty = 4, kSentinel = 8 };

struct Desc {
  uint32_t mlo, mhi;                 // valid keys of the chunk (bit j: key j)
  int flags;
  int row, hk, hg, vp, b, tq;
  int64_t kbase, vbase;              // K / V gather rows of key 0 of this item's sequence / kv head
  int64_t sbase;                     // fp8 kv: scale index of key 0
  int keys[kKeys];                   // key ids (an invalid slot repeats a valid key of the chunk)
};

struct Args {
  SfaParams p;
  int nitems, nrows, n_hg, n_vp, HG, G, nq;
  int dvp;                           // dims of a full V part (<= 256)
  int kst, vst;                      // ring stages (2 slabs each)
  uint32_t off_k, off_v, off_desc, off_bar;   // smem offsets (Q at 0)
  int64_t k_rs, v_rs;                // element strides of one gather row (k / v)
  int fp8;                           // kv stored as e4m3 + row scales: slabs converted to bf16 here
  int32_t* status;
};

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, p_empty;
  uint64_t o_full, o_empty;
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint32_t tmem_base;
  uint32_t pad;
  uint64_t k_full[8], k_empty[8], v_full[8], v_empty[8];
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (4 << 16) | site);
  return false;
}

__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}



// Two e4m3 kv rows (64 dims each, at byte offsets o0 / o1 of kv) into rows
// `lane` and `lane + 32` of a bf16 64 x 64 slab, times their row scales, with
// the 128-byte swizzle of the TMA copies (16-byte group g of row j at
// group g ^ (j & 7)).  Exact when the scales are powers of two.
__device__ __forceinline__ void fp8_rows_to_slab(uint8_t* slab, const uint8_t* kv, int64_t o0, int64_t o1, float s0,
                                                 float s1, int lane) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4* src = reinterpret_cast<const uint4*>(kv + (r ? o1 : o0));
    const float sc = r ? s1 : s0;
    const int j = lane + 32 * r;
    uint8_t* row = slab + j * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = __ldg(src + q);                      // 16 e4m3 values: dims 16q .. 16q + 15
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(words[i] & 0xffffu), __NV_E4M3);
        const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(words[i] >> 16), __NV_E4M3);
        const float2 a = __half22float2(__half2(lo)), b = __half22float2(__half2(hi));
        o[2 * i] = pack_bf16x2(a.x * sc, a.y * sc);
        o[2 * i + 1] = pack_bf16x2(b.x * sc, b.y * sc);
      }
      // two 16-byte groups (8 dims each) of the bf16 row
      const int g0 = 2 * q, g1 = 2 * q + 1;
      *reinterpret_cast<uint4*>(row + ((g0 ^ (j & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(row + ((g1 ^ (j & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

// Item index -> (row, kv head, head tile, V part); the parts of one (row, kv
// head, head tile) are consecutive so the CTAs computing them run together
// and share the K gathers in L2.
__device__ __forceinline__ void decode_item(const Args& a, int item, int& row, int& hk, int& hg, int& vp) {
  vp = item % a.n_vp;
  int r = item / a.n_vp;
  hg = r % a.n_hg;
  r /= a.n_hg;
  hk = r % a.p.h_kv;
  row = r / a.p.h_kv;
}

// FP8: kv rows are e4m3 + row scales, widened by the gather warps; PAGED: keys
// reach their rows through the block table.  Each mode is its own
// instantiation: the runtime checks cost the bf16 kernel ~10 % at tok128.
template <bool FP8, bool PAGED>
__global__ void __launch_bounds__(kThreads, 1)
sfa_tok_fwd_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaParams& p = args.p;
  uint8_t* sq = sbase;
  uint8_t* sk = sbase + args.off_k;
  uint8_t* sv = sbase + args.off_v;
  Desc* jd = reinterpret_cast<Desc*>(sbase + args.off_desc);
  Bars& B = *reinterpret_cast<Bars*>(sbase + args.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* st = args.status;
  const int KS = args.kst, VS = args.vst, NQ = args.nq;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.s_full[i], 1);
      mbar_init(&B.s_empty[i], 4);
    }
    mbar_init(&B.p_full, 4);
    mbar_init(&B.p_empty, 1);
    mbar_init(&B.o_full, 1);
    mbar_init(&B.o_empty, 4);
    // consumers of a descriptor: S issuer, PV issuer, the gather warps, 4 softmax warps
    for (int i = 0; i < kJD; ++i) {
      mbar_init(&B.jd_full[i], 1);
      mbar_init(&B.jd_empty[i], 2 + kGatherWarps + 4);
    }
    // a stage's two slab positions have their own owners: each arrives once per use
    for (int i = 0; i < KS; ++i) { mbar_init(&B.k_full[i], 2); mbar_init(&B.k_empty[i], 1); }
    for (int i = 0; i < VS; ++i) { mbar_init(&B.v_full[i], 2); mbar_init(&B.v_empty[i], 1); }
    fence_barrier_init();
  }
  // head rows past the tile's HG stay zero for the whole kernel (TMA writes HG rows)
  if (args.HG < 128)
    for (int i = threadIdx.x; i < NQ * kQSlab / 16; i += kThreads) reinterpret_cast<uint4*>(sq)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(&B.tmem_base, kTmemCols);
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
  const uint32_t tmem = B.tmem_base;
  const int quad = lane & 15;        // gather copy of this lane: keys 4*quad .. 4*quad+3

  if (warp == 0) {
    // ============================================================ descriptor producer
    int job = 0, item_i = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x) {
      int row, hk, hg, vp;
      decode_item(args, item, row, hk, hg, vp);
      const Row r = row_info(p, row);
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      const int nch = (p.topk + kKeys - 1) / kKeys;
      // pass 1: lane c keeps the valid-key mask of chunk c
      uint32_t my_lo = 0, my_hi = 0;
      for (int c = 0; c < nch; ++c) {
        const int s0 = c * kKeys + lane, s1 = s0 + 32;
        const int e0 = s0 < p.topk ? __ldg(idx + s0) : -1;
        const int e1 = s1 < p.topk ? __ldg(idx + s1) : -1;
        const bool v0 = e0 >= 0 && e0 < r.kv_len && (!p.causal || e0 <= r.pos);
        const bool v1 = e1 >= 0 && e1 < r.kv_len && (!p.causal || e1 <= r.pos);
        const uint32_t lo = __ballot_sync(0xffffffffu, v0), hi = __ballot_sync(0xffffffffu, v1);
        if (lane == c) { my_lo = lo; my_hi = hi; }
      }
      const uint32_t chunks = __ballot_sync(0xffffffffu, (my_lo | my_hi) != 0u);
      const int64_t kbase = ((int64_t)r.b * p.k_sb + r.kv0 * p.k_st + (int64_t)hk * p.k_sh) / args.k_rs;
      const int64_t vbase = ((int64_t)r.b * p.v_sb + r.kv0 * p.v_st + (int64_t)hk * p.v_sh) / args.v_rs;
      const int64_t sbase = (int64_t)r.b * p.ks_sb + r.kv0 * p.ks_st + (int64_t)hk * p.ks_sh;
      if (chunks == 0u) {
        // nothing selected: one descriptor tells the softmax warps to write zeros
        if (lane == 0) {
          const int js = job % kJD;
          ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 1);
          if (ok) {
            Desc& d = jd[js];
            d.flags = kFirst | kLast | kEmpty;
            d.row = row; d.hk = hk; d.hg = hg; d.vp = vp; d.b = r.b; d.tq = (int)r.tq;
            mbar_arrive(&B.jd_full[js]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        ++job;
        continue;
      }
      // Q of the head tile: one 4-D box per 64-dim slab
      if (lane == 0) {
        ok = wt(&B.q_empty, (item_i & 1) ^ 1, st, 2);
        if (ok) {
          mbar_arrive_expect_tx(&B.q_full, (uint32_t)(args.HG * 128 * NQ));
          for (int s = 0; s < NQ; ++s)
            tma_load_4d(sq + s * kQSlab, &tmq, &B.q_full, s * 64, hk * args.G + hg * 128, (int)r.tq, r.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      ++item_i;
      const int cfirst = __ffs(chunks) - 1, clast = 31 - __clz(chunks);
      for (uint32_t rem = chunks; rem && ok; rem &= rem - 1u, ++job) {
        const int c = __ffs(rem) - 1;
        const uint32_t lo = __shfl_sync(0xffffffffu, my_lo, c), hi = __shfl_sync(0xffffffffu, my_hi, c);
        const int s0 = c * kKeys + lane, s1 = s0 + 32;
        int e0 = s0 < p.topk ? __ldg(idx + s0) : -1;
        int e1 = s1 < p.topk ? __ldg(idx + s1) : -1;
        // an invalid slot repeats the chunk's first valid key (masked out of the softmax)
        const int fl = lo ? __ffs(lo) - 1 : __ffs(hi) - 1;
        const int f0 = __shfl_sync(0xffffffffu, e0, fl), f1 = __shfl_sync(0xffffffffu, e1, fl);
        const int fk = lo ? f0 : f1;
        if (!((lo >> lane) & 1u)) e0 = fk;
        if (!((hi >> lane) & 1u)) e1 = fk;
        if (PAGED) {                           // paged cache: the keys' rows in the page pool
          e0 = (int)kv_row(p, r, e0);
          e1 = (int)kv_row(p, r, e1);
        }
        const int js = job % kJD;
        if (lane == 0) ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 3);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        Desc& d = jd[js];
        d.keys[lane] = e0;
        d.keys[lane + 32] = e1;
        if (lane == 0) {
          d.mlo = lo; d.mhi = hi;
          d.flags = (c == cfirst ? kFirst : 0) | (c == clast ? kLast : 0);
          d.row = row; d.hk = hk; d.hg = hg; d.vp = vp; d.b = r.b; d.tq = (int)r.tq;
          d.kbase = kbase;
          d.vbase = vbase;
          d.sbase = sbase;
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
  } else if (warp == 3 || warp >= 8) {
    // ============================================================ gather pool
    // Each (ring, stage slot, slab half) position has one owner warp
    // (position % kGatherWarps), which takes part in every use of its slot, in
    // order: it waits for the slot's previous use to be consumed, then either
    // announces and copies its slab or, when the stage has a single slab,
    // arrives without bytes (the full barriers count two arrivals).  Because
    // an owner never skips a use, its parity wait can never be satisfied by a
    // phase two laps old.  (Dealing slabs to warps round-robin instead let a
    // warp run laps ahead of a slot and refill it early.)
    const int g = warp == 3 ? 0 : warp - 7;
    const int64_t kstep = p.k_st / args.k_rs, vstep = p.v_st / args.v_rs;
    int job = 0, kuse = 0, vuse = 0;
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
      const int e0 = d.keys[lane], e1 = d.keys[lane + 32];
      const int64_t kbase = d.kbase, vbase = d.vbase, sbase = d.sbase;
      const int vp = d.vp;
      // fp8 kv: this lane's two keys' row scales (keys lane and lane + 32 of the chunk)
      float sc0 = 0.f, sc1 = 0.f;
      if (FP8) {
        sc0 = __ldg(p.kv_scale + sbase + (int64_t)e0 * p.ks_st);
        sc1 = __ldg(p.kv_scale + sbase + (int64_t)e1 * p.ks_st);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.jd_empty[js]);
      int kq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int src = (4 * quad + i) & 31;
        const int a = __shfl_sync(0xffffffffu, e0, src), bb = __shfl_sync(0xffffffffu, e1, src);
        kq[i] = quad < 8 ? a : bb;
      }
      const int d0 = vp * args.dvp;
      const int nv = (min(p.d_v - d0, args.dvp)) / 64;
      for (int r = 0; r < 2 && ok; ++r) {
        const bool isk = r == 0;
        const int tot = isk ? NQ : nv, nst = isk ? KS : VS, ubase = isk ? kuse : vuse;
        const int64_t base = isk ? kbase : vbase, step = isk ? kstep : vstep;
        for (int t = 0; t < (tot + 1) / 2 && ok; ++t) {
          const int use = ubase + t, s_ = use % nst;
          for (int h = 0; h < 2 && ok; ++h) {
            const int pos = isk ? s_ * 2 + h : 2 * KS + s_ * 2 + h;
            if (pos % kGatherWarps != g) continue;
            const bool real = 2 * t + h < tot;
            uint64_t* full = isk ? &B.k_full[s_] : &B.v_full[s_];
            if (lane == 0) {
              ok = wt(isk ? &B.k_empty[s_] : &B.v_empty[s_], ((use / nst) & 1) ^ 1, st, 7);
              if (ok) {
                if (!real) mbar_arrive(full);
                else if (!FP8) mbar_arrive_expect_tx(full, (uint32_t)kSlab);
              }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (FP8 && ok && real) {
              // e4m3 rows -> bf16 slab: lane l converts keys l and l + 32 (64 dims each), stores
              // them 128B-swizzled as TMA would, and the warp arrives once its stores are visible
              // to the tensor cores
              uint8_t* dst = (isk ? sk : sv) + s_ * 2 * kSlab + h * kSlab;
              const int col = (isk ? 0 : d0) + (2 * t + h) * 64;
              fp8_rows_to_slab(dst, static_cast<const uint8_t*>(p.k), (base + (int64_t)e0 * step) * args.k_rs + col,
                               (base + (int64_t)e1 * step) * args.k_rs + col, sc0, sc1, lane);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) mbar_arrive(full);
            } else if (ok && real && lane < 16) {
              uint8_t* dst = (isk ? sk : sv) + s_ * 2 * kSlab + h * kSlab + quad * 512;
              gather4(dst, isk ? &tmk : &tmv, full, (isk ? 0 : d0) + (2 * t + h) * 64, (int)(base + kq[0] * step),
                      (int)(base + kq[1] * step), (int)(base + kq[2] * step), (int)(base + kq[3] * step));
            }
          }
        }
      }
      kuse += (NQ + 1) / 2;
      vuse += (nv + 1) / 2;
      ++job;
    }
  } else if (warp == 1) {
    // ============================================================ S issuer
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, kKeys, false, false);
      int job = 0, kuse = 0, item_i = 0, chunk = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 8))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          if (flags & kFirst)
            if (!(ok = wt(&B.q_full, item_i & 1, st, 9))) break;
          const int sb = chunk & 1;
          if (!(ok = wt(&B.s_empty[sb], ((chunk >> 1) & 1) ^ 1, st, 10))) break;
          tc_fence_after();
          const uint32_t dcol = tmem + kColS + sb * kKeys;
          for (int s = 0; s < NQ && ok; s += 2, ++kuse) {
            const int ks = kuse % KS;
            const int nsl = NQ - s < 2 ? NQ - s : 2;
            if (!(ok = wt(&B.k_full[ks], (kuse / KS) & 1, st, 11))) break;
            for (int h = 0; h < nsl; ++h) {
              const uint64_t kd = smem_desc(smem_u32(sk + ks * 2 * kSlab + h * kSlab), 16, 1024, kSw128);
              const uint64_t qd = smem_desc(smem_u32(sq + (s + h) * kQSlab), 16, 1024, kSw128);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_bf16_ss(dcol, qd + (uint64_t)((k * 32) >> 4), kd + (uint64_t)((k * 32) >> 4), id_s,
                            (s + h + k) != 0);
            }
            mma_commit(&B.k_empty[ks]);
          }
          if (!ok) break;
          mma_commit(&B.s_full[sb]);
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
  } else if (warp == 2) {
    // ============================================================ PV issuer
    if (lane == 0) {
      int job = 0, vuse = 0, item_i = 0, chunk = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 12))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          const int d0 = jd[js].vp * args.dvp;
          const int nv = (min(p.d_v - d0, args.dvp)) / 64;
          if (flags & kFirst)
            if (!(ok = wt(&B.o_empty, (item_i & 1) ^ 1, st, 13))) break;
          if (!(ok = wt(&B.p_full, chunk & 1, st, 14))) break;
          tc_fence_after();
          for (int s = 0; s < nv && ok; s += 2, ++vuse) {
            const int vs = vuse % VS;
            const int nsl = nv - s < 2 ? nv - s : 2;
            if (!(ok = wt(&B.v_full[vs], (vuse / VS) & 1, st, 15))) break;
            // V stage as the MN-major B operand: 64-dim slabs 8 KB apart, 8-key groups 1 KB apart
            const uint64_t vd = smem_desc(smem_u32(sv + vs * 2 * kSlab), kSlab, 1024, kSw128);
            const uint32_t id_o = idesc_bf16(128, 64 * nsl, false, true);
#pragma unroll
            for (int k = 0; k < 4; ++k)   // A = P from TMEM: 16 keys = 8 columns per K step
              mma_bf16_ts(tmem + s * 64, tmem + kColP + k * 8, vd + (uint64_t)((k * 2048) >> 4), id_o,
                          !((flags & kFirst) && k == 0));
            mma_commit(&B.v_empty[vs]);
          }
          if (!ok) break;
          mma_commit(&B.p_empty);
          if (flags & kLast) {
            mma_commit(&B.o_full);
            ++item_i;
          }
          ++chunk;
        }
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else {
    // ============================================================ softmax / epilogue
    const int wq = warp & 3;                    // TMEM lane quadrant
    const int m = wq * 32 + lane;               // head row of the tile
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    float mref = -INFINITY, l = 0.f;
    int job = 0, chunk = 0, item_i = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 16))) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      const uint32_t mlo = d.mlo, mhi = d.mhi;
      const int vp = d.vp;
      const int nd = min(p.d_v - vp * args.dvp, args.dvp);
      // this thread's output row, from the descriptor where it is written (so
      // nothing of it stays live through the chunk)
      auto out_row = [&](const Desc& dd, int& h, bool& hv, __nv_bfloat16*& orow, float*& lrow) {
        h = dd.hk * args.G + dd.hg * 128 + m;                 // query head of this thread
        hv = dd.hg * 128 + m < args.G;
        orow = reinterpret_cast<__nv_bfloat16*>(p.o) + (int64_t)dd.b * p.o_sb + (int64_t)dd.tq * p.o_st +
               (int64_t)h * p.o_sh + dd.vp * args.dvp;
        lrow = p.lse + (int64_t)dd.b * p.l_sb + (int64_t)dd.tq * p.l_st + (int64_t)h * p.l_sh;
      };
      if (flags & kEmpty) {
        int h;
        bool hv;
        __nv_bfloat16* orow;
        float* lrow;
        out_row(d, h, hv, orow, lrow);
        if (hv) {
          for (int i = 0; i < nd; i += 8)
            *reinterpret_cast<uint4*>(orow + i) = make_uint4(0, 0, 0, 0);
          if (vp == 0) *lrow = p.attn_sink ? __ldg(p.attn_sink + h) : -INFINITY;
        }
        warp_arrive(&B.jd_empty[js]);
        ++job;
        continue;
      }
      const int sb = chunk & 1;
      if (!(ok = wtw(&B.s_full[sb], (chunk >> 1) & 1, st, 17))) break;
      tc_fence_after();
      const uint32_t ts = tl + kColS + sb * kKeys;
      // pass 1: the chunk's max over its valid keys (S read in 32-column halves).
      // A chunk whose 64 keys are all valid (every chunk of a row that selects
      // a full top-k) skips the per-key mask tests, which otherwise keep the
      // integer pipe busier than the exponentials keep the MUFU.
      const bool full = (mlo & mhi) == 0xffffffffu;
      const bool compat = (p.compat & SFA_COMPAT_REFERENCE_P) != 0;
      float mc = -INFINITY;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float sv[32];
        tmem_ld32(ts + hh * 32, sv);
        tmem_ld_wait();
        const uint32_t msk = hh ? mhi : mlo;
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mc = fmaxf(mc, sv[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if ((msk >> i) & 1u) mc = fmaxf(mc, sv[i]);
        }
      }
      const float zc = mc * c2;                // finite: the chunk has a valid key
      float mnew = mref, fac = 1.f;
      if (flags & kFirst) {
        mnew = zc;
        l = 0.f;
      } else if (zc > mref + kRescaleLog2) {
        mnew = zc;
        fac = ex2(mref - zc);
      }
      // the P buffer (and O) are free once the previous chunk's PV completed
      if (!(ok = wtw(&B.p_empty, (chunk & 1) ^ 1, st, 18))) break;
      mref = mnew;
      const float nm = -mref;
      // pass 2: P = exp2(S*c - m) for the valid keys, bf16 pairs into this
      // thread's TMEM lane (keys 2i, 2i+1 in column kColP + i)
      float lc = 0.f;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float sv[32];
        tc_fence_after();
        tmem_ld32(ts + hh * 32, sv);
        tmem_ld_wait();
        const uint32_t msk = hh ? mhi : mlo;
        float pk[16];
        if (full && !compat) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = ex2(fmaf(sv[i], c2, nm)), p1 = ex2(fmaf(sv[i + 1], c2, nm));
            lc += p0;
            lc += p1;
            pk[i / 2] = __uint_as_float(pack_bf16x2(p0, p1));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float p0 = ((msk >> i) & 1u) ? ex2(fmaf(sv[i], c2, nm)) : 0.f;
            float p1 = ((msk >> (i + 1)) & 1u) ? ex2(fmaf(sv[i + 1], c2, nm)) : 0.f;
            lc += p0;
            lc += p1;
            if (compat) {
              p0 = ref_p(p0);
              p1 = ref_p(p1);
            }
            pk[i / 2] = __uint_as_float(pack_bf16x2(p0, p1));
          }
        }
        tmem_st16(tl + kColP + hh * 16, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&B.s_empty[sb]);
      // O (and the running sum) to the raised maximum, after P: nothing of the
      // P pass is live here, so the rare rescale costs the common path no
      // registers; PV of this chunk is issued only after p_full below
      if (__any_sync(0xffffffffu, fac != 1.f)) {
        tc_fence_after();
        for (int c0 = 0; c0 < nd; c0 += 16) {
          float o[16];
          tmem_ld16(tl + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= fac;
          tmem_st16(tl + c0, o);
        }
        tmem_st_wait();
        l *= fac;
        tc_fence_before();
      }
      l += lc;
      warp_arrive(&B.p_full);
      ++chunk;
      if (flags & kLast) {
        // epilogue: O / (l + exp(sink)), lse in natural log
        if (!(ok = wtw(&B.o_full, item_i & 1, st, 19))) break;
        tc_fence_after();
        int h;
        bool hv;
        __nv_bfloat16* orow;
        float* lrow;
        out_row(jd[js], h, hv, orow, lrow);
        const float s2 = (p.attn_sink && hv) ? __ldg(p.attn_sink + h) * kLog2e : -INFINITY;
        const float M = fmaxf(mref, s2);
        const float w = ex2(mref - M);
        const float lt = l * w + ex2(s2 - M);
        const float inv = __fdividef(w, lt);
        for (int c0 = 0; c0 < nd; c0 += 32) {
          float o[32];
          tmem_ld32(tl + c0, o);
          tmem_ld_wait();
          if (hv) {
#pragma unroll
            for (int i = 0; i < 32; i += 8)
              *reinterpret_cast<uint4*>(orow + c0 + i) =
                  make_uint4(pack_bf16x2(o[i] * inv, o[i + 1] * inv), pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv),
                             pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv), pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv));
          }
        }
        if (hv && vp == 0) *lrow = (M + lg2(lt)) * kLn2;
        tc_fence_before();
        warp_arrive(&B.o_empty);
        ++item_i;
        mref = -INFINITY;
        l = 0.f;
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
  a.nq = p.d_qk / 64;
  a.dvp = p.d_v < 256 ? p.d_v : 256;
  a.n_vp = (p.d_v + 255) / 256;
  int64_t krows = 0, vrows = 0;
  a.k_rs = gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  a.v_rs = gather_rows(p, p.v_sb, p.v_st, p.v_sh, p.d_v, &vrows);
  if (!a.k_rs || !a.v_rs) { *why = "k/v batch, token and head strides must fold into evenly spaced rows"; return false; }
  a.fp8 = p.kv_dtype == SFA_KV_FP8_E4M3 ? 1 : 0;
  if (krows > INT32_MAX || vrows > INT32_MAX) { *why = "too many kv rows for 32-bit gather coordinates"; return false; }
  // shared memory: Q (nq slabs of 16 KB), K / V rings of 2-slab (16 KB) stages (P is in TMEM)
  const size_t budget = 227 * 1024 - 1024;
  const size_t desc = ((sizeof(Desc) * kJD + 127) / 128) * 128;
  const size_t bars = ((sizeof(Bars) + 127) / 128) * 128;
  const size_t fixed = (size_t)a.nq * kQSlab + desc + bars;
  if (fixed + 4 * 2 * kSlab > budget) { *why = "head dims too large for shared memory"; return false; }
  // grow the K ring first (MLA: 3 K + 2 V stages measured 68.5 ms at c4
  // against 74.6 for 2 K + 3 V)
  int ks = 2, vs = 2;
  while (fixed + (size_t)(ks + vs + 1) * 2 * kSlab <= budget && ks + vs < 8) {
    if (ks <= vs) ++ks; else ++vs;
  }
  a.kst = ks;
  a.vst = vs;
  a.off_k = (uint32_t)a.nq * kQSlab;
  a.off_v = a.off_k + ks * 2 * kSlab;
  a.off_desc = a.off_v + vs * 2 * kSlab;
  a.off_bar = a.off_desc + (uint32_t)desc;
  out->smem = a.off_bar + bars + 1024;
  a.nrows = num_rows_host(p);
  a.nitems = a.nrows * p.h_kv * a.n_hg * a.n_vp;
  return true;
}

}  // namespace tokf

bool tok_fwd_supported(const SfaParams& p, const char** why) {
  if (device_cc() != 100) { *why = "needs an sm_100 device"; return false; }
  if (p.block_size != 1) { *why = "token-level family: block_size must be 1"; return false; }
  if (p.topk > tokf::kMaxTopk) { *why = "token-level family: topk must be <= 2048"; return false; }
  if (p.d_qk % 64 || p.d_v % 64 || p.d_qk > 576 || p.d_v > 576) {
    *why = "token-level family: head dims must be multiples of 64, at most 576";
    return false;
  }
  if (!(p.scale > 0.f)) { *why = "needs a positive softmax scale"; return false; }
  const bool fp8 = p.kv_dtype == SFA_KV_FP8_E4M3;
  // fp8 kv rows are read 16 bytes at a time: byte strides multiples of 16
  const bool kv_ok = fp8 ? ((reinterpret_cast<uintptr_t>(p.k) & 15) == 0 && p.k_sb % 16 == 0 && p.k_st % 16 == 0 &&
                            p.k_sh % 16 == 0)
                         : (tma_compatible(p.k, p.k_sb, p.k_st, p.k_sh) && tma_compatible(p.v, p.v_sb, p.v_st, p.v_sh));
  if (!tma_compatible(p.q, p.q_sb, p.q_st, p.q_sh) || !kv_ok) {
    *why = "q/k/v need 16-byte aligned base and strides";
    return false;
  }
  if ((p.o_sh % 8) || (p.o_st % 8) || (p.o_sb % 8) || (reinterpret_cast<uintptr_t>(p.o) & 15)) {
    *why = "o needs a 16-byte aligned base and strides";
    return false;
  }
  tokf::Plan pl;
  return tokf::plan(p, &pl, why);
}

cudaError_t launch_fwd_tok(const SfaParams& p, cudaStream_t stream) {
  tokf::Plan pl;
  const char* why = "";
  if (!tokf::plan(p, &pl, &why)) return cudaErrorInvalidValue;
  tokf::Args& a = pl.a;
  if (a.nitems == 0) return cudaSuccess;
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len;
  const int64_t nb = vl ? 1 : p.batch;
  CUtensorMap tq, tk, tv;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)p.d_qk, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)a.HG, 1u, 1u});
  if (e != cudaSuccess) return e;
  if (a.fp8) {
    // fp8 rows are converted by the gather warps, not copied by TMA: the maps go unused
    tk = tq;
    tv = tq;
  } else {
    int64_t krows = 0, vrows = 0;
    tok::gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
    tok::gather_rows(p, p.v_sb, p.v_st, p.v_sh, p.d_v, &vrows);
    if ((e = tok::make_tmap_rows(&tk, p.k, (uint64_t)p.d_qk, (uint64_t)krows, a.k_rs)) != cudaSuccess) return e;
    if ((e = tok::make_tmap_rows(&tv, p.v, (uint64_t)p.d_v, (uint64_t)vrows, a.v_rs)) != cudaSuccess) return e;
  }
  a.status = device_status_ptr();
  const bool paged = p.block_table != nullptr;
  auto kern = a.fp8 ? (paged ? tokf::sfa_tok_fwd_kernel<true, true> : tokf::sfa_tok_fwd_kernel<true, false>)
                    : (paged ? tokf::sfa_tok_fwd_kernel<false, true> : tokf::sfa_tok_fwd_kernel<false, false>);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  kern<<<grid, tokf::kThreads, pl.smem, stream>>>(a, tq, tk, tv);
  note_launch("fwd_tok", stream);
  return cudaGetLastError();
}

}  // namespace sfa
