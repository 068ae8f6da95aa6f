// sfa_tok_bwd.cu — tensor-core SFA backward for token-level top-k (block_size 1)
// on sm_100a, head dims up to 256: dq directly, dk / dv through fp32 reductions
// into the workspace accumulators (query-centric, like the reference's
// `_attn_bwd_dk_dv` atomics, SFA.py:851-853, but one 128-byte line per warp
// instruction and one reduction per selected (key, dim) per head tile).
//
// Work item = (query row, kv head, head tile of up to 128 heads).  Per 64-key
// chunk of the row's selected keys (gathered with tile::gather4, as in the
// token-level forward):
//     S   = Q . K_sel^T          dP  = dO . V_sel^T         (M = 128 heads, N = 64 keys)
//     P   = exp2(S*c - lse2)     dS' = scale * P * (dP - delta)       (one thread per head row)
//     dQ += dS' . K_sel                                      (M = 128 heads, N = D_qk; TMEM for the row)
//     dK^T = Q^T . dS'^T         dV^T = dO^T . P^T           (M = 128 dims, N = 64 keys, K = heads)
// and the dK^T / dV^T tiles are drained from TMEM into fp32 accumulators with
// coalesced reductions (a warp covers 32 consecutive dims of one key row).
// When dk and dv are one buffer (k is v, or v is k's leading dims) dV^T adds
// into the dK^T tiles and one drain serves both.  Formulas: SFA.py:678-714
// (dS, dq), SFA.py:782-853 (dk, dv); delta = rowsum(o * dO) comes from the
// preprocess kernel (SFA.py:590-610) and the sink gradient from its partials.
//
// TMEM (512 columns): S [0, 64), dP [64, 128), dQ [128, 128 + D_qk), then the
// dK^T tiles (64 columns per 128 dims) and, unless merged, the dV^T tiles —
// twice when they fit, so the drain of one chunk overlaps the next chunk's MMAs.
//
// Warp roles (512 threads, one persistent CTA per SM):
//   warp 0          descriptor producer: validity masks, chunk descriptors,
//                   Q and dO of each item (4-D TMA boxes);
//   warp 1          MMA issuer A: S and dP;
//   warp 2          MMA issuer B: dQ, dK^T, dV^T;
//   warps 3, 8-11   gather pool: K (and V) slabs, a fixed owner per ring position;
//   warps 4-7       P / dS' (thread = head row) and the dq epilogue (two-pass
//                   form: the second half of the drain and the dq epilogue);
//   warps 12-15     drain: dK^T / dV^T tiles (thread = dim) -> fp32 reductions.
// Every wait is bounded (~2 s); on expiry the kernel records (5 << 16) | site in
// the status word and returns.
//
// Two-pass form (head dims above 256, sfa_mla_bwd.cu): P and dS' come from the
// workspace the first pass wrote, so S and dP are not formed here.  The work
// item gains a part index (a 192-dim range of the head dims): Q, dO and the K
// slabs of that range only, dQ of the range in TMEM (columns from 0), the P
// and dS' tiles of each chunk loaded by TMA (4-D box: 64 slots x the head
// tile) into two tile buffers, and the drain and the dq epilogue offset to
// the range.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"
#include "sfa_tok_common.cuh"

namespace sfa {
using namespace tc;
using namespace tok;

namespace tokb {

constexpr int kThreads = 512;
constexpr int kGatherWarps = 5;        // warps 3 and 8-11
constexpr int kKeys = 64;
constexpr int kMaxTopk = 32 * kKeys;
constexpr int kJD = 4;
constexpr int kSlab = 64 * 128;        // 64 rows x 64 dims bf16
constexpr int kQSlab = 128 * 128;      // 128 head rows x 64 dims bf16
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSDCols = 128;      // one S / dP buffer: S [0, 64), dP [64, 128)
constexpr int kPartSlabs = 3;          // two-pass form: 64-dim slabs of q/k per part
constexpr int kTileBytes = 2 * kQSlab; // two-pass form: P and dS' tiles of one chunk

enum : int { kFirst = 1, kLast = 2, kEmpty = 4, kSentinel = 8 };

struct Desc {
  uint32_t mlo, mhi;
  int flags;
  int row, hk, hg, b, tq;
  int part, nqi, nvi, chunk, wrow;     // two-pass form: dim part, its q/k and dO slabs, chunk, wave row
  int64_t kbase, vbase;                // gather rows of key 0 (K / V maps)
  int64_t accrow;                      // accumulator row of key 0: b * kv_len (dense) or kv0 (varlen)
  int keys[kKeys];
};

struct Args {
  SfaParams p;
  const float* delta;                  // [rows][h_q]
  float* dk_acc;                       // fp32 [kv_rows][h_kv][d_qk]
  float* dv_acc;                       // fp32 [kv_rows][h_kv][d_v] (unused when merged)
  int nitems, nrows, n_hg, HG, G, nq, nv;
  int vsrc_k;                          // V slabs are the K stage's first nv slabs (v is k's leading dims)
  int merged;                          // dv adds into the dk tiles (one gradient buffer)
  int kst, vst;
  int ntk, ntv;                        // 128-dim tiles of dK^T / dV^T
  uint32_t col_dk, col_dv;
  uint32_t kv_stride;                  // TMEM columns between the two dK^T/dV^T buffers (0: one buffer)
  int nkvb;                            // dK^T/dV^T buffers (2 when TMEM allows)
  uint32_t off_do, off_k, off_v, off_p, off_ds, off_desc, off_bar;
  int64_t k_rs, v_rs;
  int32_t* status;
  // two-pass form
  int parts;                           // dim parts per (row, head tile); 0: one-pass form
  int nq_all, nv_all;                  // 64-dim slabs of d_qk / d_v
  int r0;                              // first row of the wave
  uint32_t col_dq;                     // TMEM column of dQ
  int nsd, npd;                        // S / dP buffers in TMEM, P / dS' tile pairs in shared memory
  uint32_t off_tiles;                  // P / dS' tile buffers [2][kTileBytes]
};

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t sd_full[2], sd_empty[2];    // S / dP in TMEM (double-buffered when TMEM allows)
  uint64_t pd_full[2], pd_empty[2];    // P / dS' tiles in shared memory (double-buffered when it fits)
  uint64_t dq_full, dq_empty;          // dQ accumulator
  uint64_t kv_full[2], kv_empty[2];    // dK^T / dV^T tiles (double-buffered when TMEM allows)
  uint64_t jd_full[kJD], jd_empty[kJD];
  uint32_t tmem_base;
  uint32_t pad;
  uint64_t k_full[4], k_empty[4], v_full[4], v_empty[4];
  uint64_t t_full[2], t_empty[2];      // two-pass form: P / dS' tile buffers
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (5 << 16) | site);
  return false;
}

__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

__device__ __forceinline__ void decode_item(const Args& a, int item, int& row, int& hk, int& hg, int& part) {
  part = 0;
  if (a.parts) {
    part = item % a.parts;              // the parts of one row run side by side: its P / dS' rows stay in L2
    item /= a.parts;
  }
  hg = item % a.n_hg;
  const int r = item / a.n_hg;
  hk = r % a.p.h_kv;
  row = a.r0 + r / a.p.h_kv;
}

// TWO: the two-pass form's gradient half (its own instantiation, so the
// one-pass kernel carries none of its checks)
template <bool TWO>
__global__ void __launch_bounds__(kThreads, 1)
sfa_tok_bwd_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmp,
                   const __grid_constant__ CUtensorMap tmds) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaParams& p = args.p;
  uint8_t* sq = sbase;
  uint8_t* sdo = sbase + args.off_do;
  uint8_t* sk = sbase + args.off_k;
  uint8_t* sv = sbase + args.off_v;
  uint8_t* spp = sbase + args.off_p;
  uint8_t* sds = sbase + args.off_ds;
  uint8_t* stile = sbase + args.off_tiles;
  constexpr bool two = TWO;
  Desc* jd = reinterpret_cast<Desc*>(sbase + args.off_desc);
  Bars& B = *reinterpret_cast<Bars*>(sbase + args.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* st = args.status;
  const int KS = args.kst, VS = args.vst, NQ = args.nq, NV = args.nv;
  const int kstage = NQ * kSlab, vstage = NV * kSlab;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.sd_full[i], 1);
      mbar_init(&B.sd_empty[i], 4);
      mbar_init(&B.pd_full[i], 4);
      mbar_init(&B.pd_empty[i], 1);
    }
    mbar_init(&B.dq_full, 1);
    mbar_init(&B.dq_empty, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.kv_full[i], 1);
      mbar_init(&B.kv_empty[i], two ? 8 : 4);     // the two-pass form drains from eight warps
    }
    // consumers of a descriptor: two MMA issuers (one in the two-pass form), the
    // gather pool, P/dS warps, drain warps
    for (int i = 0; i < kJD; ++i) {
      mbar_init(&B.jd_full[i], 1);
      mbar_init(&B.jd_empty[i], (two ? 1 : 2) + kGatherWarps + 4 + 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.t_full[i], 1);
      mbar_init(&B.t_empty[i], 1);
    }
    // one arrival per slab position of a stage
    for (int i = 0; i < KS; ++i) { mbar_init(&B.k_full[i], NQ); mbar_init(&B.k_empty[i], 1); }
    for (int i = 0; i < VS; ++i) { mbar_init(&B.v_full[i], NV); mbar_init(&B.v_empty[i], 1); }
    fence_barrier_init();
  }
  // head rows past the tile's HG stay zero (TMA writes HG rows of Q and dO, and
  // of the two-pass form's P / dS' tiles)
  if (args.HG < 128) {
    for (int i = threadIdx.x; i < (NQ + NV) * kQSlab / 16; i += kThreads)   // Q and dO are adjacent
      reinterpret_cast<uint4*>(sq)[i] = make_uint4(0, 0, 0, 0);
    if (two)
      for (int i = threadIdx.x; i < 2 * kTileBytes / 16; i += kThreads)
        reinterpret_cast<uint4*>(stile)[i] = make_uint4(0, 0, 0, 0);
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
    prefetch_tmap(&tmv);
    if (two) {
      prefetch_tmap(&tmp);
      prefetch_tmap(&tmds);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;
  const int quad = lane & 15;

  // Drain of one chunk's dK^T / dV^T tiles (TMEM lanes = dims, columns = keys)
  // into the fp32 accumulators, key halves [h_lo, h_hi) of 32 keys each.  Each
  // lane holds two of the chunk's keys (i and i + 32) and those keys'
  // accumulator rows; a reduction takes its key's row from the owning lane by
  // shuffle, so the loop is shuffle + reduction, a warp covering 32
  // consecutive dims (128 bytes) of one key per instruction.
  auto drain_chunk = [&](const Desc& d, int chunk, int h_lo, int h_hi, int site) -> bool {
    const int wq = warp & 3;                 // TMEM lanes 32*wq.. = dims 32*wq.. of a 128-dim tile
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t mlo = d.mlo, mhi = d.mhi;
    // accumulator row (units of h_kv-head rows; below 2^31, as the gather rows) of keys lane, lane + 32
    const int r0 = (int)((d.accrow + d.keys[lane]) * p.h_kv + d.hk);
    const int r1 = (int)((d.accrow + d.keys[lane + 32]) * p.h_kv + d.hk);
    // dims of this item (the part's, in the two-pass form) and its tiles
    const int nk = d.nqi * 64, nv = d.nvi * 64, d0 = two ? d.part * kPartSlabs * 64 : 0;
    const int ntk = (nk + 127) / 128, ntv = (nv + 127) / 128;
    const int kb = args.nkvb == 2 ? (chunk & 1) : 0;
    const int kuse_b = args.nkvb == 2 ? (chunk >> 1) : chunk;
    if (!wtw(&B.kv_full[kb], kuse_b & 1, st, site)) return false;
    tc_fence_after();
    for (int t = 0; t < ntk + (args.merged ? 0 : ntv); ++t) {
      const bool isk = t < ntk;
      const int j = isk ? t : t - ntk;
      const int D = isk ? p.d_qk : p.d_v;
      float* acc = (isk ? args.dk_acc : args.dv_acc) + d0 + 128 * j + 32 * wq + lane;
      const bool dim_ok = 128 * j + 32 * wq + lane < (isk ? nk : nv);
      const uint32_t col = kb * args.kv_stride + (isk ? args.col_dk + 64 * j : args.col_dv + 64 * j);
      for (int hh = h_lo; hh < h_hi; ++hh) {
        float v[32];
        tmem_ld32(tl + col + 32 * hh, v);
        tmem_ld_wait();
        const uint32_t msk = hh ? mhi : mlo;
        const int rr = hh ? r1 : r0;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int ri = __shfl_sync(0xffffffffu, rr, i);
          if (((msk >> i) & 1u) && dim_ok) atomicAdd(acc + (int64_t)ri * D, v[i]);
        }
      }
    }
    tc_fence_before();
    warp_arrive(&B.kv_empty[kb]);
    return true;
  };

  if (warp == 0) {
    // ============================================================ descriptor producer
    int job = 0, item_i = 0, tile = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.nitems && ok; item += gridDim.x) {
      int row, hk, hg, part;
      decode_item(args, item, row, hk, hg, part);
      const Row r = row_info(p, row);
      // slabs of this item's dims: all of them, or the part's (two-pass form)
      const int s0q = part * kPartSlabs;
      const int nqi = two ? min(kPartSlabs, args.nq_all - s0q) : NQ;
      const int nvi = two ? max(0, min(kPartSlabs, args.nv_all - s0q)) : NV;
      const int32_t* idx = p.block_indices + r.b * p.i_sb + r.tq * p.i_st + (int64_t)hk * p.i_sh;
      const int nch = (p.topk + kKeys - 1) / kKeys;
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
      const int64_t accrow = p.cu_seqlens_q == nullptr ? (int64_t)r.b * p.kv_len : r.kv0;
      if (chunks == 0u) {
        // nothing selected: dq of the tile is zero and nothing reaches dk / dv
        if (lane == 0) {
          const int js = job % kJD;
          ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 1);
          if (ok) {
            Desc& d = jd[js];
            d.flags = kFirst | kLast | kEmpty;
            d.row = row; d.hk = hk; d.hg = hg; d.b = r.b; d.tq = (int)r.tq;
            d.part = part; d.nqi = nqi; d.nvi = nvi;
            mbar_arrive(&B.jd_full[js]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        ++job;
        continue;
      }
      if (lane == 0) {
        ok = wt(&B.q_empty, (item_i & 1) ^ 1, st, 2);
        if (ok) {
          mbar_arrive_expect_tx(&B.q_full, (uint32_t)(args.HG * 128 * (nqi + nvi)));
          for (int s = 0; s < nqi; ++s)
            tma_load_4d(sq + s * kQSlab, &tmq, &B.q_full, (s0q + s) * 64, hk * args.G + hg * 128, (int)r.tq, r.b);
          for (int s = 0; s < nvi; ++s)
            tma_load_4d(sdo + s * kQSlab, &tmdo, &B.q_full, (s0q + s) * 64, hk * args.G + hg * 128, (int)r.tq,
                        r.b);
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
        const int fl = lo ? __ffs(lo) - 1 : __ffs(hi) - 1;
        const int f0 = __shfl_sync(0xffffffffu, e0, fl), f1 = __shfl_sync(0xffffffffu, e1, fl);
        const int fk = lo ? f0 : f1;
        if (!((lo >> lane) & 1u)) e0 = fk;
        if (!((hi >> lane) & 1u)) e1 = fk;
        const int js = job % kJD;
        if (lane == 0) ok = wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 3);
        // two-pass form: this chunk's P and dS' tiles into tile buffer tile % 2
        if (two && lane == 0 && ok) {
          const int tb = tile & 1;
          ok = wt(&B.t_empty[tb], ((tile >> 1) & 1) ^ 1, st, 22);
          if (ok) {
            mbar_arrive_expect_tx(&B.t_full[tb], (uint32_t)(2 * args.HG * 128));
            uint8_t* tdst = stile + tb * kTileBytes;
            const int wrow = row - args.r0;
            tma_load_4d(tdst, &tmp, &B.t_full[tb], c * kKeys, hk * args.G + hg * 128, wrow, 0);
            tma_load_4d(tdst + kQSlab, &tmds, &B.t_full[tb], c * kKeys, hk * args.G + hg * 128, wrow, 0);
          }
        }
        if (two) ++tile;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        Desc& d = jd[js];
        d.keys[lane] = e0;
        d.keys[lane + 32] = e1;
        if (lane == 0) {
          d.mlo = lo; d.mhi = hi;
          d.flags = (c == cfirst ? kFirst : 0) | (c == clast ? kLast : 0);
          d.row = row; d.hk = hk; d.hg = hg; d.b = r.b; d.tq = (int)r.tq;
          d.part = part; d.nqi = nqi; d.nvi = nvi; d.chunk = c;
          d.kbase = kbase; d.vbase = vbase; d.accrow = accrow;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.jd_full[js]);
      }
    }
    if (lane == 0 && ok) {
      const int js = job % kJD;
      if (wt(&B.jd_empty[js], ((job / kJD) & 1) ^ 1, st, 4)) {
        jd[js].flags = kSentinel;
        mbar_arrive(&B.jd_full[js]);
      }
    }
  } else if (warp == 3 || (warp >= 8 && warp < 12)) {
    // ============================================================ gather pool
    // A fixed owner per (ring, stage slot, slab) position; each owner takes part
    // in every use of its slot in order (see the token-level forward).
    const int g = warp == 3 ? 0 : warp - 7;
    const int64_t kstep = p.k_st / args.k_rs, vstep = p.v_st / args.v_rs;
    int job = 0, kuse = 0, vuse = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 5);
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
      const int64_t kbase = d.kbase, vbase = d.vbase;
      const int nqi = d.nqi, kcol0 = d.part * kPartSlabs;
      __syncwarp();
      if (lane == 0) mbar_arrive(&B.jd_empty[js]);
      int kq[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int src = (4 * quad + i) & 31;
        const int a = __shfl_sync(0xffffffffu, e0, src), bb = __shfl_sync(0xffffffffu, e1, src);
        kq[i] = quad < 8 ? a : bb;
      }
      for (int r = 0; r < 2 && ok; ++r) {
        const bool isk = r == 0;
        if (!isk && args.vsrc_k) break;
        const int n = isk ? NQ : NV, nst = isk ? KS : VS, use = isk ? kuse : vuse, s_ = use % nst;
        const int64_t base = isk ? kbase : vbase, step = isk ? kstep : vstep;
        for (int sl = 0; sl < n && ok; ++sl) {
          const int pos = isk ? s_ * NQ + sl : KS * NQ + s_ * NV + sl;
          if (pos % kGatherWarps != g) continue;
          uint64_t* full = isk ? &B.k_full[s_] : &B.v_full[s_];
          // a K slot of a part with fewer slabs (two-pass form) gets a plain arrive
          const bool real = !isk || sl < nqi;
          if (lane == 0) {
            ok = wt(isk ? &B.k_empty[s_] : &B.v_empty[s_], ((use / nst) & 1) ^ 1, st, 6);
            if (ok) {
              if (real) mbar_arrive_expect_tx(full, (uint32_t)kSlab);
              else mbar_arrive(full);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
          if (ok && real && lane < 16)
            gather4((isk ? sk + s_ * kstage : sv + s_ * vstage) + sl * kSlab + quad * 512, isk ? &tmk : &tmv, full,
                    ((isk ? kcol0 : 0) + sl) * 64, (int)(base + kq[0] * step), (int)(base + kq[1] * step),
                    (int)(base + kq[2] * step), (int)(base + kq[3] * step));
        }
      }
      ++kuse;
      ++vuse;
      ++job;
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer A: S, dP
    // (the two-pass form has no S / dP: P and dS' come from the workspace)
    if (lane == 0 && !two) {
      const uint32_t id_s = idesc_bf16(128, kKeys, false, false);
      int job = 0, kuse = 0, vuse = 0, item_i = 0, chunk = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 7))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          if (flags & kFirst) {
            if (!(ok = wt(&B.q_full, item_i & 1, st, 8))) break;
            ++item_i;
          }
          const int sb = chunk % args.nsd;
          if (!(ok = wt(&B.sd_empty[sb], ((chunk / args.nsd) & 1) ^ 1, st, 9))) break;
          const int ks = kuse % KS;
          if (!(ok = wt(&B.k_full[ks], (kuse / KS) & 1, st, 10))) break;
          tc_fence_after();
          for (int s = 0; s < NQ; ++s) {
            const uint64_t kd = smem_desc(smem_u32(sk + ks * kstage + s * kSlab), 16, 1024, kSw128);
            const uint64_t qd = smem_desc(smem_u32(sq + s * kQSlab), 16, 1024, kSw128);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16_ss(tmem + sb * kSDCols, qd + (uint64_t)((k * 32) >> 4), kd + (uint64_t)((k * 32) >> 4), id_s,
                          (s | k) != 0);
          }
          const uint8_t* vstg = sk + ks * kstage;
          int vs = 0;
          if (!args.vsrc_k) {
            vs = vuse % VS;
            if (!(ok = wt(&B.v_full[vs], (vuse / VS) & 1, st, 11))) break;
            vstg = sv + vs * vstage;
          }
          for (int s = 0; s < NV; ++s) {
            const uint64_t vd = smem_desc(smem_u32(vstg + s * kSlab), 16, 1024, kSw128);
            const uint64_t od = smem_desc(smem_u32(sdo + s * kQSlab), 16, 1024, kSw128);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16_ss(tmem + sb * kSDCols + 64, od + (uint64_t)((k * 32) >> 4), vd + (uint64_t)((k * 32) >> 4), id_s,
                          (s | k) != 0);
          }
          if (!args.vsrc_k) mma_commit(&B.v_empty[vs]);
          mma_commit(&B.sd_full[sb]);
          ++kuse;
          ++vuse;
          ++chunk;
        }
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp == 2) {
    // ============================================================ MMA issuer B: dQ, dK^T, dV^T
    if (lane == 0) {
      const uint32_t id_kv = idesc_bf16(128, kKeys, true, true);
      int job = 0, kuse = 0, item_i = 0, chunk = 0;
      bool ok = true;
      while (ok) {
        const int js = job % kJD;
        if (!(ok = wt(&B.jd_full[js], (job / kJD) & 1, st, 12))) break;
        const int flags = jd[js].flags;
        if (flags & kSentinel) break;
        if (!(flags & kEmpty)) {
          const int nqi = jd[js].nqi, nvi = jd[js].nvi;
          // P and dS' tiles: formed in this kernel, or (two-pass form) tile buffer chunk % 2
          const int pb = chunk % args.npd;
          const uint8_t* tp = two ? stile + (chunk & 1) * kTileBytes : spp + pb * 32768;
          const uint8_t* tds = two ? tp + kQSlab : sds + pb * 32768;
          const uint64_t dsd = smem_desc(smem_u32(tds), 16, 1024, kSw128);    // dS' [heads][keys], K-major
          const uint64_t dst_ = smem_desc(smem_u32(tds), 0, 1024, kSw128);    // dS'^T as MN-major B
          const uint64_t pt = smem_desc(smem_u32(tp), 0, 1024, kSw128);       // P^T as MN-major B
          const uint32_t id_q = idesc_bf16(128, (uint32_t)(nqi * 64), false, true);
          const int ntk = two ? (nqi * 64 + 127) / 128 : args.ntk;
          const int ntv = two ? (nvi * 64 + 127) / 128 : args.ntv;
          if (flags & kFirst) {
            if (!(ok = wt(&B.dq_empty, (item_i & 1) ^ 1, st, 13))) break;
            if (two && !(ok = wt(&B.q_full, item_i & 1, st, 23))) break;
          }
          if (two) {
            if (!(ok = wt(&B.t_full[chunk & 1], (chunk >> 1) & 1, st, 24))) break;
            if (!(ok = wt(&B.k_full[kuse % KS], (kuse / KS) & 1, st, 25))) break;
          } else if (!(ok = wt(&B.pd_full[pb], (chunk / args.npd) & 1, st, 14))) {
            break;
          }
          const int kb = args.nkvb == 2 ? (chunk & 1) : 0;
          const int kuse_b = args.nkvb == 2 ? (chunk >> 1) : chunk;
          if (!(ok = wt(&B.kv_empty[kb], (kuse_b & 1) ^ 1, st, 15))) break;
          tc_fence_after();
          const uint32_t kvoff = kb * args.kv_stride;
          const int ks = kuse % KS;
          // dQ += dS' . K: K stage as MN-major B (64-dim slabs 8 KB apart, 8-key groups 1 KB apart)
          const uint64_t kmn = smem_desc(smem_u32(sk + ks * kstage), kSlab, 1024, kSw128);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tmem + args.col_dq, dsd + (uint64_t)((k * 32) >> 4), kmn + (uint64_t)((k * 2048) >> 4), id_q,
                        !((flags & kFirst) && k == 0));
          // dK^T tile j = Q^T (dims 128j.., MN-major: 64-dim slabs 16 KB apart) . dS'^T
          for (int j = 0; j < ntk; ++j) {
            const uint64_t qt = smem_desc(smem_u32(sq + 2 * j * kQSlab), kQSlab, 1024, kSw128);
            for (int k = 0; k < 8; ++k)
              mma_bf16_ss(tmem + kvoff + args.col_dk + 64 * j, qt + (uint64_t)((k * 2048) >> 4),
                          dst_ + (uint64_t)((k * 2048) >> 4), id_kv, k != 0);
          }
          for (int j = 0; j < ntv; ++j) {
            const uint64_t ot = smem_desc(smem_u32(sdo + 2 * j * kQSlab), kQSlab, 1024, kSw128);
            const uint32_t col = kvoff + (args.merged ? args.col_dk + 64 * j : args.col_dv + 64 * j);
            for (int k = 0; k < 8; ++k)
              mma_bf16_ss(tmem + col, ot + (uint64_t)((k * 2048) >> 4), pt + (uint64_t)((k * 2048) >> 4), id_kv,
                          args.merged || k != 0);
          }
          mma_commit(&B.k_empty[ks]);
          mma_commit(two ? &B.t_empty[chunk & 1] : &B.pd_empty[pb]);
          mma_commit(&B.kv_full[kb]);
          if (flags & kLast) {
            mma_commit(&B.dq_full);
            mma_commit(&B.q_empty);
            ++item_i;
          }
          ++kuse;
          ++chunk;
        }
        mbar_arrive(&B.jd_empty[js]);
        ++job;
      }
    }
  } else if (warp < 8) {
    // ============================================================ P / dS' + dq epilogue
    const int wq = warp & 3;
    const int m = wq * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = p.scale * kLog2e;
    float lse2 = -INFINITY, dl = 0.f;
    int job = 0, chunk = 0, item_i = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 16))) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      const int h = d.hk * args.G + d.hg * 128 + m;
      const bool hv = d.hg * 128 + m < args.G;
      const uint32_t mlo = d.mlo, mhi = d.mhi;
      // dq dims of this item: all, or the part's (two-pass form)
      const int dqn = d.nqi * 64;
      // the dq row, from the descriptor where it is written (nothing of it stays
      // live through the chunk)
      auto dq_row = [&](const Desc& dd) {
        return reinterpret_cast<__nv_bfloat16*>(p.dq) + (int64_t)dd.b * p.dq_sb + (int64_t)dd.tq * p.dq_st +
               (int64_t)(dd.hk * args.G + dd.hg * 128 + m) * p.dq_sh + (two ? dd.part * kPartSlabs * 64 : 0);
      };
      if (flags & kEmpty) {
        __nv_bfloat16* dqrow = dq_row(d);
        if (hv)
          for (int i = 0; i < dqn; i += 8) *reinterpret_cast<uint4*>(dqrow + i) = make_uint4(0, 0, 0, 0);
        warp_arrive(&B.jd_empty[js]);
        ++job;
        continue;
      }
      if (two) {
        // P and dS' come from the workspace: these warps drain keys 32-63 of the
        // chunk's dK^T / dV^T tiles and run the dq epilogue
        if (!(ok = drain_chunk(d, chunk, 1, 2, 27))) break;
        ++chunk;
        if (flags & kLast) {
          if (!(ok = wtw(&B.dq_full, item_i & 1, st, 26))) break;
          tc_fence_after();
          __nv_bfloat16* dqrow = dq_row(d);
          for (int c0 = 0; c0 < dqn; c0 += 32) {
            float o[32];
            tmem_ld32(tl + args.col_dq + c0, o);
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
        warp_arrive(&B.jd_empty[js]);
        ++job;
        continue;
      }
      if (flags & kFirst) {
        lse2 = hv ? __ldg(p.lse + (int64_t)d.b * p.l_sb + (int64_t)d.tq * p.l_st + (int64_t)h * p.l_sh) * kLog2e
                  : -INFINITY;
        dl = hv ? __ldg(args.delta + (int64_t)d.row * p.h_q + h) : 0.f;
        if (!(lse2 > -INFINITY)) lse2 = INFINITY;          // a row with no mass: P = 0
      }
      // the P / dS' tiles are free once the previous chunk's MMAs read them
      const int pb = chunk % args.npd, sb = chunk % args.nsd;
      if (!(ok = wtw(&B.pd_empty[pb], ((chunk / args.npd) & 1) ^ 1, st, 17))) break;
      if (!(ok = wtw(&B.sd_full[sb], (chunk / args.nsd) & 1, st, 18))) break;
      tc_fence_after();
      const uint32_t prow = smem_u32(spp + pb * 32768) + m * 128, drow = smem_u32(sds + pb * 32768) + m * 128;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float sv[32], dv[32];
        tmem_ld32(tl + sb * kSDCols + hh * 32, sv);
        tmem_ld32(tl + sb * kSDCols + 64 + hh * 32, dv);
        tmem_ld_wait();
        const uint32_t msk = hv ? (hh ? mhi : mlo) : 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float pr[8], ds[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int kk = 8 * j + i;
            pr[i] = ((msk >> kk) & 1u) ? ex2(fmaf(sv[kk], c2, -lse2)) : 0.f;
            ds[i] = p.scale * pr[i] * (dv[kk] - dl);
          }
          const int jj = 4 * hh + j;
          st_shared_v4(prow + ((jj ^ (m & 7)) << 4), pack_bf16x2(pr[0], pr[1]), pack_bf16x2(pr[2], pr[3]),
                       pack_bf16x2(pr[4], pr[5]), pack_bf16x2(pr[6], pr[7]));
          st_shared_v4(drow + ((jj ^ (m & 7)) << 4), pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]),
                       pack_bf16x2(ds[4], ds[5]), pack_bf16x2(ds[6], ds[7]));
        }
      }
      tc_fence_before();
      warp_arrive(&B.sd_empty[sb]);
      fence_proxy_async_smem();
      warp_arrive(&B.pd_full[pb]);
      ++chunk;
      if (flags & kLast) {
        if (!(ok = wtw(&B.dq_full, item_i & 1, st, 19))) break;
        tc_fence_after();
        __nv_bfloat16* dqrow = dq_row(d);
        for (int c0 = 0; c0 < dqn; c0 += 32) {
          float o[32];
          tmem_ld32(tl + args.col_dq + c0, o);
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
      warp_arrive(&B.jd_empty[js]);
      ++job;
    }
  } else {
    // ============================================================ drain (warps 12-15)
    // (keys 0-31 of each chunk in the two-pass form, where warps 4-7 take 32-63)
    int job = 0, chunk = 0;
    bool ok = true;
    while (ok) {
      const int js = job % kJD;
      if (!(ok = wtw(&B.jd_full[js], (job / kJD) & 1, st, 20))) break;
      const Desc& d = jd[js];
      const int flags = d.flags;
      if (flags & kSentinel) break;
      if (!(flags & kEmpty)) {
        if (!(ok = drain_chunk(d, chunk, 0, two ? 1 : 2, 21))) break;
        ++chunk;
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

// two: the two-pass form's gradient half (parts of kPartSlabs slabs; P and dS'
// from the workspace)
static bool plan(const SfaParams& p, Plan* out, const char** why, bool two = false) {
  const int G = p.h_q / p.h_kv;
  Args& a = out->a;
  a = Args{};
  a.p = p;
  a.G = G;
  a.HG = G < 128 ? G : 128;
  a.n_hg = (G + 127) / 128;
  if (G > 128 && G % 128) { *why = "query heads per kv head must be <= 128 or a multiple of 128"; return false; }
  a.nq_all = p.d_qk / 64;
  a.nv_all = p.d_v / 64;
  a.parts = two ? (a.nq_all + kPartSlabs - 1) / kPartSlabs : 0;
  a.nq = two ? kPartSlabs : a.nq_all;
  a.nv = two ? kPartSlabs : a.nv_all;
  int64_t krows = 0, vrows = 0;
  a.k_rs = gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  a.v_rs = gather_rows(p, p.v_sb, p.v_st, p.v_sh, p.d_v, &vrows);
  if (!a.k_rs || !a.v_rs) { *why = "k/v batch, token and head strides must fold into evenly spaced rows"; return false; }
  if (krows > INT32_MAX || vrows > INT32_MAX) { *why = "too many kv rows for 32-bit gather coordinates"; return false; }
  // the two-pass form gathers no V (dP is not formed here)
  a.vsrc_k = (two || (p.v == p.k && p.v_sb == p.k_sb && p.v_st == p.k_st && p.v_sh == p.k_sh && p.d_v <= p.d_qk))
                 ? 1 : 0;
  a.merged = p.dk == p.dv ? 1 : 0;
  a.ntk = (a.nq * 64 + 127) / 128;
  a.ntv = (a.nv * 64 + 127) / 128;
  // TMEM: S / dP buffers (one-pass form; two when they fit beside the rest, so
  // the next chunk's S and dP are formed while the P / dS' warps read this
  // one's), dQ, dK^T tiles, dV^T tiles
  auto layout = [&](int nsd) {
    a.nsd = nsd;
    a.col_dq = two ? 0u : (uint32_t)nsd * kSDCols;
    a.col_dk = a.col_dq + (uint32_t)(a.nq * 64);
    a.col_dv = a.col_dk + 64u * a.ntk;
    return a.col_dv + (a.merged ? 0u : 64u * a.ntv);
  };
  uint32_t cols = layout(two ? 1 : 2);
  if (cols > kTmemCols && !two) cols = layout(1);
  if (cols > kTmemCols) { *why = "token-level backward: dQ plus the dK/dV tiles exceed tensor memory"; return false; }
  // a second dK^T/dV^T buffer lets the next chunk's MMAs run while the drain reads this one
  a.kv_stride = cols - a.col_dk;
  a.nkvb = cols + a.kv_stride <= kTmemCols ? 2 : 1;
  if (a.nkvb == 1) a.kv_stride = 0;
  // shared memory: Q, dO (16 KB slabs), K ring (full-chunk stages), V ring, and
  // the P and dS' tiles (formed here: one pair; two-pass form: two pairs loaded by TMA)
  const size_t budget = 227 * 1024 - 1024;
  const size_t desc = ((sizeof(Desc) * kJD + 127) / 128) * 128;
  const size_t bars = ((sizeof(Bars) + 127) / 128) * 128;
  const size_t kst = (size_t)a.nq * kSlab, vst = a.vsrc_k ? 0 : (size_t)a.nv * kSlab;
  // regions after Q / dO must cover the 128-dim tiles the dK^T / dV^T MMAs read
  // (a 64-dim Q or dO reads its neighbour's slab for the ignored rows)
  int ks = 2, vs = a.vsrc_k ? 0 : 2;
  // one P / dS' pair: a second one (the P / dS' warps a chunk ahead of the
  // gradient MMAs) measured slower at tok128, 8.76 against 8.38 ms for the
  // backward, while a second S / dP buffer in TMEM measured even (8.34)
  a.npd = 1;
  const size_t tiles = two ? 2 * (size_t)kTileBytes : (size_t)a.npd * 32768;
  const size_t fixed = (size_t)(a.nq + a.nv) * kQSlab + tiles + desc + bars;
  if (fixed + ks * kst + vs * vst > budget) { *why = "head dims too large for shared memory"; return false; }
  while (ks < 4 || (!a.vsrc_k && vs < 4)) {
    const bool grow_k = a.vsrc_k || ks <= vs;
    const size_t add = grow_k ? kst : vst;
    if ((grow_k ? ks : vs) >= 4 || fixed + ks * kst + vs * vst + add > budget) break;
    if (grow_k) ++ks; else ++vs;
  }
  a.kst = ks;
  a.vst = vs;
  a.off_do = (uint32_t)a.nq * kQSlab;
  a.off_k = a.off_do + (uint32_t)a.nv * kQSlab;
  a.off_v = a.off_k + (uint32_t)(ks * kst);
  a.off_p = a.off_v + (uint32_t)(vs * vst);
  a.off_ds = a.off_p + 16384;
  a.off_tiles = a.off_p;
  a.off_desc = a.off_p + (uint32_t)tiles;
  a.off_bar = a.off_desc + (uint32_t)desc;
  out->smem = a.off_bar + bars + 1024;
  a.nrows = num_rows_host(p);
  a.nitems = a.nrows * p.h_kv * a.n_hg;
  return true;
}

static cudaError_t launch(const Plan& pl, const SfaParams& p, const CUtensorMap& tp, const CUtensorMap& tds,
                          cudaStream_t stream) {
  const Args& a = pl.a;
  const bool vl = p.cu_seqlens_q != nullptr;
  const int64_t qrows = vl ? p.total_q : p.q_len;
  const int64_t nb = vl ? 1 : p.batch;
  CUtensorMap tq, tdo, tk, tv;
  cudaError_t e = make_tmap_bf16_4d(&tq, p.q, {(uint64_t)p.d_qk, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                                    {p.q_sh, p.q_st, p.q_sb}, {64u, (uint32_t)a.HG, 1u, 1u});
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_4d(&tdo, p.dout, {(uint64_t)p.d_v, (uint64_t)p.h_q, (uint64_t)qrows, (uint64_t)nb},
                        {p.do_sh, p.do_st, p.do_sb}, {64u, (uint32_t)a.HG, 1u, 1u});
  if (e != cudaSuccess) return e;
  int64_t krows = 0, vrows = 0;
  gather_rows(p, p.k_sb, p.k_st, p.k_sh, p.d_qk, &krows);
  gather_rows(p, p.v_sb, p.v_st, p.v_sh, p.d_v, &vrows);
  if ((e = make_tmap_rows(&tk, p.k, (uint64_t)p.d_qk, (uint64_t)krows, a.k_rs)) != cudaSuccess) return e;
  if ((e = make_tmap_rows(&tv, p.v, (uint64_t)p.d_v, (uint64_t)vrows, a.v_rs)) != cudaSuccess) return e;
  auto kern = a.parts ? tokb::sfa_tok_bwd_kernel<true> : tokb::sfa_tok_bwd_kernel<false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return e;
  const int grid = a.nitems < device_sm_count() ? a.nitems : device_sm_count();
  kern<<<grid, tokb::kThreads, pl.smem, stream>>>(a, tq, tdo, tk, tv, tp, tds);
  note_launch(a.parts ? "bwd_tok_grad" : "bwd_tok", stream);
  return cudaGetLastError();
}

}  // namespace tokb

bool tok_bwd_supported(const SfaParams& p, const char** why) {
  if (device_cc() != 100) { *why = "needs an sm_100 device"; return false; }
  if (p.block_size != 1) { *why = "token-level family: block_size must be 1"; return false; }
  if (p.topk > tokb::kMaxTopk) { *why = "token-level family: topk must be <= 2048"; return false; }
  if (p.d_qk % 64 || p.d_v % 64 || p.d_qk > 256 || p.d_v > 256) {
    *why = "token-level backward: head dims must be multiples of 64, at most 256";
    return false;
  }
  if (!(p.scale > 0.f)) { *why = "needs a positive softmax scale"; return false; }
  if (!tma_compatible(p.q, p.q_sb, p.q_st, p.q_sh) || !tma_compatible(p.k, p.k_sb, p.k_st, p.k_sh) ||
      !tma_compatible(p.v, p.v_sb, p.v_st, p.v_sh) || !tma_compatible(p.dout, p.do_sb, p.do_st, p.do_sh)) {
    *why = "q/k/v/dout need 16-byte aligned base and strides";
    return false;
  }
  if ((p.dq_sh % 8) || (p.dq_st % 8) || (p.dq_sb % 8) || (reinterpret_cast<uintptr_t>(p.dq) & 15)) {
    *why = "dq needs a 16-byte aligned base and strides";
    return false;
  }
  tokb::Plan pl;
  return tokb::plan(p, &pl, why);
}

bool tok_bwd_parts_supported(const SfaParams& p, const char** why) {
  tokb::Plan pl;
  return tokb::plan(p, &pl, why, true);
}

cudaError_t launch_bwd_tok(const SfaParams& p, const float* delta, float* dk_acc, float* dv_acc,
                           cudaStream_t stream) {
  tokb::Plan pl;
  const char* why = "";
  if (!tokb::plan(p, &pl, &why)) return cudaErrorInvalidValue;
  tokb::Args& a = pl.a;
  if (a.nitems == 0) return cudaSuccess;
  a.delta = delta;
  a.dk_acc = dk_acc;
  a.dv_acc = dv_acc;
  a.status = device_status_ptr();
  // the P / dS' maps are unused in the one-pass form: any valid map will do
  CUtensorMap dummy;
  cudaError_t e = make_tmap_bf16_4d(&dummy, p.q, {64u, 1u, 1u, 1u}, {64, 64, 64}, {64u, 1u, 1u, 1u});
  if (e != cudaSuccess) return e;
  return tokb::launch(pl, p, dummy, dummy, stream);
}

cudaError_t launch_bwd_tok_parts(const SfaParams& p, float* dk_acc, float* dv_acc, const void* pws, const void* dsws,
                                 int64_t ld, int r0, int r1, cudaStream_t stream) {
  tokb::Plan pl;
  const char* why = "";
  if (!tokb::plan(p, &pl, &why, true)) return cudaErrorInvalidValue;
  tokb::Args& a = pl.a;
  a.r0 = r0;
  a.nitems = (r1 - r0) * p.h_kv * a.n_hg * a.parts;
  if (a.nitems <= 0) return cudaSuccess;
  a.dk_acc = dk_acc;
  a.dv_acc = dv_acc;
  a.status = device_status_ptr();
  // P / dS' workspace rows of this wave: [r1 - r0][h_q][ld] bf16, a box of 64 slots x HG heads
  CUtensorMap tp, tds;
  const uint64_t wr = (uint64_t)(r1 - r0);
  cudaError_t e = make_tmap_bf16_4d(&tp, pws, {(uint64_t)ld, (uint64_t)p.h_q, wr, 1u},
                                    {ld, ld * p.h_q, ld * p.h_q * (int64_t)wr}, {64u, (uint32_t)a.HG, 1u, 1u});
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16_4d(&tds, dsws, {(uint64_t)ld, (uint64_t)p.h_q, wr, 1u},
                        {ld, ld * p.h_q, ld * p.h_q * (int64_t)wr}, {64u, (uint32_t)a.HG, 1u, 1u});
  if (e != cudaSuccess) return e;
  return tokb::launch(pl, p, tp, tds, stream);
}

}  // namespace sfa
