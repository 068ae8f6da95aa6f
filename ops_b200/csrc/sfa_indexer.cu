// sfa_indexer.cu — top-k token indexer on sm_100a: the step before the sparse
// attention op, producing its token-level indices (the reference consumes
// topk_idxs, SFA.py:90, and has no indexer of its own).
//
// Scores (the lightning-indexer formula of DeepSeek-V3.2's sparse attention):
//     I[t, s] = sum_h w[t, h] * ReLU(q_idx[t, h] . k_idx[s])
// over the keys s of t's sequence (causal: s <= t + Tk - Tq).  k_idx has one
// head shared by every query head, so the products of QG = 256 / H queries x
// H heads against a tile of 128 keys are one dense MMA in the swapped
// orientation: D[key, (query, head)] = K_tile . Q_group^T (M = 128 keys,
// N = 256, K = D).  A thread of the epilogue owns one key (TMEM lane): ReLU,
// weight and the sum over heads stay inside the thread, and it writes its
// key's score of every query of the group (fp32, one coalesced row segment a
// query).  The query group stays in shared memory while the K tiles stream
// through a TMA ring; two TMEM buffers of 256 columns let the epilogue of one
// tile run under the next tile's MMAs.
//
// Selection: one CTA per query row reads the row's valid scores into shared
// memory as order-preserving integers, finds the topk-th largest by a radix
// select (11 + 11 + 10 bits, shared-memory histograms), and writes the keys
// above it plus the first of the keys equal to it (ties: lower index first)
// in ascending index order; -1 fills the row when it has fewer keys.
//
// Rows go through in waves so the score workspace stays bounded.  Warp roles
// of the score kernel (384 threads, one persistent CTA per SM): warp 0 loads
// (query group, weights, K tiles), warp 1 issues the MMAs, warps 4-11 are the
// epilogue (two per TMEM lane quadrant, each half the columns).  Every wait is
// bounded (~2 s); on expiry the kernel records (7 << 16) | site in the status
// word and returns.
#include "sfa_common.cuh"
#include "sfa_internal.h"
#include "sfa_tc_common.cuh"
#include "sfa_tc_host.h"
#include "sfa_tok_common.cuh"

#include <algorithm>

namespace sfa {
using namespace tc;
using namespace tok;

namespace idxr {

constexpr int kThreads = 384;
constexpr int kN = 256;                 // query-group columns: QG queries x H heads
constexpr int kKeys = 128;              // keys per tile (MMA M)
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;     // two 256-column buffers
constexpr int kSelThreads = 1024;
constexpr int kMaxKv = 49152;           // fp32 scores of a row in shared memory
constexpr int kMaxTopk = 4096;

struct Args {
  SfaIndexerParams p;
  float* scores;                        // [B][wave rows][ld]
  int64_t ld;
  int tw0, wrows;                       // first query row of the wave, rows a batch
  int QG, nslab, ngroups, nitems;
  int32_t* status;
};

struct Bars {
  uint64_t q_full, q_empty, w_full, w_empty;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t d_full[2], d_empty[2];
  uint32_t tmem_base;
  uint32_t pad;
};

__device__ __forceinline__ bool wt(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  if (mbar_wait(bar, parity)) return true;
  record_status(status, (7 << 16) | site);
  return false;
}

__device__ __forceinline__ bool wtw(uint64_t* bar, uint32_t parity, int32_t* status, int site) {
  return __all_sync(0xffffffffu, wt(bar, parity, status, site));
}

// Item -> (batch, first query, key tiles).  Later groups of a causal row
// range have more keys and go first.
struct Item {
  int b, t0, ntiles;
};

__device__ __forceinline__ Item item_info(const Args& a, int i) {
  const SfaIndexerParams& p = a.p;
  Item it;
  it.b = i % p.batch;
  const int gr = a.ngroups - 1 - i / p.batch;
  it.t0 = a.tw0 + gr * a.QG;
  const int tl = min(it.t0 + a.QG, a.tw0 + a.wrows) - 1;          // last query of the group
  int nk = p.kv_len;
  if (p.causal) nk = min(nk, max(0, tl + p.kv_len - p.q_len + 1));
  it.ntiles = (nk + kKeys - 1) / kKeys;
  return it;
}

__global__ void __launch_bounds__(kThreads, 1)
sfa_indexer_score_kernel(const __grid_constant__ Args args, const __grid_constant__ CUtensorMap tmq,
                         const __grid_constant__ CUtensorMap tmk) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sbase = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const SfaIndexerParams& p = args.p;
  const int NS = args.nslab;
  const int qbytes = NS * kN * 128, kbytes = NS * kKeys * 128;
  uint8_t* sq = sbase;                                    // query group: NS slabs of 256 rows x 64 dims
  uint8_t* sk = sbase + qbytes;                           // K ring
  float* sw = reinterpret_cast<float*>(sk + kStages * kbytes);   // weights of the group [QG][H]
  Bars& B = *reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(sw) + kN * 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int32_t* st = args.status;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    mbar_init(&B.w_full, 1);
    mbar_init(&B.w_empty, 8);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&B.k_full[i], 1);
      mbar_init(&B.k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.d_full[i], 1);
      mbar_init(&B.d_empty[i], 8);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&B.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_base;

  if (warp == 0) {
    // ============================================================ loads
    int use = 0, item_i = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < args.nitems && ok; i += gridDim.x) {
      const Item it = item_info(args, i);
      if (it.ntiles == 0) continue;
      // weights of the group (the epilogue of the previous item has read its own)
      ok = wtw(&B.w_empty, (item_i & 1) ^ 1, st, 1);
      if (!ok) break;
      for (int j = lane; j < kN; j += 32) {
        const int q = j / p.heads, h = j - q * p.heads, t = it.t0 + q;
        sw[j] = t < args.tw0 + args.wrows ? __ldg(p.weights + it.b * p.w_sb + (int64_t)t * p.w_st + h) : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&B.w_full);
        ok = wt(&B.q_empty, (item_i & 1) ^ 1, st, 2);
        if (ok) {
          mbar_arrive_expect_tx(&B.q_full, (uint32_t)qbytes);
          for (int s = 0; s < NS; ++s) tma_load_4d(sq + s * kN * 128, &tmq, &B.q_full, s * 64, 0, it.t0, it.b);
        }
        for (int tile = 0; tile < it.ntiles && ok; ++tile, ++use) {
          const int sg = use % kStages;
          if (!(ok = wt(&B.k_empty[sg], ((use / kStages) & 1) ^ 1, st, 3))) break;
          mbar_arrive_expect_tx(&B.k_full[sg], (uint32_t)kbytes);
          for (int s = 0; s < NS; ++s)
            tma_load_4d(sk + sg * kbytes + s * kKeys * 128, &tmk, &B.k_full[sg], s * 64, tile * kKeys, it.b, 0);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      use = __shfl_sync(0xffffffffu, use, 0);
      ++item_i;
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id = idesc_bf16(kKeys, kN, false, false);
      int use = 0, item_i = 0, tcount = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < args.nitems && ok; i += gridDim.x) {
        const Item it = item_info(args, i);
        if (it.ntiles == 0) continue;
        if (!(ok = wt(&B.q_full, item_i & 1, st, 4))) break;
        for (int tile = 0; tile < it.ntiles && ok; ++tile, ++use, ++tcount) {
          const int sg = use % kStages, buf = tcount & 1;
          if (!(ok = wt(&B.d_empty[buf], ((tcount >> 1) & 1) ^ 1, st, 5))) break;
          if (!(ok = wt(&B.k_full[sg], (use / kStages) & 1, st, 6))) break;
          tc_fence_after();
          for (int s = 0; s < NS; ++s) {
            const uint64_t kd = smem_desc(smem_u32(sk + sg * kbytes + s * kKeys * 128), 16, 1024, kSw128);
            const uint64_t qd = smem_desc(smem_u32(sq + s * kN * 128), 16, 1024, kSw128);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16_ss(tmem + buf * kN, kd + (uint64_t)((k * 32) >> 4), qd + (uint64_t)((k * 32) >> 4), id,
                          (s | k) != 0);
          }
          mma_commit(&B.k_empty[sg]);
          mma_commit(&B.d_full[buf]);
        }
        if (ok) mma_commit(&B.q_empty);
        ++item_i;
      }
    }
  } else if (warp >= 4) {
    // ============================================================ epilogue
    const int sub = warp & 3, half = (warp - 4) >> 2;
    const uint32_t tl = tmem + ((uint32_t)(sub * 32) << 16);
    const int H = p.heads, QH = args.QG / 2;            // queries of this warp's column half
    int tcount = 0, item_i = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < args.nitems && ok; i += gridDim.x) {
      const Item it = item_info(args, i);
      if (it.ntiles == 0) continue;
      if (!(ok = wtw(&B.w_full, item_i & 1, st, 8))) break;
      for (int tile = 0; tile < it.ntiles && ok; ++tile, ++tcount) {
        const int buf = tcount & 1;
        if (!(ok = wtw(&B.d_full[buf], (tcount >> 1) & 1, st, 7))) break;
        tc_fence_after();
        float acc[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = 0.f;
        // this half's 128 columns: queries half*QH .. half*QH + QH - 1, all heads.
        // 32 columns hold one query's heads (H >= 32) or two queries' (H = 16)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tl + buf * kN + half * 128 + c * 32, v);
          tmem_ld_wait();
          const float4* w4 = reinterpret_cast<const float4*>(sw + half * 128 + c * 32);
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 w = w4[j];
            const float x = fmaxf(v[4 * j], 0.f) * w.x + fmaxf(v[4 * j + 1], 0.f) * w.y +
                            fmaxf(v[4 * j + 2], 0.f) * w.z + fmaxf(v[4 * j + 3], 0.f) * w.w;
            if (H == 16 && j >= 4) s1 += x; else s0 += x;
          }
          const int ql = (half * 128 + c * 32) / H - half * QH;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (q == ql) acc[q] += s0;
            if (q == ql + 1) acc[q] += s1;
          }
        }
        tc_fence_before();
        warp_arrive(&B.d_empty[buf]);
        const int s = tile * kKeys + sub * 32 + lane;
        for (int q = 0; q < QH && q < 8; ++q) {
          const int t = it.t0 + half * QH + q;
          if (t >= args.tw0 + args.wrows) break;
          const bool valid = s < p.kv_len && (!p.causal || s <= t + p.kv_len - p.q_len);
          args.scores[((int64_t)it.b * args.wrows + (t - args.tw0)) * args.ld + s] = valid ? acc[q] : -INFINITY;
        }
      }
      if (!ok) break;
      // the weights of this item are no longer needed
      warp_arrive(&B.w_empty);
      ++item_i;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ selection

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Exclusive scan of one value per thread over the block (1024 threads);
// returns the prefix and writes the block total to *total.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;                                // inclusive over warps
  }
  __syncthreads();
  const uint32_t before = (warp ? warp_sums[warp - 1] : 0u) + x - v;
  *total = warp_sums[31];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kSelThreads)
sfa_indexer_select_kernel(const __grid_constant__ Args args) {
  extern __shared__ uint32_t su[];                      // row keys [ld], then the histogram
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t pick[2];
  const SfaIndexerParams& p = args.p;
  const int r = blockIdx.x, b = blockIdx.y;
  const int t = args.tw0 + r;
  if (r >= args.wrows || t >= p.q_len) return;
  int n = p.kv_len;
  if (p.causal) n = min(n, max(0, t + p.kv_len - p.q_len + 1));
  const int K = p.topk;
  int32_t* out = p.out + b * p.o_sb + (int64_t)t * p.o_st;
  const int tid = threadIdx.x;
  if (n <= K) {
    for (int i = tid; i < K; i += kSelThreads) out[i] = i < n ? i : -1;
    return;
  }
  const float* row = args.scores + ((int64_t)b * args.wrows + r) * args.ld;
  uint32_t* hist = su + args.ld;
  for (int i = tid; i < n; i += kSelThreads) su[i] = order_key(row[i]);
  // radix select of the K-th largest key: 11, 11 and 10 bits from the top
  uint32_t prefix = 0, pmask = 0;
  uint32_t krem = (uint32_t)K;
  const int shifts[3] = {21, 10, 0}, widths[3] = {11, 11, 10};
  for (int ps = 0; ps < 3; ++ps) {
    const int sh = shifts[ps], nb = 1 << widths[ps];
    for (int i = tid; i < nb; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kSelThreads) {
      const uint32_t u = su[i];
      if ((u & pmask) == prefix) atomicAdd(&hist[(u >> sh) & (uint32_t)(nb - 1)], 1u);
    }
    __syncthreads();
    // bins from the top: thread j sums bins nb-1-2j and nb-2-2j
    uint32_t c0 = 0, c1 = 0;
    const int b0 = nb - 1 - 2 * tid, b1 = b0 - 1;
    if (b0 >= 0) c0 = hist[b0];
    if (b1 >= 0) c1 = hist[b1];
    uint32_t tot;
    const uint32_t above = block_excl_scan(c0 + c1, warp_sums, &tot);
    // the bin where the count from the top first reaches krem
    if (b0 >= 0 && above < krem && above + c0 >= krem) { pick[0] = (uint32_t)b0; pick[1] = above; }
    else if (b1 >= 0 && above + c0 < krem && above + c0 + c1 >= krem) { pick[0] = (uint32_t)b1; pick[1] = above + c0; }
    __syncthreads();
    prefix |= pick[0] << sh;
    pmask |= (uint32_t)(nb - 1) << sh;
    krem -= pick[1];
    __syncthreads();
  }
  // keys above the threshold, then the first krem keys equal to it, in index order
  const uint32_t tau = prefix;
  const int per = (n + kSelThreads - 1) / kSelThreads;
  const int i0 = min(n, tid * per), i1 = min(n, i0 + per);
  uint32_t gt = 0, eq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t u = su[i];
    gt += u > tau;
    eq += u == tau;
  }
  uint32_t tot;
  const uint32_t pre = block_excl_scan(gt | (eq << 16), warp_sums, &tot);
  uint32_t g = pre & 0xffffu, e = pre >> 16;
  for (int i = i0; i < i1; ++i) {
    const uint32_t u = su[i];
    if (u > tau) {
      out[g + min(e, krem)] = i;
      ++g;
    } else if (u == tau) {
      if (e < krem) out[g + e] = i;
      ++e;
    }
  }
}

}  // namespace idxr

// ------------------------------------------------------------------ host side

static int idx_fail(int code, const std::string& msg) { return report_error(code, msg); }

static int indexer_validate(const SfaIndexerParams* p) {
  if (!p) return idx_fail(SFA_ERR_INVALID_ARGUMENT, "params is NULL");
  if (!p->q_idx || !p->k_idx || !p->weights || !p->out)
    return idx_fail(SFA_ERR_INVALID_ARGUMENT, "q_idx, k_idx, weights and out must be non-NULL");
  if (p->batch < 0 || p->q_len < 0 || p->kv_len < 0)
    return idx_fail(SFA_ERR_INVALID_ARGUMENT, "batch, q_len and kv_len must be >= 0");
  if (p->heads != 16 && p->heads != 32 && p->heads != 64 && p->heads != 128)
    return idx_fail(SFA_ERR_UNSUPPORTED, "indexer heads must be 16, 32, 64 or 128");
  if (p->dim != 64 && p->dim != 128) return idx_fail(SFA_ERR_UNSUPPORTED, "indexer head dim must be 64 or 128");
  if (p->topk <= 0 || p->topk > idxr::kMaxTopk)
    return idx_fail(SFA_ERR_INVALID_ARGUMENT, "topk must be in [1, 4096]");
  if (p->kv_len > idxr::kMaxKv) return idx_fail(SFA_ERR_UNSUPPORTED, "indexer kv_len must be <= 49152");
  if (!tma_compatible(p->q_idx, p->q_sb, p->q_st, p->q_sh) || !tma_compatible(p->k_idx, p->k_sb, p->k_st, 8))
    return idx_fail(SFA_ERR_INVALID_ARGUMENT, "q_idx / k_idx need 16-byte aligned base and strides");
  if (p->q_sh != p->dim)
    return idx_fail(SFA_ERR_INVALID_ARGUMENT, "q_idx heads must be contiguous rows (head stride == dim)");
  return SFA_OK;
}

// Query rows a wave (a multiple of the query group): fp32 scores of the wave
// within 1 GiB.
static int indexer_wave_rows(const SfaIndexerParams& p, int64_t ld) {
  const int QG = idxr::kN / p.heads;
  const int64_t per_row = (int64_t)(p.batch > 0 ? p.batch : 1) * ld * 4;
  int64_t w = ((int64_t)1 << 30) / per_row;
  w = w / QG * QG;
  if (w < QG) w = QG;
  const int64_t qr = (p.q_len + QG - 1) / QG * QG;
  return (int)(w < qr ? w : qr);
}

static int64_t indexer_ld(const SfaIndexerParams& p) {
  return (int64_t)((p.kv_len + idxr::kKeys - 1) / idxr::kKeys) * idxr::kKeys;
}

}  // namespace sfa

using namespace sfa;

extern "C" {

size_t sfa_indexer_workspace_bytes(const SfaIndexerParams* p) {
  if (indexer_validate(p)) return 0;
  const int64_t ld = indexer_ld(*p);
  return (size_t)((int64_t)p->batch * indexer_wave_rows(*p, ld) * ld * 4);
}

int sfa_indexer_topk(const SfaIndexerParams* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = indexer_validate(p);
  if (rc) return rc;
  if (device_cc() != 100) return idx_fail(SFA_ERR_UNSUPPORTED, "the indexer needs an sm_100 device");
  if (p->batch == 0 || p->q_len == 0) return SFA_OK;
  const int64_t ld = indexer_ld(*p);
  const int wave = indexer_wave_rows(*p, ld);
  const size_t need = (size_t)((int64_t)p->batch * wave * ld * 4);
  if (ld > 0 && (workspace == nullptr || workspace_bytes < need))
    return idx_fail(SFA_ERR_WORKSPACE, "indexer workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  idxr::Args a{};
  a.p = *p;
  a.scores = reinterpret_cast<float*>(workspace);
  a.ld = ld;
  a.QG = idxr::kN / p->heads;
  a.nslab = p->dim / 64;
  a.status = device_status_ptr();
  CUtensorMap tq, tk;
  cudaError_t e = make_tmap_bf16_4d(&tq, p->q_idx, {(uint64_t)p->dim, (uint64_t)p->heads, (uint64_t)p->q_len,
                                                     (uint64_t)p->batch},
                                    {p->q_sh, p->q_st, p->q_sb}, {64u, (uint32_t)p->heads, (uint32_t)a.QG, 1u});
  if (e == cudaSuccess && p->kv_len > 0)
    e = make_tmap_bf16_4d(&tk, p->k_idx, {(uint64_t)p->dim, (uint64_t)p->kv_len, (uint64_t)p->batch, 1u},
                          {p->k_st, p->k_sb, 0}, {64u, (uint32_t)idxr::kKeys, 1u, 1u});
  if (e != cudaSuccess) return report_error(SFA_ERR_CUDA, "indexer tensor maps");
  const size_t smem = 1024 + (size_t)a.nslab * idxr::kN * 128 + (size_t)idxr::kStages * a.nslab * idxr::kKeys * 128 +
                      idxr::kN * 4 + sizeof(idxr::Bars);
  const size_t sel_smem = (size_t)ld * 4 + 2048 * 4;
  if (p->kv_len > 0) {
    e = cudaFuncSetAttribute(idxr::sfa_indexer_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(idxr::sfa_indexer_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sel_smem);
    if (e != cudaSuccess) return report_error(SFA_ERR_CUDA, std::string("indexer attributes: ") + cudaGetErrorString(e));
  }
  for (int tw0 = 0; tw0 < p->q_len; tw0 += wave) {
    a.tw0 = tw0;
    a.wrows = std::min(wave, p->q_len - tw0);
    a.ngroups = (a.wrows + a.QG - 1) / a.QG;
    a.nitems = a.ngroups * p->batch;
    if (p->kv_len > 0) {
      const int grid = std::min(a.nitems, device_sm_count());
      idxr::sfa_indexer_score_kernel<<<grid, idxr::kThreads, smem, st>>>(a, tq, tk);
      note_launch("indexer_score", st);
    }
    idxr::sfa_indexer_select_kernel<<<dim3(a.wrows, p->batch), idxr::kSelThreads, sel_smem, st>>>(a);
    note_launch("indexer_select", st);
    if ((e = cudaGetLastError()) != cudaSuccess)
      return report_error(SFA_ERR_CUDA, std::string("indexer launch: ") + cudaGetErrorString(e));
  }
  return SFA_OK;
}

}  // extern "C"
