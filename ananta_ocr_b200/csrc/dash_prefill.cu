// dash_prefill.cu -- DASH prefill gather attention on sm_100a tensor cores.
//
// Work unit: one CTA per (tile of 128 query rows, kv head).  A tile row is a
// (query token, query head of this kv head) pair; with G query heads per kv
// head a tile covers 128/G consecutive tokens.  The tile walks, in ascending
// order, every 64-key tile of the blocks that any of its rows routed to (the
// per-tile union built by plan_kernel) plus the blocks of its local windows.
// Per key tile:
//   TMA (warp 8)      K and V tiles -> shared memory (128-byte swizzle), 4 stages
//   MMA (warps 9,10)  one issuer per query tile:
//                     S = Q K^T   (tcgen05.mma M=128 N=64, Q and K from shared
//                                  memory, fp32 in TMEM, 2 buffers)
//                     O += P V    (tcgen05.mma M=128 N=128, P from TMEM, V from
//                                  shared memory, fp32 in TMEM)
//   softmax (w0-7)    one thread per row of one of the two query tiles: S from
//                     TMEM, per-row mask + bias (local window: no bias; routed
//                     block: + bias; else -inf), online softmax in the exp2
//                     domain with lazy rescaling of O, P (bf16/fp16) written
//                     back over the S buffer it came from.
// Keeping P in TMEM removes the P round trip through shared memory, which
// (with the Q operand re-read by every QK MMA) bounds this kernel.  The
// softmax warpgroups take 200 registers each and the TMA/MMA warpgroup 104
// (setmaxnreg), so a thread holds its whole 64-column S row.
// Rows that did not route a block of the union simply get P = 0 there.
//
// Semantics: sparse_gather_e2e_triton.py:34-115 (_e2e_attn_fwd_kernel),
// sparse_gather_triton.py:29-104 (_gather_attn_fwd_kernel, seg/packing),
// WHL attend_triton.py:88-292 (_dash_sparse_fwd_kernel, paged).
#include <cudaTypedefs.h>
#include <algorithm>
#include <climits>
#include "dash_common.cuh"
#include "dash_internal.h"
#include "dash_prefill_plan.cuh"

namespace dash {

constexpr int BM = 128;          // tile rows (M of both MMAs)
constexpr int BN = 64;           // keys per key tile (N of QK, K of PV)
constexpr int HD = 128;          // head dim
constexpr int NSTAGE = 4;
// two query tiles (A, B) per CTA share the K/V stream
constexpr int OFF_Q = 0;                          // 2 tiles x 2 x [128 x 128 B]
constexpr int OFF_K = 65536;                      // NSTAGE x 2 x [64 x 128 B]
constexpr int OFF_V = OFF_K + NSTAGE * 16384;     // NSTAGE x 2 x [64 x 128 B]
constexpr int OFF_MASK = OFF_V + NSTAGE * 16384;  // block mask words
constexpr int MAX_MASK_WORDS = 256;               // <= 8192 blocks
constexpr int OFF_BAR = OFF_MASK + MAX_MASK_WORDS * 4;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// warps 0-7 softmax (two groups), 8 TMA, 9-10 MMA issuers, 11 idle
constexpr int NTHREADS = 384;
// Register split: launched at kLaunchRegs per thread (3 warps per SM
// sub-partition), then 2 x 128 softmax threads grow to kSoftmaxRegs while the
// 128 TMA/MMA threads shrink to kOtherRegs.  The host refuses to launch a
// build whose register count does not cover the split (the growth would wait).
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 200;
constexpr int kOtherRegs = 104;
static_assert(2 * 128 * kSoftmaxRegs + 128 * kOtherRegs <= NTHREADS * kLaunchRegs, "register split");
static_assert(2 * kSoftmaxRegs + kOtherRegs <= 3 * kLaunchRegs, "register split per sub-partition");
constexpr uint32_t TMEM_COLS = 512;               // per query tile: S0 | S1 | O
// O is rescaled only when a row's logit exceeds its running max by more than
// 2^kGrowLog2 (then p < 2^32: no bf16/fp32 overflow for any sequence length)
constexpr float kGrowLog2 = 32.0f;
constexpr float kGrowP = 4294967296.0f;

// ---------------------------------------------------------------------------
// plan_kernel: one CTA per (query tile, index head), one warp per token row
// (strided).  Canonicalises each row's routed list (drops -1, ids without a
// remote key for the row, later duplicates; ascending order), records the
// row's largest kept bias, and builds the tile's block union in shared memory;
// the union words are written once, so no global atomics and no pre-zeroing.
// Slot j of a row lives in lane j % 32, register j / 32 (PER registers);
// duplicate and rank tests run over warp shuffles.  The next row's slots are
// loaded before the current row is processed.
// With 32-token blocks (PAIR) a 64-key tile holds blocks 2p and 2p+1, and the
// list is written per tile instead of per block: entry = (p << 2) | routed
// bits (bit h: block 2p+h routed), biases [2j + h], ascending in p, so the
// attention kernel's cursor still moves at most one entry per key tile.
// ---------------------------------------------------------------------------
constexpr int kPlanWarps = 16;

template <int PER, bool PAIR>
__global__ void __launch_bounds__(kPlanWarps * 32) plan_kernel(DashPrefillArgs a, PrefillPlan p,
                                                               int32_t* cidx, float* cbias,
                                                               uint32_t* tmask, float* rowmax) {
  __shared__ uint32_t s_mask[MAX_MASK_WORDS];
  extern __shared__ uint32_t s_flags[];        // gathered mode: [nblk_cap][wpt]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, ih = blockIdx.y;
  const int s = tile / p.tiles_per_seq, t = tile - s * p.tiles_per_seq;
  for (int w = threadIdx.x; w < p.nwords; w += kPlanWarps * 32) s_mask[w] = 0u;
  if (p.flags)
    for (int w = threadIdx.x; w < p.nblk_cap * p.wpt; w += kPlanWarps * 32) s_flags[w] = 0u;
  __syncthreads();
  const int qlen = q_len_of(a.seqs, s);
  const int i_end = min(qlen, (t + 1) * p.TT);
  const int kvl = kv_len_of(a.seqs, s);
  const int pos0 = pos0_of(a.seqs, s);
  const int nblk_seq = (kvl + a.block_size - 1) / a.block_size;
  const int K = a.routes.K;
  const int64_t rb = row_base(a.seqs, s);
  auto load_row = [&](int i, int (&b)[PER], float (&bias)[PER]) {
    const int64_t r = rb + i;
    const int32_t* il = a.routes.idx + r * a.routes.row_stride + (int64_t)ih * a.routes.ihead_stride;
    const float* bl = a.routes.bias ? a.routes.bias + r * a.routes.row_stride +
                                          (int64_t)ih * a.routes.ihead_stride
                                    : nullptr;
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int j = lane + 32 * q;
      b[q] = j < K ? il[j] : -1;
      bias[q] = (j < K && bl) ? bl[j] : 0.0f;
    }
  };
  int b_nx[PER];
  float bias_nx[PER];
  int i = t * p.TT + warp;
  if (i < i_end) load_row(i, b_nx, bias_nx);
  for (; i < i_end; i += kPlanWarps) {
    int b[PER];
    float bias[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) { b[q] = b_nx[q]; bias[q] = bias_nx[q]; }
    if (i + kPlanWarps < i_end) load_row(i + kPlanWarps, b_nx, bias_nx);
    const int64_t r = rb + i;
    const int lstart = pos0 + i - a.local_window + 1;
    // keep ids with a remote key for this row; drop later duplicates (the
    // validity test depends only on the id, so a duplicate of a dropped id is
    // dropped by the same test).  The shuffle loops below visit the K live
    // slots only: a slot j >= K holds -1, which is never kept and never
    // matches or ranks below a kept id.
    bool keep[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int bb = b[q];
      keep[q] = bb >= 0 && bb < nblk_seq && bb < p.nblk_cap && (int64_t)bb * a.block_size < lstart;
      if (bb >= nblk_seq) record_error(a.device_error, DASH_DEV_BAD_BLOCK, 30, bb);
    }
#pragma unroll
    for (int qs = 0; qs < PER; ++qs) {
      for (int src = 0; src < min(32, K - 32 * qs); ++src) {
        const int bu = __shfl_sync(0xffffffffu, b[qs], src);
        const int u = src + 32 * qs;
#pragma unroll
        for (int q = 0; q < PER; ++q)
          if (u < lane + 32 * q && bu == b[q]) keep[q] = false;
      }
    }
    // rank of each kept id among the kept ids (distinct): ascending position
    int rank[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) rank[q] = 0;
#pragma unroll
    for (int qs = 0; qs < PER; ++qs) {
      const int key = keep[qs] ? b[qs] : INT_MAX;
      for (int src = 0; src < min(32, K - 32 * qs); ++src) {
        const int ku = __shfl_sync(0xffffffffu, key, src);
#pragma unroll
        for (int q = 0; q < PER; ++q) rank[q] += ku < b[q] ? 1 : 0;
      }
    }
    int32_t* oi = cidx + ((int64_t)ih * p.n_rows + r) * K;
    float* ob = cbias + ((int64_t)ih * p.n_rows + r) * K * (PAIR ? 2 : 1);
    int nk = 0;
    float bmax = -INFINITY;
    if constexpr (!PAIR) {
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        if (keep[q]) {
          oi[rank[q]] = b[q];
          ob[rank[q]] = bias[q];
        }
        nk += __popc(__ballot_sync(0xffffffffu, keep[q]));
      }
      for (int j = nk + lane; j < K; j += 32) { oi[j] = -1; ob[j] = 0.0f; }
    } else {
      // partner = the other block of the same 64-key tile (ids are distinct
      // after the duplicate test, so at most one kept slot matches)
      bool pk[PER];
      float pbias[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) { pk[q] = false; pbias[q] = 0.0f; }
#pragma unroll
      for (int qs = 0; qs < PER; ++qs) {
        const int key = keep[qs] ? b[qs] : -2;
        for (int src = 0; src < min(32, K - 32 * qs); ++src) {
          const int ku = __shfl_sync(0xffffffffu, key, src);
          const float bu = __shfl_sync(0xffffffffu, bias[qs], src);
#pragma unroll
          for (int q = 0; q < PER; ++q)
            if (keep[q] && ku == (b[q] ^ 1)) { pk[q] = true; pbias[q] = bu; }
        }
      }
      // the lower kept block of a tile leads its entry; entries ranked by tile
      bool lead[PER];
      int prank[PER];
#pragma unroll
      for (int q = 0; q < PER; ++q) { lead[q] = keep[q] && (!(b[q] & 1) || !pk[q]); prank[q] = 0; }
#pragma unroll
      for (int qs = 0; qs < PER; ++qs) {
        const int key = lead[qs] ? (b[qs] >> 1) : INT_MAX;
        for (int src = 0; src < min(32, K - 32 * qs); ++src) {
          const int ku = __shfl_sync(0xffffffffu, key, src);
#pragma unroll
          for (int q = 0; q < PER; ++q) prank[q] += ku < (b[q] >> 1) ? 1 : 0;
        }
      }
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        if (lead[q]) {
          const int hb = b[q] & 1;
          oi[prank[q]] = ((b[q] >> 1) << 2) | (1 << hb) | (pk[q] ? (1 << (hb ^ 1)) : 0);
          ob[2 * prank[q] + hb] = bias[q];
          ob[2 * prank[q] + (hb ^ 1)] = pk[q] ? pbias[q] : 0.0f;
        }
        nk += __popc(__ballot_sync(0xffffffffu, lead[q]));
      }
      for (int j = nk + lane; j < K; j += 32) { oi[j] = -1; ob[2 * j] = 0.0f; ob[2 * j + 1] = 0.0f; }
    }
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      if (keep[q]) {
        atomicOr(s_mask + (b[q] >> 5), 1u << (b[q] & 31));
        if (p.flags) {
          const int li = i - t * p.TT;                  // token within this tile
          atomicOr(s_flags + b[q] * p.wpt + (li >> 5), 1u << (li & 31));
        }
        if (a.routes.bias) bmax = fmaxf(bmax, bias[q]);
      }
    }
    for (int o = 16; o > 0; o >>= 1) bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
    if (lane == 0) rowmax[(int64_t)ih * p.n_rows + r] = bmax;
  }
  __syncthreads();
  uint32_t* tm = tmask + ((int64_t)ih * a.seqs.n_seq * p.tiles_per_seq + tile) * p.nwords;
  for (int w = threadIdx.x; w < p.nwords; w += kPlanWarps * 32) tm[w] = s_mask[w];
  if (p.flags) {
    // this tile owns words [t*wpt, (t+1)*wpt) of every block's row mask
    uint32_t* fl = p.flags + ((int64_t)ih * a.seqs.n_seq + s) * p.nblk_cap * p.wps + (int64_t)t * p.wpt;
    for (int e = threadIdx.x; e < p.nblk_cap * p.wpt; e += kPlanWarps * 32) {
      const int bb = e / p.wpt, w = e - bb * p.wpt;
      fl[(int64_t)bb * p.wps + w] = s_flags[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Key-tile iterator over the shared block mask (ascending).  After a call that
// returned kt0 >= 0, b is the block of the tile and half its 64-key part, so
// callers need no division by the block size.  With 32-token blocks (PAIR) a
// tile is kept when either of its blocks 2p, 2p+1 is set and b = 2p.
// ---------------------------------------------------------------------------
struct TileIter {
  int w, b, half;
  uint32_t bits;
};
template <bool PAIR>
__device__ __forceinline__ int next_tile(TileIter& t, const uint32_t* mask, int nwords, int bs,
                                         int64_t pmax, int kvl) {
  if constexpr (PAIR) {
    while (true) {
      while (t.bits == 0) {
        if (++t.w >= nwords) return -1;
        const uint32_t m = mask[t.w];
        t.bits = (m | (m >> 1)) & 0x55555555u;
      }
      const int bit = __ffs(t.bits) - 1;
      t.bits &= t.bits - 1;
      t.b = t.w * 32 + bit;
      const int64_t kt0 = (int64_t)t.b * 32;
      if (kt0 > pmax || kt0 >= kvl) continue;
      return (int)kt0;
    }
  }
  const int halves = bs / BN;
  while (true) {
    if (t.half + 1 < halves && t.b >= 0) {
      t.half++;
    } else {
      while (t.bits == 0) {
        if (++t.w >= nwords) return -1;
        t.bits = mask[t.w];
      }
      int bit = __ffs(t.bits) - 1;
      t.bits &= t.bits - 1;
      t.b = t.w * 32 + bit;
      t.half = 0;
    }
    int64_t kt0 = (int64_t)t.b * bs + t.half * BN;
    if (kt0 > pmax || kt0 >= kvl) continue;
    return (int)kt0;
  }
}

template <typename T, bool PAGED, bool PAIR>
__global__ void __launch_bounds__(NTHREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const DashPrefillArgs a, const PrefillPlan p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* smask = reinterpret_cast<uint32_t*>(sm + OFF_MASK);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* kv_full = bars + 0;            // [NSTAGE]
  uint64_t* kv_empty = bars + NSTAGE;      // [NSTAGE]
  // per softmax group g (7 barriers each from bars + 2*NSTAGE + 7g):
  //   s_full[2], p_full[2], pv_done[2], q_full
  uint64_t* mma_done = bars + 2 * NSTAGE + 14;   // [2], one per MMA warp
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * NSTAGE + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * NSTAGE + 17);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_seq = a.seqs.n_seq;
  // two consecutive query tiles per CTA; heaviest (last) pairs of the
  // chunk first
  const int jj = blockIdx.x / p.sn;
  const int s = p.s0 + (blockIdx.x - jj * p.sn);
  const int pj = p.pj0 + p.npj - 1 - jj;
  const int hk = p.hk0 + blockIdx.y;
  const int qlen = q_len_of(a.seqs, s);
  const int i0A = 2 * pj * p.TT;
  if (i0A >= qlen) return;
  const bool hasB = i0A + p.TT < qlen;
  const int ngroups = hasB ? 2 : 1;
  const int kvl = kv_len_of(a.seqs, s);
  const int pos0 = pos0_of(a.seqs, s);
  const int ntok_all = min(2 * p.TT, qlen - i0A);
  const int64_t pmin = (int64_t)pos0 + i0A, pmax = pmin + ntok_all - 1;
  const int G = p.G;
  const int H = a.qo.n_heads;
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const int ih = (hk * G) / (H / nih);
  const int bs = a.block_size;

  // ---- setup: barriers, TMEM, block mask ----
  if (tid == 0) {
    // a K/V stage is free once every group's PV of it completed
    for (int k = 0; k < NSTAGE; ++k) { mbar_init(kv_full + k, 1); mbar_init(kv_empty + k, ngroups); }
    for (int g = 0; g < 2; ++g) {
      uint64_t* gb = bars + 2 * NSTAGE + 7 * g;
      for (int k = 0; k < 2; ++k) {
        mbar_init(gb + 0 + k, 1);      // s_full   (MMA commit)
        mbar_init(gb + 2 + k, 4);      // p_full   (one arrive per softmax warp)
        mbar_init(gb + 4 + k, 1);      // pv_done  (MMA commit)
      }
      mbar_init(gb + 6, 4);            // q_full
    }
    mbar_init(mma_done, 1);
    mbar_init(mma_done + 1, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 9) { tmem_alloc(tmem_holder, TMEM_COLS); tmem_relinquish(); }
  {
    const int64_t tbase = (int64_t)ih * n_seq * p.tiles_per_seq + (int64_t)s * p.tiles_per_seq + 2 * pj;
    const uint32_t* umA = p.tmask + tbase * p.nwords;
    const uint32_t* umB = hasB ? umA + p.nwords : nullptr;
    const int64_t lb0 = max((int64_t)0, (pmin - a.local_window + 1) / bs);
    const int64_t lb1 = pmax / bs;
    for (int w = tid; w < p.nwords; w += NTHREADS) {
      // gathered mode: the local window only (the routed keys are partials)
      uint32_t m = p.flags ? 0u : (umA[w] | (umB ? umB[w] : 0u));
      int64_t b0 = (int64_t)w * 32;
      for (int k = 0; k < 32; ++k) {
        int64_t b = b0 + k;
        if (b >= lb0 && b <= lb1) m |= 1u << k;
      }
      smask[w] = m;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  DeviceError* derr = a.device_error;
  // register split (inside each role's branch so that the compiler budgets
  // each role's code with its own count): softmax warpgroups grow, the
  // TMA/MMA warpgroup shrinks

  if (warp >= 8) {
    regs_shrink<kOtherRegs>();
    if (warp == 8) {
      // =================== TMA producer ===================
      if (lane == 0) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        TileIter itr{-1, -1, 0, 0u};
        int it = 0;
        while (true) {
          int kt0 = next_tile<PAIR>(itr, smask, p.nwords, bs, pmax, kvl);
          if (kt0 < 0) break;
          const int st = it % NSTAGE;
          if (it >= NSTAGE && !mbar_wait(kv_empty + st, ((it / NSTAGE) - 1) & 1, abort_flag, derr, 40)) break;
          uint8_t* dK = sm + OFF_K + st * 16384;
          uint8_t* dV = sm + OFF_V + st * 16384;
          if constexpr (PAGED && PAIR) {
            // two 32-token pages per key tile (32-row boxes at rows 0 and 32 of
            // each swizzled half; 4096 B keeps the 1024 B swizzle atom); the
            // second page exists only when the tile reaches past the first
            const int64_t brow = (int64_t)s * a.kv.bt_stride + itr.b;
            const int page0 = a.kv.block_table[brow];
            const bool two = kt0 + 32 < kvl;
            const int page1 = two ? a.kv.block_table[brow + 1] : 0;
            const bool ok0 = page0 >= 0 && (int64_t)page0 < a.kv.num_pages;
            const bool ok1 = two && page1 >= 0 && (int64_t)page1 < a.kv.num_pages;
            if (!ok0) record_error(derr, DASH_DEV_BAD_PAGE, 43, page0);
            if (two && !ok1) record_error(derr, DASH_DEV_BAD_PAGE, 44, page1);
            const uint32_t bytes = (ok0 ? 16384u : 0u) + (ok1 ? 16384u : 0u);
            if (bytes) {
              mbar_arrive_expect_tx(kv_full + st, bytes);
#pragma unroll
              for (int dh = 0; dh < 2; ++dh) {
                if (ok0) {
                  tma_load_4d(dK + dh * 8192, &tmK, kv_full + st, dh * 64, 0, hk, page0);
                  tma_load_4d(dV + dh * 8192, &tmV, kv_full + st, dh * 64, 0, hk, page0);
                }
                if (ok1) {
                  tma_load_4d(dK + dh * 8192 + 4096, &tmK, kv_full + st, dh * 64, 0, hk, page1);
                  tma_load_4d(dV + dh * 8192 + 4096, &tmV, kv_full + st, dh * 64, 0, hk, page1);
                }
              }
            } else {
              mbar_arrive(kv_full + st);
            }
            ++it;
            continue;
          }
          int c1, c3;
          bool ok = true;
          if (PAGED) {
            int64_t page = a.kv.block_table[(int64_t)s * a.kv.bt_stride + itr.b];
            if (page < 0 || page >= a.kv.num_pages) {
              record_error(derr, DASH_DEV_BAD_PAGE, 41, page);
              ok = false;
            }
            c1 = itr.half * BN;
            c3 = (int)page;
          } else {
            c1 = kt0;
            c3 = s;
          }
          if (ok) {
            mbar_arrive_expect_tx(kv_full + st, 4 * 8192);
            tma_load_4d(dK, &tmK, kv_full + st, 0, c1, hk, c3);
            tma_load_4d(dK + 8192, &tmK, kv_full + st, 64, c1, hk, c3);
            tma_load_4d(dV, &tmV, kv_full + st, 0, c1, hk, c3);
            tma_load_4d(dV + 8192, &tmV, kv_full + st, 64, c1, hk, c3);
          } else {
            mbar_arrive(kv_full + st);
          }
          ++it;
        }
        // drain: never leave the CTA with bulk copies in flight
        for (int k = max(0, it - NSTAGE); k < it; ++k) {
          volatile int no_abort = 0;
          mbar_wait(kv_full + (k % NSTAGE), (k / NSTAGE) & 1, &no_abort, nullptr, 42);
        }
      }
    } else if (warp == 9 || warp == 10) {
      // ============ MMA issuers: warp 9 for group 0, warp 10 for group 1 ============
      // Each group has its own issuer so neither waits on the other's softmax.
      const int g = warp - 9;
      if (lane == 0 && g < ngroups) {
        constexpr uint32_t fmt = DType<T>::fmt;
        constexpr uint32_t idesc_qk = make_idesc(fmt, 0, 0, BM, BN);
        constexpr uint32_t idesc_pv = make_idesc(fmt, 0, 1, BM, HD);
        uint64_t* gb = bars + 2 * NSTAGE + 7 * g;
        const uint32_t sQ = smem_u32(sm + OFF_Q + g * 32768);
        const uint32_t tSg = tmem + g * 256, tO = tmem + g * 256 + 128;
        bool alive = mbar_wait(gb + 6, 0, abort_flag, derr, 50);
        TileIter itr{-1, -1, 0, 0u};
        int it = 0;
        // O += P V with P (bf16, K-major) read from the first 32 columns of S buffer j&1
        auto issue_pv = [&](int j) -> bool {
          const int pb = j & 1;
          if (!mbar_wait(gb + 2 + pb, (j >> 1) & 1, abort_flag, derr, 51)) return false;
          tc_fence_after();
          const uint32_t sV = smem_u32(sm + OFF_V + (j % NSTAGE) * 16384);
          const uint32_t tP = tSg + pb * BN;
  #pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            uint64_t bd = sw128_desc(sV + kk * 2048, 8192, 1024);
            umma_ts(tO, tP + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(gb + 4 + pb);
          umma_commit(kv_empty + (j % NSTAGE));
          return true;
        };
        while (alive) {
          int kt0 = next_tile<PAIR>(itr, smask, p.nwords, bs, pmax, kvl);
          if (kt0 < 0) break;
          const int st = it % NSTAGE, sb = it & 1;
          if (!mbar_wait(kv_full + st, (it / NSTAGE) & 1, abort_flag, derr, 52)) { alive = false; break; }
          // S buffer sb holds P(it-2), read by PV(it-2).  This thread issued
          // PV(it-2) (after the softmax had released S(it-2)) before this QK,
          // and tcgen05.mma ops of one thread execute in issue order, so the
          // QK below cannot overwrite P before PV(it-2) has read it: no wait.
          tc_fence_after();
          const uint32_t sK = smem_u32(sm + OFF_K + st * 16384);
  #pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            uint64_t ad = sw128_desc(sQ + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            uint64_t bd = sw128_desc(sK + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
            umma_ss(tSg + sb * BN, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(gb + 0 + sb);
          if (it >= 1 && !issue_pv(it - 1)) { alive = false; break; }
          ++it;
        }
        if (alive && it >= 1) issue_pv(it - 1);
        // all MMAs of this group complete before TMEM is released
        umma_commit(mma_done + g);
        volatile int no_abort = 0;
        mbar_wait(mma_done + g, 0, &no_abort, nullptr, 54);
      }
      __syncwarp();
    }
  } else {
    regs_grow<kSoftmaxRegs>();
    if ((warp >> 2) < ngroups) {
      // ============ softmax / epilogue: group g, one thread per tile row ============
      const int g = warp >> 2;
      uint64_t* gb = bars + 2 * NSTAGE + 7 * g;
      uint64_t* s_full = gb + 0;
      uint64_t* p_full = gb + 2;
      uint64_t* pv_done = gb + 4;
      uint64_t* q_full = gb + 6;
      const uint32_t tS = tmem + g * 256, tO = tmem + g * 256 + 128;
      const int m = tid & 127;                 // row 0..127 of this group's tile
      const int i0 = i0A + g * p.TT;
      const int ntok = min(p.TT, qlen - i0);
      const int tok = i0 + m / G;
      const int hq = hk * G + (m % G);
      const bool row_ok = (m / G) < ntok;
      const int64_t pos = row_ok ? (int64_t)pos0 + tok : -1;
      const int64_t lstart = pos - a.local_window + 1;
      const int64_t rglob = row_base(a.seqs, s) + tok;
      const int64_t segs = (row_ok && a.seg_start) ? (int64_t)a.seg_start[rglob] : 0;
      // positions inside one sequence fit in 32 bits (kv lengths are int32)
      const int pos_i = (int)pos, lstart_i = (int)lstart, seg_i = (int)segs;
      // ---- Q row -> shared (swizzled K-major) ----
      {
        const T* qp = reinterpret_cast<const T*>(a.qo.q) +
                      (a.seqs.q_start ? rglob * a.qo.q_stride_tok
                                      : (int64_t)s * a.qo.q_stride_seq + (int64_t)tok * a.qo.q_stride_tok) +
                      (int64_t)hq * a.qo.q_stride_head;
        uint8_t* sq = sm + OFF_Q + g * 32768;
  #pragma unroll
        for (int cc = 0; cc < 16; ++cc) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (row_ok) v = *reinterpret_cast<const uint4*>(qp + cc * 8);
          const int region = cc >> 3, c8 = cc & 7;
          *reinterpret_cast<uint4*>(sq + region * 16384 + m * 128 + ((c8 ^ (m & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
      }
      // routed list cursor (none in gathered mode: the routed keys arrive as
      // partials merged in the epilogue)
      const int K = p.flags ? 0 : a.routes.K;
      // rows past the end of the tile read row 0's list (never used)
      const int64_t lrow = (int64_t)ih * p.n_rows + (row_ok ? rglob : 0);
      const int32_t* rl = p.cidx + lrow * K;
      const float* rbl = p.cbias + lrow * K * (PAIR ? 2 : 1);
      const bool has_bias = a.routes.bias != nullptr;
      // An entry's biases for the two 32-column halves of its key tile (PAIR:
      // the tile's two blocks; otherwise the block's bias for both).  plan_kernel
      // zero-fills the bias lists when there is no bias.
      auto ld_bias = [&](int j) -> float2 {
        if constexpr (PAIR) {
          return reinterpret_cast<const float2*>(rbl)[j];
        } else {
          const float v = rbl[j];
          return make_float2(v, v);
        }
      };
      auto key_of = [](int raw) -> int { return PAIR ? (raw >= 0 ? raw >> 2 : -1) : raw; };
      // cursor = entry cur_j; the raw entry after it is kept prefetched in
      // registers.  The prefetch is unconditional (index clamped to the list) and
      // its value is first used at the next advance, at least one key tile
      // later, so no instruction of the tile loop waits on it.
      int cur_j = 0;
      int cur_raw = (row_ok && K > 0) ? rl[0] : -1;
      float2 cur_bias = (row_ok && K > 0) ? ld_bias(0) : make_float2(0.0f, 0.0f);
      int nxt_raw = (row_ok && K > 1) ? rl[1] : -1;
      float2 nxt_bias_raw = (row_ok && K > 1) ? ld_bias(1) : make_float2(0.0f, 0.0f);
      const float sl2 = a.scale * 1.4426950408889634f;
      const float LOG2E = 1.4426950408889634f;
      // Running max (exp2 domain) starts at the row's largest routed bias: the
      // bias of the top entmax block is what makes a row's max jump.  Any start
      // value is exact (O and l share the reference).  O is rescaled only when a
      // logit exceeds the running max by more than kGrowLog2: p stays below
      // 2^kGrowLog2, far inside the bf16/fp32 range, and a start above the true
      // max only scales p by a power of two.
      float m_run = 0.0f, l_run = 0.0f;
      if (row_ok && has_bias && K > 0)
        m_run = fmaxf(0.0f, p.rowmax[(int64_t)ih * p.n_rows + rglob] * LOG2E);
      const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
      TileIter itr{-1, -1, 0, 0u};
      int it = 0;
      bool alive = true;
      // Advance the routed-list cursor to the entry of key tile `key` (block
      // id, or tile index with PAIR); sel0/sel1 and b20/b21 describe the two
      // 32-column halves of the tile for this row.  Every kept entry has a key
      // tile of its own, so the cursor moves at most one entry per tile and
      // takes the prefetched entry; the refill is unconditional (same address
      // while the cursor stays) and first read a tile later.  The inner walk
      // only serves lists that skip a tile, which plan_kernel never writes.
      auto cursor_to = [&](int key, bool& sel0, bool& sel1, float& b20, float& b21) {
        int cur = key_of(cur_raw);
        if (K > 0) {
          if (cur >= 0 && cur < key) {
            ++cur_j;
            cur_raw = cur_j < K ? nxt_raw : -1;
            cur_bias = nxt_bias_raw;
            cur = key_of(cur_raw);
            while (cur >= 0 && cur < key) {
              ++cur_j;
              cur_raw = cur_j < K ? rl[cur_j] : -1;
              cur_bias = cur_j < K ? ld_bias(cur_j) : make_float2(0.0f, 0.0f);
              cur = key_of(cur_raw);
            }
          }
          const int j2 = min(cur_j + 1, K - 1);
          nxt_raw = rl[j2];
          nxt_bias_raw = ld_bias(j2);
        }
        const bool on = cur == key;
        sel0 = on && (!PAIR || (cur_raw & 1));
        sel1 = on && (!PAIR || (cur_raw & 2));
        b20 = sel0 ? cur_bias.x * LOG2E : 0.0f;
        b21 = sel1 ? cur_bias.y * LOG2E : 0.0f;
      };
      auto tile_key = [&]() -> int { return PAIR ? (itr.b >> 1) : itr.b; };
      // The iterator and the cursor run one tile ahead: the next tile's
      // bookkeeping is done while this tile's S load is in flight.
      int kt0 = next_tile<PAIR>(itr, smask, p.nwords, bs, pmax, kvl);
      bool sel0 = false, sel1 = false;
      float b20 = 0.0f, b21 = 0.0f;
      if (kt0 >= 0) cursor_to(tile_key(), sel0, sel1, b20, b21);
      while (alive && kt0 >= 0) {
        const int st = it % NSTAGE, sb = it & 1;
        // zero V rows past the end of the sequence (never multiply garbage by P = 0)
        if (kt0 + BN > kvl) {
          if (!mbar_wait_warp(kv_full + st, (it / NSTAGE) & 1, abort_flag, derr, 60)) { alive = false; break; }
          const int r0 = kvl - kt0;
          uint8_t* dV = sm + OFF_V + st * 16384;
          for (int e = m; e < (BN - r0) * 16; e += 128) {
            const int row = r0 + e / 16, ch = e % 16;
            *reinterpret_cast<uint4*>(dV + (ch >> 3) * 8192 + row * 128 + ((ch & 7) << 4)) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        if (!mbar_wait_warp(s_full + sb, (it >> 1) & 1, abort_flag, derr, 61)) { alive = false; break; }
        tc_fence_after();
        // Column c (half h = c / 32) of this key tile is kept iff
        // lo_h <= c <= hi, where lo_h is the first local column, or the first
        // attendable column when half h's block is routed; logits are
        // x = s*scale*log2e + (local ? 0 : bias of half h) - m_run.
        // S(it) -> registers; the row's mask terms are computed while the
        // load is in flight (the wait comes before any branch on them)
        const uint32_t tSb = tS + sb * BN + lane_base;
        float x[64];
        tmem_ld32f(tSb, x);
        tmem_ld32f(tSb + 32, x + 32);
        const int hi = min(63, max(-1, pos_i - kt0));
        const int lo_seg = min(64, max(0, seg_i - kt0));
        const int lo_loc = min(64, max(0, lstart_i - kt0));
        const int lo0 = max(sel0 ? 0 : lo_loc, lo_seg);
        const int lo1 = PAIR ? max(sel1 ? 0 : lo_loc, lo_seg) : lo0;
        const float add_loc = -m_run;
        const float add_rem0 = b20 - m_run;
        const float add_rem1 = PAIR ? b21 - m_run : add_rem0;
        const int kt_next = next_tile<PAIR>(itr, smask, p.nwords, bs, pmax, kvl);
        bool sel0_next = false, sel1_next = false;
        float b20_next = 0.0f, b21_next = 0.0f;
        if (kt_next >= 0) cursor_to(tile_key(), sel0_next, sel1_next, b20_next, b21_next);
        uint32_t pk[32];
        tmem_ld_wait();
        // Pure halves for this row: all 32 columns of a half kept with one
        // additive term, or none kept.  When both halves of every row of the
        // warp are pure and the tile lies inside the sequence (tiles away from
        // the window edge and the diagonal), the logits take one packed FFMA
        // per 2 columns (an empty half adds -inf), P is produced directly, and
        // the rescale test runs on the row's partial sums.
        const bool empty0 = lo0 > min(hi, 31);
        const bool full0 = lo0 == 0 && hi >= 31 && (lo_loc == 0 || lo_loc >= 32);
        const bool empty1 = max(lo1, 32) > hi;
        const bool full1 = lo1 <= 32 && hi == 63 && (lo_loc <= 32 || lo_loc == 64);
        bool done = false;
        if (__all_sync(0xffffffffu, (empty0 || full0) && (empty1 || full1)) && kt0 + BN <= kvl) {
          const float add0 = empty0 ? -INFINITY : (lo_loc == 0 ? add_loc : add_rem0);
          const float add1 = empty1 ? -INFINITY : (lo_loc <= 32 ? add_loc : add_rem1);
          const uint64_t sl2v = f2_pack(sl2, sl2), addv0 = f2_pack(add0, add0),
                         addv1 = f2_pack(add1, add1);
          uint64_t lsv = f2_pack(0.0f, 0.0f);
  #pragma unroll
          for (int e = 0; e < 32; ++e) {
            float y0, y1;
            f2_unpack(ffma2(f2_pack(x[2 * e], x[2 * e + 1]), sl2v, e < 16 ? addv0 : addv1), y0, y1);
            // one pair in four on the FMA pipe, the rest on the MUFU unit
            float p0, p1;
            if ((e & 3) == 3) {
              f2_unpack(exp2_poly2(y0, y1), p0, p1);
            } else {
              p0 = fast_exp2(y0);
              p1 = fast_exp2(y1);
            }
            lsv = fadd2(lsv, f2_pack(p0, p1));
            pk[e] = pack2(p0, p1, (T*)nullptr);
          }
          // every p <= 2^kGrowLog2 when both partial sums are (sums of
          // non-negative terms; inf / NaN fail the test too)
          float l0, l1;
          f2_unpack(lsv, l0, l1);
          const bool big = !(fmaxf(l0, l1) <= kGrowP);
          if (!__any_sync(0xffffffffu, big)) {
            l_run += l0 + l1;
            done = true;
          }
        }
        if (!done) {
          // general path: row max, optional rescale of O, then P.  S is read
          // in 32-column halves, once per pass (it is intact until P is stored
          // over it), which keeps the rare path inside the register budget.
          float mx = -INFINITY;
  #pragma unroll
          for (int h = 0; h < 2; ++h) {
            float x[32];
            tmem_ld32f(tSb + 32 * h, x);
            tmem_ld_wait();
  #pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int c = 32 * h + j;
              const float v = fmaf(x[j], sl2, c >= lo_loc ? add_loc : (h ? add_rem1 : add_rem0));
              mx = fmaxf(mx, (c >= (h ? lo1 : lo0) && c <= hi) ? v : -INFINITY);
            }
          }
          const bool need = mx > kGrowLog2;
          float shift = 0.0f;
          if (__any_sync(0xffffffffu, need)) {
            const float f = need ? fast_exp2(-mx) : 1.0f;
            if (it > 0) {
              if (!mbar_wait_warp(pv_done + ((it - 1) & 1), ((it - 1) >> 1) & 1, abort_flag, derr, 62)) { alive = false; break; }
              tc_fence_after();
  #pragma unroll 1
              for (int q4 = 0; q4 < 4; ++q4) {
                uint32_t o[32];
                tmem_ld32(tO + q4 * 32 + lane_base, o);
                tmem_ld_wait();
  #pragma unroll
                for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
                tmem_st32(tO + q4 * 32 + lane_base, o);
              }
              tmem_st_wait();
            }
            l_run *= f;
            if (need) {
              m_run += mx;
              shift = mx;
            }
          }
          float ls4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  #pragma unroll
          for (int h = 0; h < 2; ++h) {
            float x[32];
            tmem_ld32f(tSb + 32 * h, x);
            tmem_ld_wait();
  #pragma unroll
            for (int e = 0; e < 16; ++e) {
              float pp[2];
  #pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int j = 2 * e + u, c = 32 * h + j;
                const float v = fmaf(x[j], sl2, (c >= lo_loc ? add_loc : (h ? add_rem1 : add_rem0)) - shift);
                pp[u] = fast_exp2((c >= (h ? lo1 : lo0) && c <= hi) ? v : -INFINITY);
              }
              ls4[e & 3] += pp[0] + pp[1];
              pk[16 * h + e] = pack2(pp[0], pp[1], (T*)nullptr);
            }
          }
          l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
        }
        // P(it) over the first 32 columns of S buffer sb (this thread's S reads
        // completed above), then hand it to the MMA warp
        tmem_st32(tSb, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + sb);
        ++it;
        kt0 = kt_next;
        sel0 = sel0_next;
        sel1 = sel1_next;
        b20 = b20_next;
        b21 = b21_next;
      }
      // ---- epilogue ----
      bool have_o = alive && it > 0;
      if (have_o && !mbar_wait_warp(pv_done + ((it - 1) & 1), ((it - 1) >> 1) & 1, abort_flag, derr, 64)) have_o = false;
      tc_fence_after();
      // Gathered mode: this kernel holds the row's window keys only; their
      // normalised output and log2-sum-exp go to the row's partial slot K,
      // merged with the routed partials by the merge kernel.
      const bool win = have_o && l_run > 0.0f;
      const float inv_l = win ? 1.0f / l_run : 0.0f;
      const int Kf = a.routes.K;
      const int64_t pent =
          p.flags ? (((int64_t)(s - p.s0) * p.prows + (tok - 2 * p.pj0 * p.TT)) * p.hqn + (hq - p.hq0)) * (Kf + 1) + Kf
                  : 0;
      T* op = reinterpret_cast<T*>(a.qo.out) +
              (a.seqs.q_start ? rglob * a.qo.o_stride_tok
                              : (int64_t)s * a.qo.o_stride_seq + (int64_t)tok * a.qo.o_stride_tok) +
              (int64_t)hq * a.qo.o_stride_head;
      if (p.flags) op = reinterpret_cast<T*>(const_cast<uint16_t*>(p.part_o) + pent * HD);
      // The group's Q buffer is free (its last QK completed before the last
      // PV): the rows are staged there (16-byte chunk c of row m at
      // ((c ^ (m & 15)) << 4)), then every warp writes its 32 rows two per
      // instruction (lanes 0-15 one row, 16-31 the next: 512 contiguous
      // bytes per instruction instead of 32 scattered 16-byte pieces), to
      // the output and, fused output gather, to every peer rank's copy of it
      // (P2P stores over NVLink; same strides, same offset).
      uint8_t* stg = sm + OFF_Q + g * 32768;
  #pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o[32];
        tmem_ld32(tO + q4 * 32 + lane_base, o);
        tmem_ld_wait();
        uint32_t pko[16];
  #pragma unroll
        for (int c = 0; c < 32; c += 2)
          pko[c >> 1] = pack2(win ? __uint_as_float(o[c]) * inv_l : 0.0f,
                              win ? __uint_as_float(o[c + 1]) * inv_l : 0.0f, (T*)nullptr);
  #pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int c = q4 * 4 + v;
          *reinterpret_cast<uint4*>(stg + m * 256 + ((c ^ (m & 15)) << 4)) =
              make_uint4(pko[4 * v], pko[4 * v + 1], pko[4 * v + 2], pko[4 * v + 3]);
        }
      }
      __syncwarp();
      {
        T* obase = p.flags ? reinterpret_cast<T*>(const_cast<uint16_t*>(p.part_o)) : reinterpret_cast<T*>(a.qo.out);
        const int64_t myoff = row_ok ? (int64_t)(op - obase) : -1;
        const int npeer = p.flags ? 0 : a.n_peers;
        const int c = lane & 15;
  #pragma unroll 4
        for (int j = 0; j < 16; ++j) {
          const int rr = 2 * j + (lane >> 4);                 // row of the warp
          const int64_t off = __shfl_sync(0xffffffffu, myoff, rr);
          const int mr = (warp & 3) * 32 + rr;
          const uint4 val = *reinterpret_cast<const uint4*>(stg + mr * 256 + ((c ^ (mr & 15)) << 4));
          if (off >= 0) {
            *reinterpret_cast<uint4*>(obase + off + c * 8) = val;
            for (int pr = 0; pr < npeer; ++pr)
              *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out_peers[pr]) + off + c * 8) = val;
          }
        }
      }
      // The peer stores are posted: no fence here, so an SM takes its next
      // tile while they drain over NVLink.  The grid completes only once all
      // of its writes are performed, and the caller's completion step is
      // stream-ordered after the grid, so it sees every row in place.
      if (row_ok && p.flags) {
        const_cast<float*>(p.part_lse)[pent] = win ? m_run + log2f(l_run) : -INFINITY;
      } else if (row_ok && a.qo.lse) {
        const float lse = win ? (m_run + log2f(l_run)) * 0.6931471805599453f : -INFINITY;
        a.qo.lse[(a.seqs.q_start ? rglob * a.qo.lse_stride_tok
                                 : (int64_t)s * a.qo.lse_stride_seq + (int64_t)tok * a.qo.lse_stride_tok) +
                 (int64_t)hq * a.qo.lse_stride_head] = lse;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// K/V tensor map, boxes of 64 dims x `rows` tokens (128-byte swizzle)
static int make_kv_map(CUtensorMap* map, const void* base, const DashPrefillArgs& a, bool paged, int rows) {
  auto enc = get_encode();
  if (!enc) return set_error(DASH_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int esz = 2;
  cuuint64_t dims[4], strides[3];
  dims[0] = HD;
  dims[1] = paged ? (cuuint64_t)a.block_size : (cuuint64_t)a.seqs.kv_len_fixed;
  dims[2] = (cuuint64_t)a.kv.n_kv_heads;
  dims[3] = paged ? (cuuint64_t)a.kv.num_pages : (cuuint64_t)a.seqs.n_seq;
  strides[0] = (cuuint64_t)a.kv.stride_tok * esz;
  strides[1] = (cuuint64_t)a.kv.stride_head * esz;
  strides[2] = (cuuint64_t)a.kv.stride_seq * esz;
  cuuint32_t box[4] = {64, (cuuint32_t)rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int k = 0; k < 3; ++k)
    if (strides[k] % 16 != 0 || strides[k] == 0)
      return set_error(DASH_ERR_INVALID, "K/V strides must be non-zero multiples of 16 bytes");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(DASH_ERR_INVALID, "K/V base must be 16-byte aligned");
  CUresult r = enc(map, a.kv.dtype == DASH_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DASH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DASH_OK;
}

static void plan_geometry(const DashPrefillArgs& a, int64_t n_rows, PrefillPlan& p) {
  const int G = a.qo.n_heads / a.kv.n_kv_heads;
  p.G = G;
  p.TT = BM / G;
  p.tiles_per_seq = (a.seqs.max_q_len + p.TT - 1) / p.TT;
  p.paged = a.kv.block_table != nullptr;
  p.nblk_cap = p.paged ? (int)a.kv.bt_stride
                       : (a.seqs.kv_len_fixed + a.block_size - 1) / a.block_size;
  p.nwords = (p.nblk_cap + 31) / 32;
  p.n_rows = n_rows;
  // one chunk: every sequence, tile pair and kv head
  p.s0 = 0;
  p.sn = a.seqs.n_seq;
  p.pj0 = 0;
  p.npj = (p.tiles_per_seq + 1) / 2;
  p.hk0 = 0;
  p.hq0 = 0;
  p.hqn = a.qo.n_heads;
}

bool prefill_gathered_supported(const DashPrefillArgs& a) {
  if (a.kv.dtype == DASH_DTYPE_F32 || a.kv.n_kv_heads <= 0) return false;
  const int G = a.qo.n_heads / a.kv.n_kv_heads;
  const int bs = a.block_size;
  return (bs == 32 || bs == 64 || bs == 128) && (G == 1 || G == 2 || G == 4) && a.routes.K > 0 &&
         a.routes.K <= kPlanMaxSlots;
}

// Mode 0 picks by the expected union waste.  A 128-row tile's union covers
// nearly every candidate block when routes vary from row to row, so the
// tile-major kernel executes about (candidates x block) keys per row against
// K x block routed ones; the gathered split pays a 260-byte partial per
// routed (row, head, block) instead.  Measured on B200: 128-token blocks
// with K = 64 run 572 ms gathered vs 625 ms tile-major;
// 64-token blocks with K = 16 (config 2) 2.25 ms vs 1.13 ms.  So the gathered
// split is taken for blocks of 128 tokens with K >= 32, or on request (2).
static bool use_gathered(const DashPrefillArgs& a) {
  if (a.mode == 1 || !prefill_gathered_supported(a)) return false;
  return a.mode == 2 || (a.block_size >= 128 && a.routes.K >= 32);
}

// Gathered mode: chunks of sequences x tile pairs x kv heads whose partials
// (bf16/fp16 output row + fp32 log2-sum-exp per list slot and one for the
// window part) fit the budget.
struct GatherChunks {
  int hcn, sn, npj;      // kv heads, sequences, tile pairs per chunk
  int wpt, wps;          // flag words per tile / per (sequence, block)
  size_t flags_bytes, lse_bytes, o_bytes;
};
constexpr size_t kPartBytes = HD * 2 + 4;        // one partial
constexpr int kDefaultPartMiB = 2048;

static GatherChunks gather_chunks(const DashPrefillArgs& a, const PrefillPlan& p) {
  GatherChunks c{};
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  c.wpt = p.TT / 32;
  c.wps = p.tiles_per_seq * c.wpt;
  c.flags_bytes = (size_t)nih * a.seqs.n_seq * p.nblk_cap * c.wps * 4;
  const int pairs = (p.tiles_per_seq + 1) / 2;
  const int nkv = a.kv.n_kv_heads, ns = a.seqs.n_seq;
  // one unit = (sequence, tile pair, kv head): 256 query rows x heads, K
  // routed slots + the window slot each
  const size_t unit = (size_t)2 * BM * (a.routes.K + 1) * kPartBytes;
  const size_t budget = (size_t)(a.part_budget_mib > 0 ? a.part_budget_mib : kDefaultPartMiB) << 20;
  const size_t cap = budget / unit > 0 ? budget / unit : 1;
  auto balance = [](int total, size_t per) -> int {
    const int n = (int)((total + per - 1) / per);          // chunks
    return (total + n - 1) / n;                            // even split
  };
  c.hcn = nkv;
  c.sn = ns;
  c.npj = pairs;
  if ((size_t)ns * pairs * nkv > cap) {
    if ((size_t)ns * pairs <= cap) {
      c.hcn = balance(nkv, cap / ((size_t)ns * pairs));
    } else if ((size_t)pairs <= cap) {
      c.hcn = 1;
      c.sn = balance(ns, cap / pairs);
    } else {
      c.hcn = 1;
      c.sn = 1;
      c.npj = balance(pairs, cap);
    }
  }
  const size_t entries = (size_t)c.sn * (2 * c.npj * p.TT) * (c.hcn * p.G) * (a.routes.K + 1);
  c.lse_bytes = entries * 4;
  c.o_bytes = entries * HD * 2;
  return c;
}

// Workspace: canonical block lists, their biases (two per entry with
// 32-token blocks in the tile-major kernel), per-tile unions, per-row largest
// bias; gathered mode adds the per-block row flags and the partials.
static size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

struct PrefillWs {
  size_t lists, blists, masks, rowmax;
  size_t flags, lse, o;
  size_t total() const { return lists + blists + masks + rowmax + flags + lse + o; }
};

static PrefillWs prefill_ws(const DashPrefillArgs& a, int64_t n_rows, const PrefillPlan& p, bool gathered) {
  PrefillWs w{};
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const bool pair = a.block_size == 32 && a.kv.dtype != DASH_DTYPE_F32 && !gathered;
  w.lists = round256((size_t)nih * n_rows * a.routes.K * 4);
  w.blists = pair ? 2 * w.lists : w.lists;
  w.masks = round256((size_t)nih * a.seqs.n_seq * p.tiles_per_seq * p.nwords * 4);
  w.rowmax = round256((size_t)nih * n_rows * 4);
  if (gathered) {
    const GatherChunks c = gather_chunks(a, p);
    w.flags = round256(c.flags_bytes);
    w.lse = round256(c.lse_bytes);
    w.o = round256(c.o_bytes);
  }
  return w;
}

size_t prefill_workspace(const DashPrefillArgs& a, int64_t n_rows) {
  PrefillPlan p{};
  plan_geometry(a, n_rows, p);
  return prefill_ws(a, n_rows, p, use_gathered(a)).total();
}

template <bool PAIR>
static int launch_plan(const DashPrefillArgs& a, const PrefillPlan& p, int32_t* cidx, float* cbias,
                       uint32_t* tmask, float* rowmax, cudaStream_t st) {
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  // every tile's union words (and flag words) are written, also with no lists
  dim3 g1((unsigned)(a.seqs.n_seq * p.tiles_per_seq), nih);
  const int K = a.routes.K;
  const size_t dyn = p.flags ? (size_t)p.nblk_cap * p.wpt * 4 : 0;
  auto plan = [&](auto kern) -> int {
    if (dyn > 0 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess)
      return set_error(DASH_ERR_CUDA, "cudaFuncSetAttribute(plan_kernel) failed");
    kern<<<g1, kPlanWarps * 32, dyn, st>>>(a, p, cidx, cbias, tmask, rowmax);
    count_launch();
    return check_launch("plan_kernel");
  };
  if (K <= 32) return plan(plan_kernel<1, PAIR>);
  if (K <= 64) return plan(plan_kernel<2, PAIR>);
  return plan(plan_kernel<kPlanMaxSlots / 32, PAIR>);
}

template <typename T, bool PAGED, bool PAIR>
static int launch_local(const DashPrefillArgs& a, const PrefillPlan& p, const CUtensorMap& mk,
                        const CUtensorMap& mv, int hcn, cudaStream_t st) {
  auto kern = prefill_kernel<T, PAGED, PAIR>;
  // the in-kernel register growth waits until the pool covers it: launch
  // only a build whose per-thread count matches the split
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "cudaFuncGetAttributes(prefill_kernel) failed");
  if (fa.numRegs != kLaunchRegs)
    return set_error(DASH_ERR_UNSUPPORTED, "prefill_kernel built with %d registers per thread, "
                     "the register split needs %d", fa.numRegs, kLaunchRegs);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "cudaFuncSetAttribute(prefill_kernel) failed");
  dim3 grid((unsigned)(p.sn * p.npj), (unsigned)hcn);
  kern<<<grid, NTHREADS, SMEM_BYTES, st>>>(mk, mv, a, p);
  count_launch();
  return check_launch("prefill_kernel");
}

static int launch_local_any(const DashPrefillArgs& a, const PrefillPlan& p, const CUtensorMap& mk,
                            const CUtensorMap& mv, bool pair, int hcn, cudaStream_t st) {
  const bool paged = p.paged != 0;
  if (a.kv.dtype == DASH_DTYPE_BF16) {
    if (pair)
      return paged ? launch_local<__nv_bfloat16, true, true>(a, p, mk, mv, hcn, st)
                   : launch_local<__nv_bfloat16, false, true>(a, p, mk, mv, hcn, st);
    return paged ? launch_local<__nv_bfloat16, true, false>(a, p, mk, mv, hcn, st)
                 : launch_local<__nv_bfloat16, false, false>(a, p, mk, mv, hcn, st);
  }
  if (pair)
    return paged ? launch_local<__half, true, true>(a, p, mk, mv, hcn, st)
                 : launch_local<__half, false, true>(a, p, mk, mv, hcn, st);
  return paged ? launch_local<__half, true, false>(a, p, mk, mv, hcn, st)
               : launch_local<__half, false, false>(a, p, mk, mv, hcn, st);
}

int launch_prefill(const DashPrefillArgs& a, int64_t n_rows, cudaStream_t st) {
  if (n_rows == 0 || a.seqs.n_seq == 0) return DASH_OK;
  PrefillPlan p{};
  plan_geometry(a, n_rows, p);
  if (p.nwords > MAX_MASK_WORDS)
    return set_error(DASH_ERR_UNSUPPORTED, "too many blocks per sequence (%d > %d)", p.nblk_cap,
                     MAX_MASK_WORDS * 32);
  const bool f32 = a.kv.dtype == DASH_DTYPE_F32;
  const bool gathered = use_gathered(a);
  // 32-token blocks pair up in the tile-major kernel's 64-key tiles (also
  // for the window part in gathered mode); the fp32 kernel and the routed
  // kernel read plain per-block lists
  const bool pair_kernel = a.block_size == 32 && !f32;
  const bool pair_plan = pair_kernel && !gathered;
  const PrefillWs w = prefill_ws(a, n_rows, p, gathered);
  uint8_t* ws = reinterpret_cast<uint8_t*>(a.workspace);
  int32_t* cidx = reinterpret_cast<int32_t*>(ws);
  float* cbias = reinterpret_cast<float*>(ws + w.lists);
  uint32_t* tmask = reinterpret_cast<uint32_t*>(ws + w.lists + w.blists);
  float* rowmax = reinterpret_cast<float*>(ws + w.lists + w.blists + w.masks);
  p.cidx = cidx;
  p.cbias = cbias;
  p.tmask = tmask;
  p.rowmax = rowmax;
  GatherChunks gc{};
  if (gathered) {
    gc = gather_chunks(a, p);
    uint8_t* g = ws + w.lists + w.blists + w.masks + w.rowmax;
    p.flags = reinterpret_cast<uint32_t*>(g);
    p.wpt = gc.wpt;
    p.wps = gc.wps;
    p.part_lse = reinterpret_cast<const float*>(g + w.flags);
    p.part_o = reinterpret_cast<const uint16_t*>(g + w.flags + w.lse);
  }
  int rc = pair_plan ? launch_plan<true>(a, p, cidx, cbias, tmask, rowmax, st)
                     : launch_plan<false>(a, p, cidx, cbias, tmask, rowmax, st);
  if (rc) return rc;
  if (f32) return launch_prefill_f32(a, p, st);
  CUtensorMap mk, mv;
  const int rows = (p.paged && a.block_size < BN) ? a.block_size : BN;
  rc = make_kv_map(&mk, a.kv.k, a, p.paged, rows);
  if (!rc) rc = make_kv_map(&mv, a.kv.v, a, p.paged, rows);
  if (rc) return rc;
  if (!gathered) return launch_local_any(a, p, mk, mv, pair_kernel, a.kv.n_kv_heads, st);
  // gathered: the routed kernel's boxes hold min(block_size, 64) rows
  CUtensorMap rk = mk, rv = mv;
  const int rrows = a.block_size < BN ? a.block_size : BN;
  if (rrows != rows) {
    rc = make_kv_map(&rk, a.kv.k, a, p.paged, rrows);
    if (!rc) rc = make_kv_map(&rv, a.kv.v, a, p.paged, rrows);
    if (rc) return rc;
  }
  const int pairs = (p.tiles_per_seq + 1) / 2;
  for (int hk0 = 0; hk0 < a.kv.n_kv_heads; hk0 += gc.hcn) {
    const int hcn = std::min(gc.hcn, a.kv.n_kv_heads - hk0);
    for (int s0 = 0; s0 < a.seqs.n_seq; s0 += gc.sn) {
      for (int pj0 = 0; pj0 < pairs; pj0 += gc.npj) {
        PrefillPlan c = p;
        c.s0 = s0;
        c.sn = std::min(gc.sn, a.seqs.n_seq - s0);
        c.pj0 = pj0;
        c.npj = std::min(gc.npj, pairs - pj0);
        c.hk0 = hk0;
        c.hq0 = hk0 * p.G;
        c.hqn = hcn * p.G;
        c.prows = 2 * c.npj * p.TT;
        rc = launch_prefill_routed(a, c, rk, rv, hcn, st);
        if (!rc) rc = launch_local_any(a, c, mk, mv, pair_kernel, hcn, st);
        if (!rc) rc = launch_prefill_merge(a, c, st);
        if (rc) return rc;
      }
    }
  }
  return DASH_OK;
}

}  // namespace dash
