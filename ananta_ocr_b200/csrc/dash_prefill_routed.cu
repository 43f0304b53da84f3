// dash_prefill_routed.cu -- the routed part of the DASH prefill, gathered by
// key block (sm_100a tensor cores).
//
// With noise-like routes, the 128 rows of a query tile route different blocks
// and the tile-major kernel (dash_prefill.cu) multiplies every row against the
// union of their blocks: ~4x the useful work at BASELINE config 2 and ~7x at
// config 4.  Here the routed keys are taken block by block instead: one CTA
// per (sequence, kv head, key block) gathers the query rows that routed the
// block (the plan kernel's per-block row bitmask) into 128-slot batches (a
// slot = a row x one query head of the kv head), so every product is useful:
//   producer warp 5   enumerates the next batch's rows; per slot: q row
//                     offset, the slot's list position, bias, key range
//   slot warps 0-3    gather the slots' q rows into shared memory (cp.async,
//                     128-byte swizzle); softmax of the slot's row (thread =
//                     slot = TMEM lane) over the block's keys below its
//                     window; epilogue: normalised partial output (bf16) and
//                     its log2-sum-exp into the partial scratch
//   MMA warp 4        S = Q K^T  (tcgen05 M=128 slots, N=block, K=128 dims)
//                     O = P V    (M=128, N=128, K=block; P from TMEM)
// The block's K and V (TMA) stay in shared memory for all its batches.  The
// next batch's q rows are gathered while the current batch's PV runs.  The
// local-window kernel (prefill_kernel, gathered mode) merges the partials of a
// row with its window part in its epilogue.
//
// Semantics: sparse_gather_e2e_triton.py:34-115 (keys of a routed block below
// the query's local window, + the slot's bias), WHL attend_triton.py:88-292.
#include <cudaTypedefs.h>
#include <climits>
#include "dash_common.cuh"
#include "dash_internal.h"
#include "dash_prefill_plan.cuh"

namespace dash {
namespace {

constexpr int NS = 128;                  // slots per batch
constexpr int HD = 128;                  // head dim
constexpr int kSlotWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProdWarp = 5;
constexpr int kThreads = 6 * 32;
constexpr uint32_t TMEM_COLS = 256;      // S (<= 128 columns) | O (128)
constexpr float LOG2E = 1.4426950408889634f;

struct RMeta {
  int64_t qoff[NS];    // element offset of the slot's q row
  int64_t poff[NS];    // partial entry of the slot (chunk layout); -1: padding
  float bias2[NS];     // bias * log2(e)
  int klo[NS];         // keys [klo, kcut) of the block count for the slot
  int kcut[NS];
  int rowtok[NS];      // token index of each gathered row (slots row * G + g)
  int ns;
  int pad[3];
};

template <int BS>
struct RLayout {
  static constexpr int OFF_Q = 0;                        // 2 halves x [128 slots][128 B]
  static constexpr int OFF_K = 32768;                    // 2 halves x [BS keys][128 B]
  static constexpr int OFF_V = OFF_K + BS * 256;
  static constexpr int OFF_META = OFF_V + BS * 256;      // 2 x RMeta
  static constexpr int OFF_BAR = OFF_META + 2 * (int)sizeof(RMeta);
  // at most two CTAs per SM: each takes half of the SM's 512 TMEM columns
  static constexpr int USED = OFF_BAR + 128 + 1024;
  static constexpr int SMEM = USED > 80 * 1024 ? USED : 80 * 1024;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all_r() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

}  // namespace

template <typename T, bool PAGED, int BS>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_routed_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const DashPrefillArgs a, const PrefillPlan p) {
  using L = RLayout<BS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RMeta* meta = reinterpret_cast<RMeta*>(sm + L::OFF_META);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;
  uint64_t* s_full = bars + 2;
  uint64_t* p_full = bars + 3;
  uint64_t* o_full = bars + 4;
  uint64_t* o_free = bars + 5;
  uint64_t* meta_full = bars + 6;     // [2]
  uint64_t* meta_empty = bars + 8;    // [2]
  uint64_t* mma_done = bars + 10;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 12);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sl = blockIdx.x / p.nblk_cap, b = blockIdx.x - sl * p.nblk_cap;
  const int s = p.s0 + sl;
  const int hk = p.hk0 + blockIdx.y;
  const int kvl = kv_len_of(a.seqs, s);
  if ((int64_t)b * BS >= kvl) return;
  // query tokens of this chunk: [i_lo, i_hi), flag words [i_lo / 32, w_hi)
  const int qlen = q_len_of(a.seqs, s);
  const int i_lo = 2 * p.pj0 * p.TT;
  const int i_hi = min(qlen, 2 * (p.pj0 + p.npj) * p.TT);
  if (i_lo >= i_hi) return;
  const int w_lo = i_lo >> 5, w_hi = (i_hi + 31) >> 5;
  const int G = p.G, H = a.qo.n_heads, K = a.routes.K;
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const int ih = (hk * G) / (H / nih);
  const uint32_t* fl = p.flags + (((int64_t)ih * a.seqs.n_seq + s) * p.nblk_cap + b) * p.wps;
  // no row routed this block: nothing to do (uniform exit before any setup)
  {
    uint32_t any = 0u;
    for (int w = w_lo + tid; w < w_hi; w += kThreads) any |= fl[w];
    if (!__syncthreads_or(any != 0u)) return;
  }
  DeviceError* derr = a.device_error;
  if (tid == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, kSlotWarps);
    mbar_init(s_full, 1);
    mbar_init(p_full, kSlotWarps);
    mbar_init(o_full, 1);
    mbar_init(o_free, kSlotWarps);
    mbar_init(meta_full + 0, 1);
    mbar_init(meta_full + 1, 1);
    mbar_init(meta_empty + 0, kSlotWarps);
    mbar_init(meta_empty + 1, kSlotWarps);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == kMmaWarp) { tmem_alloc(tmem_holder, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == kProdWarp) {
    // ================= producer: K/V of the block, then slot batches =================
    bool kv_issued = false;
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      constexpr int R = BS < 64 ? BS : 64;            // rows per TMA box
      int c1 = b * BS, c3 = s;
      bool ok = true;
      if (PAGED) {
        const int64_t page = a.kv.block_table[(int64_t)s * a.kv.bt_stride + b];
        if (page < 0 || page >= a.kv.num_pages) {
          record_error(derr, DASH_DEV_BAD_PAGE, 90, page);
          ok = false;
        }
        c1 = 0;
        c3 = (int)page;
      }
      if (ok) {
        mbar_arrive_expect_tx(kv_full, 2 * BS * 256);
#pragma unroll
        for (int dh = 0; dh < 2; ++dh)
#pragma unroll
          for (int r0 = 0; r0 < BS; r0 += R) {
            tma_load_4d(sm + L::OFF_K + dh * BS * 128 + r0 * 128, &tmK, kv_full, dh * 64, c1 + r0, hk, c3);
            tma_load_4d(sm + L::OFF_V + dh * BS * 128 + r0 * 128, &tmV, kv_full, dh * 64, c1 + r0, hk, c3);
          }
        kv_issued = true;
      } else {
        mbar_arrive(kv_full);
      }
    }
    const int pos0 = pos0_of(a.seqs, s);
    const int64_t rb = row_base(a.seqs, s);
    const int cap = NS / G;
    // i_lo is a multiple of 64 and flag bits past qlen are zero, so whole
    // words in [w_lo, w_hi) hold exactly this chunk's tokens
    int next_row = i_lo;
    for (int n = 0;; ++n) {
      const int buf = n & 1;
      RMeta& M = meta[buf];
      if (n >= 2 && !mbar_wait_warp(meta_empty + buf, ((n >> 1) - 1) & 1, abort_flag, derr, 91)) break;
      // rows of this batch: 32 bitmask words per step, one per lane
      int cnt = 0;
      while (cnt < cap && next_row < i_hi) {
        const int w = (next_row >> 5) + lane;
        uint32_t m = 0u;
        if (w < w_hi) {
          m = fl[w];
          if (lane == 0) m &= 0xffffffffu << (next_row & 31);
        }
        const int c = __popc(m);
        int incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += o;
        }
        const int excl = incl - c;
        const int tot = __shfl_sync(0xffffffffu, incl, 31);
        const int room = cap - cnt;
        const int take = max(0, min(c, room - excl));
        uint32_t mm = m;
        for (int k = 0; k < take; ++k) {
          const int bit = __ffs(mm) - 1;
          mm &= mm - 1u;
          M.rowtok[cnt + excl + k] = w * 32 + bit;
        }
        if (tot <= room) {
          cnt += tot;
          next_row = ((next_row >> 5) + 32) * 32;
        } else {
          // the lane holding the boundary: its first untaken row resumes the next batch
          const bool bnd = excl <= room && excl + c > room;
          const int src = __ffs(__ballot_sync(0xffffffffu, bnd)) - 1;
          const int resume = w * 32 + (__ffs(mm) - 1);
          next_row = __shfl_sync(0xffffffffu, resume, src);
          cnt = cap;
        }
      }
      __syncwarp();
      const int ns = cnt * G;
#pragma unroll 1
      for (int q = 0; q < NS / 32; ++q) {
        const int n2 = lane + 32 * q;
        const bool live = n2 < ns;
        const int i = live ? M.rowtok[n2 / G] : 0;
        const int hq = hk * G + (n2 % G);
        const int64_t rg = rb + i;
        int kcut = 0, klo = 0, j = 0;
        float bias2 = 0.0f;
        int64_t qoff = 0, poff = -1;
        if (live) {
          const int lstart = pos0 + i - a.local_window + 1;
          kcut = min(min(lstart, kvl) - b * BS, BS);
          const int seg = a.seg_start ? a.seg_start[rg] : 0;
          klo = max(seg - b * BS, 0);
          // list position of the block: the row's list ascends with a -1 tail
          const int32_t* cl = p.cidx + ((int64_t)ih * p.n_rows + rg) * K;
          for (int j0 = 0; j0 < K; j0 += 16) {
            int v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = j0 + u < K ? cl[j0 + u] : -1;
#pragma unroll
            for (int u = 0; u < 16; ++u) j += (v[u] >= 0 && v[u] < b) ? 1 : 0;
          }
          if (a.routes.bias) bias2 = p.cbias[((int64_t)ih * p.n_rows + rg) * K + j] * LOG2E;
          qoff = (a.seqs.q_start ? rg * a.qo.q_stride_tok
                                 : (int64_t)s * a.qo.q_stride_seq + (int64_t)i * a.qo.q_stride_tok) +
                 (int64_t)hq * a.qo.q_stride_head;
          poff = ((((int64_t)sl * p.prows + (i - i_lo)) * p.hqn + (hq - p.hq0)) * K) + j;
        }
        M.qoff[n2] = qoff;
        M.poff[n2] = poff;
        M.bias2[n2] = bias2;
        M.klo[n2] = klo;
        M.kcut[n2] = kcut;
      }
      if (lane == 0) M.ns = ns;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_full + buf);
      if (ns == 0) break;
    }
    // never leave the CTA with bulk copies in flight
    if (kv_issued) {
      volatile int no_abort = 0;
      mbar_wait(kv_full, 0, &no_abort, nullptr, 92);
    }
  } else if (warp == kMmaWarp) {
    // ============================ MMA issuer ============================
    if (lane == 0) {
      constexpr uint32_t fmt = DType<T>::fmt;
      constexpr uint32_t idesc_qk = make_idesc(fmt, 0, 0, NS, BS);
      constexpr uint32_t idesc_pv = make_idesc(fmt, 0, 1, NS, HD);
      const uint32_t sQ = smem_u32(sm + L::OFF_Q), sK = smem_u32(sm + L::OFF_K), sV = smem_u32(sm + L::OFF_V);
      bool alive = mbar_wait(kv_full, 0, abort_flag, derr, 93);
      for (int n = 0; alive; ++n) {
        if (!mbar_wait(q_full, n & 1, abort_flag, derr, 94)) break;
        tc_fence_after();
        if (meta[n & 1].ns == 0) break;
        // S(n) overwrites P(n-1), read by PV(n-1): this thread issued that PV
        // first, and its tcgen05.mma ops execute in issue order
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = sw128_desc(sQ + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sK + (kk >> 2) * (BS * 128) + (kk & 3) * 32, 16, 1024);
          umma_ss(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!mbar_wait(p_full, n & 1, abort_flag, derr, 95)) break;
        if (n >= 1 && !mbar_wait(o_free, (n - 1) & 1, abort_flag, derr, 96)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BS / 16; ++kk) {
          const uint64_t bd = sw128_desc(sV + kk * 2048, BS * 128, 1024);
          umma_ts(tO, tS + kk * 8, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(o_full);
      }
      // every MMA completes before TMEM is released
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, nullptr, 97);
    }
    __syncwarp();
  } else {
    // ============ slot warps: gather, softmax, epilogue (thread = slot) ============
    const int n_slot = tid;                        // 0..127, TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sl2 = a.scale * LOG2E;
    const T* qbase = reinterpret_cast<const T*>(a.qo.q);
    uint8_t* sQ = sm + L::OFF_Q;
    auto gather = [&](const RMeta& M, int ns) {
      const bool live = n_slot < ns;
      const uint4* src = reinterpret_cast<const uint4*>(qbase + (live ? M.qoff[n_slot] : 0));
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        const int region = cc >> 3, c8 = cc & 7;
        uint8_t* dst = sQ + region * 16384 + n_slot * 128 + ((c8 ^ (n_slot & 7)) << 4);
        if (live) cp_async16(dst, src + cc);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
      cp_async_wait_all_r();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    };
    bool alive = mbar_wait_warp(kv_full, 0, abort_flag, derr, 100);
    // zero V rows past the end of the sequence (P is 0 there, never times garbage)
    if (alive && (b + 1) * BS > kvl) {
      const int r0 = kvl - b * BS;
      uint8_t* dV = sm + L::OFF_V;
      for (int e = n_slot; e < (BS - r0) * 16; e += NS) {
        const int row = r0 + e / 16, ch = e % 16;
        *reinterpret_cast<uint4*>(dV + (ch >> 3) * (BS * 128) + row * 128 + ((ch & 7) << 4)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    int ns_cur = 0;
    if (alive) {
      alive = mbar_wait_warp(meta_full + 0, 0, abort_flag, derr, 101);
      if (alive) {
        ns_cur = meta[0].ns;
        gather(meta[0], ns_cur);
      }
    }
    for (int n = 0; alive && ns_cur > 0; ++n) {
      const RMeta& M = meta[n & 1];
      const int klo = M.klo[n_slot], kcut = M.kcut[n_slot];
      const float bias2 = M.bias2[n_slot];
      // ---- softmax of slot n_slot over the block's keys ----
      if (!mbar_wait_warp(s_full, n & 1, abort_flag, derr, 102)) { alive = false; break; }
      tc_fence_after();
      // pass 1: the row max over the kept keys; pass 2: P (packed) over the
      // S columns already read (64 S columns per 32-column store)
      float mrow = -INFINITY, lrow = 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < BS; c0 += 32) {
        float x[32];
        tmem_ld32f(tS + c0 + lane_base, x);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c0 + c >= klo && c0 + c < kcut) mrow = fmaxf(mrow, fmaf(x[c], sl2, bias2));
      }
      const float mref = mrow == -INFINITY ? 0.0f : mrow;
#pragma unroll 1
      for (int sc = 0; sc < (BS + 63) / 64; ++sc) {
        uint32_t pk[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c0 = sc * 64 + h * 32;
          if (c0 < BS) {
            float x[32];
            tmem_ld32f(tS + c0 + lane_base, x);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int c = c0 + 2 * e;
              const float p0 = (c >= klo && c < kcut) ? fast_exp2(fmaf(x[2 * e], sl2, bias2) - mref) : 0.0f;
              const float p1 = (c + 1 >= klo && c + 1 < kcut) ? fast_exp2(fmaf(x[2 * e + 1], sl2, bias2) - mref) : 0.0f;
              lrow += p0 + p1;
              pk[h * 16 + e] = pack2(p0, p1, (T*)nullptr);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[h * 16 + e] = 0u;
          }
        }
        tmem_st32(tS + sc * 32 + lane_base, pk);
      }
      tmem_st_wait();
      mrow = mref;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // ---- the next batch's q rows, gathered while PV(n) runs ----
      int ns_next = 0;
      if (!mbar_wait_warp(meta_full + ((n + 1) & 1), ((n + 1) >> 1) & 1, abort_flag, derr, 103)) { alive = false; break; }
      ns_next = meta[(n + 1) & 1].ns;
      gather(meta[(n + 1) & 1], ns_next);
      // ---- epilogue: normalised partial output and its log2-sum-exp ----
      if (!mbar_wait_warp(o_full, n & 1, abort_flag, derr, 104)) { alive = false; break; }
      tc_fence_after();
      const int64_t poff = M.poff[n_slot];
      const float inv_l = lrow > 0.0f ? 1.0f / lrow : 0.0f;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        float o[32];
        tmem_ld32f(tO + q4 * 32 + lane_base, o);
        tmem_ld_wait();
        if (poff >= 0) {
          uint32_t pko[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) pko[c >> 1] = pack2(o[c] * inv_l, o[c + 1] * inv_l, (T*)nullptr);
          uint4* dst = reinterpret_cast<uint4*>(const_cast<uint16_t*>(p.part_o) + poff * HD + q4 * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pko[4 * v], pko[4 * v + 1], pko[4 * v + 2], pko[4 * v + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      if (poff >= 0) const_cast<float*>(p.part_lse)[poff] = lrow > 0.0f ? mrow + log2f(lrow) : -INFINITY;
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_empty + (n & 1));
      ns_cur = ns_next;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename T, bool PAGED, int BS>
static int launch_routed_typed(const DashPrefillArgs& c, const PrefillPlan& p, const CUtensorMap& mk,
                               const CUtensorMap& mv, int hcn, cudaStream_t st) {
  auto kern = prefill_routed_kernel<T, PAGED, BS>;
  constexpr int smem = RLayout<BS>::SMEM;
  static_assert(smem <= 232448, "shared memory budget");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "cudaFuncSetAttribute(prefill_routed_kernel) failed");
  dim3 grid((unsigned)(p.sn * p.nblk_cap), (unsigned)hcn);
  kern<<<grid, kThreads, smem, st>>>(mk, mv, c, p);
  count_launch();
  return check_launch("prefill_routed_kernel");
}

int launch_prefill_routed(const DashPrefillArgs& c, const PrefillPlan& p, const CUtensorMap& mk,
                          const CUtensorMap& mv, int hcn, cudaStream_t st) {
  const bool paged = c.kv.block_table != nullptr;
  const bool bf = c.kv.dtype == DASH_DTYPE_BF16;
#define DASH_ROUTED(TT, PG, B) return launch_routed_typed<TT, PG, B>(c, p, mk, mv, hcn, st)
  switch (c.block_size) {
    case 32:
      if (bf) { if (paged) DASH_ROUTED(__nv_bfloat16, true, 32); DASH_ROUTED(__nv_bfloat16, false, 32); }
      if (paged) DASH_ROUTED(__half, true, 32); DASH_ROUTED(__half, false, 32);
    case 64:
      if (bf) { if (paged) DASH_ROUTED(__nv_bfloat16, true, 64); DASH_ROUTED(__nv_bfloat16, false, 64); }
      if (paged) DASH_ROUTED(__half, true, 64); DASH_ROUTED(__half, false, 64);
    case 128:
      if (bf) { if (paged) DASH_ROUTED(__nv_bfloat16, true, 128); DASH_ROUTED(__nv_bfloat16, false, 128); }
      if (paged) DASH_ROUTED(__half, true, 128); DASH_ROUTED(__half, false, 128);
    default:
      return set_error(DASH_ERR_UNSUPPORTED, "routed kernel: block_size %d", c.block_size);
  }
#undef DASH_ROUTED
}

}  // namespace dash
