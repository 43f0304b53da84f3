// dash_prefill_routed.cu -- the routed part of the DASH prefill, gathered by
// key block (sm_100a tensor cores), and the merge of a row's partials.
//
// With noise-like routes, the 128 rows of a query tile route different blocks
// and the tile-major kernel (dash_prefill.cu) multiplies every row against the
// union of their blocks: ~4x the useful work at BASELINE config 2 and ~7x at
// config 4.  Here the routed keys are taken block by block instead: one CTA
// per (sequence, kv head, key block) gathers the query rows that routed the
// block (the plan kernel's per-block row bitmask) into 128-slot batches (a
// slot = a row x one query head of the kv head), so every product is useful.
// The block's K and V (TMA) stay in shared memory for all its batches.
//
//   enumerator (warp 5)     K/V of the block; the next batch's rows from the
//                           bitmask into a 3-stage ring
//   loaders (warps 6-13)    two groups, even / odd batches; thread = slot:
//                           q row gathered into the stage (cp.async, 128-byte
//                           swizzle), the slot's key range and partial entry
//                           (list position of the block: one vector load of
//                           the row's ascending list)
//   MMA issuer (warp 4)     S = Q K^T (tcgen05 M=128, N=block, two TMEM S
//                           buffers), O = P V (P from TMEM, two O buffers);
//                           QK of batch n+2 is issued right after PV of n
//   softmax (warps 0-3)     thread = slot = TMEM lane: softmax of batch n over
//                           the block's keys below the row's window, P over S;
//                           then the epilogue of batch n-1: normalised partial
//                           output (bf16/fp16) and its log2-sum-exp
// The block's bias of a row is constant over the block, so it only shifts the
// partial's log-sum-exp: the merge adds it.
//
//   prefill_merge_kernel    one warp per (row, query head): the row's routed
//                           partials and its window part (slot K, written by
//                           the window kernel) merged with softmax weights
//                           2^(lse_j + bias_j log2 e - max); coalesced 256-byte
//                           partial rows; output (and peer copies) + lse
//
// Semantics: sparse_gather_e2e_triton.py:34-115 (keys of a routed block below
// the query's local window, + the slot's bias), WHL attend_triton.py:88-292.
#include <cudaTypedefs.h>
#include <climits>
#include <cstring>
#include "dash_common.cuh"
#include "dash_internal.h"
#include "dash_prefill_plan.cuh"

namespace dash {
namespace {

constexpr int NS = 128;                  // slots per batch
constexpr int HD = 128;                  // head dim
constexpr int kMmaWarp = 4;
constexpr int kEnumWarp = 5;
constexpr int kLoadWarp0 = 6;            // loader groups: warps 6-9, 10-13
constexpr int kThreads = 14 * 32;
constexpr uint32_t TMEM_COLS = 512;      // S0 | S1 | O0 | O1
constexpr float LOG2E = 1.4426950408889634f;

struct RStage {
  int rowtok[NS];      // token (within the sequence) of gathered row r (slots r*G+g)
  int64_t poff[NS];    // partial entry of the slot; -1: padding
  int klo[NS];         // keys [klo, kcut) of the block count for the slot
  int kcut[NS];
  int ns;              // live slots; 0: no more batches
  int s, b, hk;        // the batch's item: sequence, key block, kv head
  int buf, kvpar;      // its K/V buffer and the parity of that buffer's load
  int item;            // item ordinal within the CTA (a change marks the next item)
  int pad;
};

template <int BS>
struct RLayout {
  // batch stages: three, two with 128-token blocks (their K/V buffers are
  // twice as large)
  static constexpr int NQS = BS == 128 ? 2 : 3;
  static constexpr int OFF_Q = 0;                           // NQS x 2 halves x [128 slots][128 B]
  static constexpr int OFF_KV = NQS * 32768;                // 2 buffers x (K, V: 2 halves x [BS][128 B])
  static constexpr int OFF_ST = OFF_KV + 2 * BS * 512;      // NQS x RStage
  static constexpr int OFF_BAR = OFF_ST + NQS * (int)sizeof(RStage);
  // epilogue staging: one 64-column half of the batch's partial rows
  static constexpr int OFF_OSTG = OFF_BAR + 256;             // [128 slots][128 B]
  static constexpr int USED = OFF_OSTG + 16384 + 1024;
  // one CTA per SM: it takes all 512 TMEM columns
  static constexpr int SMEM = USED > 120 * 1024 ? USED : 120 * 1024;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Bytes the current phase of an mbarrier waits for, without an arrival.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all_r() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

}  // namespace

template <typename T, bool PAGED, int BS>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_routed_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmQ, const DashPrefillArgs a, const PrefillPlan p,
                          const int hcn, const int qmap) {
  using L = RLayout<BS>;
  constexpr int NQS = L::NQS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  RStage* stg = reinterpret_cast<RStage*>(sm + L::OFF_ST);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* rows_full = bars + 0;       // [NQS] enumerator -> loaders, MMA, softmax
  uint64_t* q_full = bars + 3;          // [NQS] loader group (4 warps) -> MMA
  uint64_t* stage_free = bars + 6;      // [NQS] QK done (commit) + slot data read (4 softmax warps)
  uint64_t* kv_ready = bars + 9;        // [2] K/V buffer loaded (and its tail zeroed)
  uint64_t* kv_tail = bars + 11;        // [2] load of a sequence's last block (zeroed after)
  uint64_t* kv_free = bars + 13;        // [2] every PV of the buffer's item issued + done
  uint64_t* s_full = bars + 15;         // [2]
  uint64_t* p_full = bars + 17;         // [2]
  uint64_t* o_full = bars + 19;         // [2]
  uint64_t* o_free = bars + 21;         // [2]
  uint64_t* mma_done = bars + 23;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = p.sn * p.nblk_cap * hcn;
  const int G = p.G, H = a.qo.n_heads, K = a.routes.K;
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const int i_lo = 2 * p.pj0 * p.TT;       // a multiple of 64
  DeviceError* derr = a.device_error;
  if (tid == 0) {
    for (int k = 0; k < NQS; ++k) {
      mbar_init(rows_full + k, 1);
      mbar_init(q_full + k, 4);
      mbar_init(stage_free + k, 1 + 4);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(kv_ready + k, 1);
      mbar_init(kv_tail + k, 1);
      mbar_init(kv_free + k, 1);
      mbar_init(s_full + k, 1);
      mbar_init(p_full + k, 4);
      mbar_init(o_full + k, 1);
      mbar_init(o_free + k, 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == kMmaWarp) { tmem_alloc(tmem_holder, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // TMEM columns: S buffer k at k*BS, O buffer k at 2*BS + k*128
  auto tS_of = [&](int k) -> uint32_t { return tmem + (uint32_t)(k * BS); };
  auto tO_of = [&](int k) -> uint32_t { return tmem + (uint32_t)(2 * BS + k * 128); };
  auto sK_of = [&](int buf) -> uint8_t* { return sm + L::OFF_KV + buf * (BS * 512); };
  auto sV_of = [&](int buf) -> uint8_t* { return sm + L::OFF_KV + buf * (BS * 512) + BS * 256; };
  auto kv_head_of = [&](int hk) -> int { return (hk * G) / (H / nih); };

  if (warp == kEnumWarp) {
    // ===== enumerator: items (sequence, key block, kv head) round robin over the
    // grid; per item its K/V into a buffer, then its rows in batches =====
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
    }
    const int cap = NS / G;
    int n = 0;                               // batches published
    int uses[2] = {0, 0}, tail_uses[2] = {0, 0};
    uint64_t* last_bar[2] = {nullptr, nullptr};
    uint32_t last_par[2] = {0u, 0u};
    int item_no = 0;
    bool alive = true;
    for (int it = blockIdx.x; alive && it < n_items; it += gridDim.x) {
      const int hk = p.hk0 + it % hcn;
      const int r = it / hcn;
      const int b = r % p.nblk_cap, sl = r / p.nblk_cap;
      const int s = p.s0 + sl;
      const int kvl = kv_len_of(a.seqs, s);
      if ((int64_t)b * BS >= kvl) continue;
      const int i_hi = min(q_len_of(a.seqs, s), 2 * (p.pj0 + p.npj) * p.TT);
      if (i_lo >= i_hi) continue;
      const int w_hi = (i_hi + 31) >> 5;
      const uint32_t* fl =
          p.flags + (((int64_t)kv_head_of(hk) * a.seqs.n_seq + s) * p.nblk_cap + b) * p.wps;
      // flag words of the chunk in windows of 32 (one per lane), the next
      // window prefetched; flag bits past qlen are zero
      int wb = i_lo >> 5;
      uint32_t mc = wb + lane < w_hi ? fl[wb + lane] : 0u;
      uint32_t mn = wb + 32 + lane < w_hi ? fl[wb + 32 + lane] : 0u;
      while (!__any_sync(0xffffffffu, mc != 0u) && wb + 32 < w_hi) {
        wb += 32;
        mc = mn;
        mn = wb + 32 + lane < w_hi ? fl[wb + 32 + lane] : 0u;
      }
      if (!__any_sync(0xffffffffu, mc != 0u)) continue;      // no row routed the block
      const int buf = item_no & 1;
      // the buffer's previous item: every PV issued and complete
      if (uses[buf] >= 1 && !mbar_wait_warp(kv_free + buf, (uint32_t)(uses[buf] - 1) & 1u, abort_flag, derr, 90)) {
        alive = false;
        break;
      }
      const bool tail = (int64_t)(b + 1) * BS > kvl;
      uint64_t* lbar = tail ? kv_tail + buf : kv_ready + buf;
      if (lane == 0) {
        constexpr int R = BS < 64 ? BS : 64;          // rows per TMA box
        int c1 = b * BS, c3 = s;
        bool ok = true;
        if (PAGED) {
          const int64_t page = a.kv.block_table[(int64_t)s * a.kv.bt_stride + b];
          if (page < 0 || page >= a.kv.num_pages) {
            record_error(derr, DASH_DEV_BAD_PAGE, 91, page);
            ok = false;
          }
          c1 = 0;
          c3 = (int)page;
        }
        if (ok) {
          mbar_arrive_expect_tx(lbar, 2 * BS * 256);
#pragma unroll
          for (int dh = 0; dh < 2; ++dh)
#pragma unroll
            for (int r0 = 0; r0 < BS; r0 += R) {
              tma_load_4d(sK_of(buf) + dh * BS * 128 + r0 * 128, &tmK, lbar, dh * 64, c1 + r0, hk, c3);
              tma_load_4d(sV_of(buf) + dh * BS * 128 + r0 * 128, &tmV, lbar, dh * 64, c1 + r0, hk, c3);
            }
        } else {
          mbar_arrive(lbar);
        }
      }
      const int kvpar = uses[buf] & 1;
      last_bar[buf] = lbar;
      last_par[buf] = (uint32_t)(tail ? tail_uses[buf] : uses[buf]) & 1u;
      ++uses[buf];
      if (tail) {
        // V rows past the end of the sequence are zeroed before any PV reads
        // them (P is 0 there, never times garbage)
        if (!mbar_wait_warp(kv_tail + buf, (uint32_t)tail_uses[buf] & 1u, abort_flag, derr, 92)) {
          alive = false;
          break;
        }
        ++tail_uses[buf];
        const int r0 = kvl - b * BS;
        uint8_t* dV = sV_of(buf);
        for (int e = lane; e < (BS - r0) * 16; e += 32) {
          const int row = r0 + e / 16, ch = e % 16;
          *reinterpret_cast<uint4*>(dV + (ch >> 3) * (BS * 128) + row * 128 + ((ch & 7) << 4)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(kv_ready + buf);
      }
      // the item's batches
      while (alive) {
        const int st = n % NQS;
        RStage& S = stg[st];
        // (a stage reserved for a batch that turns out empty is reused by the
        // next one: the completed wait passes again)
        if (n >= NQS && !mbar_wait_warp(stage_free + st, (uint32_t)((n / NQS) - 1) & 1u, abort_flag, derr, 93)) {
          alive = false;
          break;
        }
        int cnt = 0;
        bool exhausted = false;
        while (cnt < cap) {
          if (!__any_sync(0xffffffffu, mc != 0u)) {
            if (wb + 32 >= w_hi) { exhausted = true; break; }
            wb += 32;
            mc = mn;
            mn = wb + 32 + lane < w_hi ? fl[wb + 32 + lane] : 0u;
            continue;
          }
          const int c = __popc(mc);
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
          for (int k = 0; k < take; ++k) {
            const int bit = __ffs(mc) - 1;
            mc &= mc - 1u;
            S.rowtok[cnt + excl + k] = (wb + lane) * 32 + bit;
          }
          cnt += min(tot, room);
        }
        if (cnt > 0) {
          if (lane == 0) {
            S.ns = cnt * G;
            S.s = s;
            S.b = b;
            S.hk = hk;
            S.buf = buf;
            S.kvpar = kvpar;
            S.item = item_no;
          }
          __threadfence_block();
          __syncwarp();
          if (lane == 0) mbar_arrive(rows_full + st);
          ++n;
        }
        if (exhausted) break;
      }
      ++item_no;
    }
    // two empty batches end both loader groups, the MMA warp and the softmax
    for (int z = 0; z < 2 && alive; ++z, ++n) {
      const int st = n % NQS;
      if (n >= NQS && !mbar_wait_warp(stage_free + st, (uint32_t)((n / NQS) - 1) & 1u, abort_flag, derr, 94)) break;
      if (lane == 0) stg[st].ns = 0;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(rows_full + st);
    }
    // never leave the CTA with bulk copies in flight
    for (int k = 0; k < 2; ++k) {
      if (last_bar[k] != nullptr) {
        volatile int no_abort = 0;
        mbar_wait(last_bar[k], last_par[k], &no_abort, nullptr, 95);
      }
    }
  } else if (warp == kMmaWarp) {
    // ============================ MMA issuer ============================
    if (lane == 0) {
      constexpr uint32_t fmt = DType<T>::fmt;
      constexpr uint32_t idesc_qk = make_idesc(fmt, 0, 0, NS, BS);
      constexpr uint32_t idesc_pv = make_idesc(fmt, 0, 1, NS, HD);
      bool alive = true;
      int nq = 0;               // QKs issued (batches 0 .. nq-1 exist)
      bool more = true;
      // K/V buffer and item of batches n and n + 1 (QK'd, PV pending): taken
      // at QK time, since the stage may be reused once the softmax has read it
      int qk_buf[2] = {0, 0}, qk_item[2] = {-1, -1};
      // QK(n) into S buffer n % 2.  That buffer held P(n-2), read by PV(n-2):
      // this thread issued PV(n-2) before, and its tcgen05.mma ops execute in
      // issue order; softmax finished with S(n-2) before PV(n-2) was issued.
      auto try_qk = [&]() {
        if (!more) return;
        const int n = nq, st = n % NQS;
        const uint32_t par = (uint32_t)(n / NQS) & 1u;
        if (!mbar_wait(rows_full + st, par, abort_flag, derr, 96)) { more = false; alive = false; return; }
        const RStage& S = stg[st];
        if (S.ns == 0) { more = false; return; }
        qk_buf[n & 1] = S.buf;
        qk_item[n & 1] = S.item;
        if (!mbar_wait(q_full + st, par, abort_flag, derr, 97) ||
            !mbar_wait(kv_ready + S.buf, (uint32_t)S.kvpar, abort_flag, derr, 98)) {
          more = false;
          alive = false;
          return;
        }
        tc_fence_after();
        const uint32_t sQ = smem_u32(sm + L::OFF_Q + st * 32768);
        const uint32_t sK = smem_u32(sK_of(S.buf));
        const uint32_t tS = tS_of(n & 1);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t ad = sw128_desc(sQ + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sK + (kk >> 2) * (BS * 128) + (kk & 3) * 32, 16, 1024);
          umma_ss(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full + (n & 1));
        umma_commit(stage_free + st);           // the q rows of the stage are read
        ++nq;
      };
      try_qk();
      try_qk();
      for (int n = 0; n < nq && alive; ++n) {
        if (!mbar_wait(p_full + (n & 1), (uint32_t)(n >> 1) & 1u, abort_flag, derr, 99)) break;
        if (n >= 2 && !mbar_wait(o_free + (n & 1), (uint32_t)((n - 2) >> 1) & 1u, abort_flag, derr, 100)) break;
        tc_fence_after();
        const int buf = qk_buf[n & 1];
        const uint32_t sV = smem_u32(sV_of(buf));
        const uint32_t tS = tS_of(n & 1), tO = tO_of(n & 1);
#pragma unroll
        for (int kk = 0; kk < BS / 16; ++kk) {
          const uint64_t bd = sw128_desc(sV + kk * 2048, BS * 128, 1024);
          umma_ts(tO, tS + kk * 8, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(o_full + (n & 1));
        // the last PV of an item frees its K/V buffer for the item after next
        // (batch n+1 is known: its QK was issued before this PV)
        if (n + 1 < nq && qk_item[(n + 1) & 1] != qk_item[n & 1]) umma_commit(kv_free + buf);
        try_qk();
      }
      // every MMA completes before TMEM is released
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort, nullptr, 101);
    }
    __syncwarp();
  } else if (warp >= kLoadWarp0) {
    // ============ loaders: q rows and slot data of every other batch ============
    const int grp = (warp - kLoadWarp0) >> 2;
    const int n2 = tid - (kLoadWarp0 + 4 * grp) * 32;        // slot 0..127
    const T* qbase = reinterpret_cast<const T*>(a.qo.q);
    const bool vec = (K & 3) == 0;
    int last_n = -1;                  // the last batch this group gathered rows for
    for (int n = grp;; n += 2) {
      const int st = n % NQS;
      if (!mbar_wait_warp(rows_full + st, (uint32_t)(n / NQS) & 1u, abort_flag, derr, 102)) break;
      RStage& S = stg[st];
      const int ns = S.ns;
      if (ns == 0) break;
      const int s = S.s, b = S.b, hk = S.hk;
      const bool live = n2 < ns;
      const int i = live ? S.rowtok[n2 / G] : i_lo;
      const int hq = hk * G + (n2 % G);
      const int64_t rg = row_base(a.seqs, s) + i;
      // q row -> stage (swizzled K-major)
      {
        const int64_t qoff = (a.seqs.q_start ? rg * a.qo.q_stride_tok
                                             : (int64_t)s * a.qo.q_stride_seq + (int64_t)i * a.qo.q_stride_tok) +
                             (int64_t)hq * a.qo.q_stride_head;
        uint8_t* sQ = sm + L::OFF_Q + st * 32768;
        if (qmap) {
          // TMA row gather: 4 slots x 64 columns per instruction into the
          // swizzled halves, 16 instructions for the warp's 32 slots (lanes
          // 0-15), instead of 512 lane copies through the load/store unit.
          // q rows are whole 128-element rows of the map (the host checked
          // the strides); a padding slot takes row 0 (its P is masked to 0
          // and it writes no partial).
          const int wq = n2 >> 5;
          const int row = live ? (int)(qoff >> 7) : 0;
          const int quad = lane >> 1, h = lane & 1;
          const int r0 = __shfl_sync(0xffffffffu, row, 4 * quad), r1 = __shfl_sync(0xffffffffu, row, 4 * quad + 1);
          const int r2 = __shfl_sync(0xffffffffu, row, 4 * quad + 2), r3 = __shfl_sync(0xffffffffu, row, 4 * quad + 3);
          if (lane == 0) mbar_expect_tx(q_full + st, 32 * 256);
          __syncwarp();
          if (lane < 16)
            tma_gather4(sQ + h * 16384 + (wq * 32 + 4 * quad) * 128, &tmQ, q_full + st, h * 64, r0, r1, r2, r3);
        } else {
          // padding slots are zero
          const uint4* src = reinterpret_cast<const uint4*>(qbase + qoff);
#pragma unroll
          for (int cc = 0; cc < 16; ++cc) {
            uint8_t* dst = sQ + (cc >> 3) * 16384 + n2 * 128 + (((cc & 7) ^ (n2 & 7)) << 4);
            if (live) cp_async16(dst, src + cc);
            else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      // key range and partial entry (list position of the block: the row's
      // canonical list ascends with a -1 tail)
      int64_t poff = -1;
      int klo = 0, kcut = 0;
      if (live) {
        const int kvl = kv_len_of(a.seqs, s);
        const int lstart = pos0_of(a.seqs, s) + i - a.local_window + 1;
        kcut = min(min(lstart, kvl) - b * BS, BS);
        const int seg = a.seg_start ? a.seg_start[rg] : 0;
        klo = max(seg - b * BS, 0);
        const int32_t* cl = p.cidx + ((int64_t)kv_head_of(hk) * p.n_rows + rg) * K;
        int j = 0;
        if (vec) {
          for (int j0 = 0; j0 < K; j0 += 16) {
            int4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              v[u] = j0 + 4 * u < K ? reinterpret_cast<const int4*>(cl + j0)[u] : make_int4(-1, -1, -1, -1);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              j += (v[u].x >= 0 && v[u].x < b) + (v[u].y >= 0 && v[u].y < b) + (v[u].z >= 0 && v[u].z < b) +
                   (v[u].w >= 0 && v[u].w < b);
          }
        } else {
          for (int j0 = 0; j0 < K; j0 += 16) {
            int v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = j0 + u < K ? cl[j0 + u] : -1;
#pragma unroll
            for (int u = 0; u < 16; ++u) j += (v[u] >= 0 && v[u] < b) ? 1 : 0;
          }
        }
        const int sl = s - p.s0;
        poff = (((int64_t)sl * p.prows + (i - i_lo)) * p.hqn + (hq - p.hq0)) * (K + 1) + j;
      }
      S.poff[n2] = poff;
      S.klo[n2] = klo;
      S.kcut[n2] = kcut;
      if (!qmap) {
        cp_async_wait_all_r();
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full + st);
      last_n = n;
    }
    // never leave the CTA with row gathers in flight: the last batch's rows
    // have landed (its MMA waited for them, unless the CTA gave up early)
    if (qmap && last_n >= 0 && lane == 0) {
      volatile int no_abort = 0;
      mbar_wait(q_full + last_n % NQS, (uint32_t)(last_n / NQS) & 1u, &no_abort, nullptr, 108);
    }
    __syncwarp();
  } else {
    // ======== softmax of batch n, then the epilogue of batch n-1 (thread = slot) ========
    const int n2 = tid;                             // 0..127, TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float sl2 = a.scale * LOG2E;
    bool alive = true;
    // the batch whose epilogue is pending: its partial entry, max and sum
    int64_t prev_poff = -1;
    float prev_m = 0.0f, prev_l = 0.0f;
    uint8_t* ostg = sm + L::OFF_OSTG;
    auto epilogue = [&](int m) -> bool {
      if (!mbar_wait_warp(o_full + (m & 1), (uint32_t)(m >> 1) & 1u, abort_flag, derr, 103)) return false;
      tc_fence_after();
      const uint32_t tO = tO_of(m & 1);
      const float inv_l = prev_l > 0.0f ? 1.0f / prev_l : 0.0f;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float o[64];
        tmem_ld32f(tO + h * 64 + lane_base, o);
        tmem_ld32f(tO + h * 64 + 32 + lane_base, o + 32);
        tmem_ld_wait();
        // the half-row goes through shared memory (16-byte chunk c of slot
        // n2 at ((c ^ (n2 & 7)) << 4)), then the warp writes its 32 slots'
        // half-rows four per instruction (8 lanes x 16 bytes each) instead
        // of 32 scattered 16-byte pieces
        uint32_t pko[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) pko[c >> 1] = pack2(o[c] * inv_l, o[c + 1] * inv_l, (T*)nullptr);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          *reinterpret_cast<uint4*>(ostg + n2 * 128 + ((v ^ (n2 & 7)) << 4)) =
              make_uint4(pko[4 * v], pko[4 * v + 1], pko[4 * v + 2], pko[4 * v + 3]);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int rr = 4 * j + (lane >> 3), cc = lane & 7;
          const int64_t off = __shfl_sync(0xffffffffu, prev_poff, rr);
          const int mr = warp * 32 + rr;
          const uint4 val = *reinterpret_cast<const uint4*>(ostg + mr * 128 + ((cc ^ (mr & 7)) << 4));
          if (off >= 0)
            *reinterpret_cast<uint4*>(const_cast<uint16_t*>(p.part_o) + off * HD + h * 64 + cc * 8) = val;
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free + (m & 1));
      if (prev_poff >= 0)
        const_cast<float*>(p.part_lse)[prev_poff] = prev_l > 0.0f ? prev_m + log2f(prev_l) : -INFINITY;
      return true;
    };
    int n = 0;
    for (; alive; ++n) {
      const int st = n % NQS;
      const uint32_t par = (uint32_t)(n / NQS) & 1u;
      if (!mbar_wait_warp(rows_full + st, par, abort_flag, derr, 104)) { alive = false; break; }
      if (stg[st].ns == 0) break;
      // the loaders' slot data of this stage (complete once q_full is)
      if (!mbar_wait_warp(q_full + st, par, abort_flag, derr, 105)) { alive = false; break; }
      const RStage& S = stg[st];
      const int klo = S.klo[n2], kcut = S.kcut[n2];
      const int64_t poff = S.poff[n2];
      // the stage is free for the enumerator once every slot's data is read
      // (the epilogue works from registers)
      __syncwarp();
      if (lane == 0) mbar_arrive(stage_free + st);
      if (!mbar_wait_warp(s_full + (n & 1), (uint32_t)(n >> 1) & 1u, abort_flag, derr, 106)) { alive = false; break; }
      tc_fence_after();
      const uint32_t tS = tS_of(n & 1);
      // pass 1: the row max over the kept keys; pass 2: P (packed, 64 S
      // columns per 32-column store).  S is read 64 columns per wait; with
      // 64-key blocks pass 2 reuses the registers of pass 1.
      float mrow = -INFINITY, lrow = 0.0f;
      float x[64];
      // Slots that keep every key of the block (no window cut and no segment
      // start inside it; the scale is positive): the warp takes a mask-free
      // path, max(x) * scale (the same value: rounding is monotonic) and
      // packed f32x2 arithmetic for P.
      const bool full = __all_sync(0xffffffffu, klo <= 0 && kcut >= BS) && sl2 > 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < BS; c0 += 64) {
        tmem_ld32f(tS + c0 + lane_base, x);
        if (c0 + 32 < BS) tmem_ld32f(tS + c0 + 32 + lane_base, x + 32);
        tmem_ld_wait();
        if (full) {
          float mx = x[0];
#pragma unroll
          for (int c = 1; c < 64; ++c)
            if (c0 + c < BS) mx = fmaxf(mx, x[c]);
          mrow = fmaxf(mrow, mx * sl2);
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c0 + c < BS && c0 + c >= klo && c0 + c < kcut) mrow = fmaxf(mrow, x[c] * sl2);
        }
      }
      const float mref = mrow == -INFINITY ? 0.0f : mrow;
#pragma unroll 1
      for (int sc = 0; sc < (BS + 63) / 64; ++sc) {
        const int c0 = sc * 64;
        if (BS > 64) {
          tmem_ld32f(tS + c0 + lane_base, x);
          if (c0 + 32 < BS) tmem_ld32f(tS + c0 + 32 + lane_base, x + 32);
          tmem_ld_wait();
        }
        uint32_t pk[32];
        if (full) {
          const uint64_t sv = f2_pack(sl2, sl2), mv = f2_pack(-mref, -mref);
          uint64_t lsv = f2_pack(0.0f, 0.0f);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (c0 + 2 * e < BS) {
              float y0, y1;
              f2_unpack(ffma2(f2_pack(x[2 * e], x[2 * e + 1]), sv, mv), y0, y1);
              const float p0 = fast_exp2(y0), p1 = fast_exp2(y1);
              lsv = fadd2(lsv, f2_pack(p0, p1));
              pk[e] = pack2(p0, p1, (T*)nullptr);
            } else {
              pk[e] = 0u;
            }
          }
          float l0, l1;
          f2_unpack(lsv, l0, l1);
          lrow += l0 + l1;
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = c0 + 2 * e;
            const float p0 = (c < BS && c >= klo && c < kcut) ? fast_exp2(fmaf(x[2 * e], sl2, -mref)) : 0.0f;
            const float p1 = (c + 1 < BS && c + 1 >= klo && c + 1 < kcut) ? fast_exp2(fmaf(x[2 * e + 1], sl2, -mref)) : 0.0f;
            lrow += p0 + p1;
            pk[e] = pack2(p0, p1, (T*)nullptr);
          }
        }
        tmem_st32(tS + sc * 32 + lane_base, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + (n & 1));
      // ---- epilogue of the previous batch while PV(n) runs ----
      if (n >= 1 && !epilogue(n - 1)) { alive = false; break; }
      prev_poff = poff;
      prev_m = mref;
      prev_l = lrow;
    }
    if (alive && n >= 1) epilogue(n - 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// prefill_merge_kernel: one warp per (row, query head) of the chunk.  Slots:
// the row's routed partials j < npart (its canonical list ascends with a -1
// tail) and the window part at slot K.  Lane l owns dims [4l, 4l+4).
// ---------------------------------------------------------------------------
constexpr int kMergeWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kMergeWarps * 32)
    prefill_merge_kernel(const DashPrefillArgs a, const PrefillPlan p) {
  __shared__ float s_w[kMergeWarps][kPlanMaxSlots + 1];
  const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * kMergeWarps + wl;
  const int64_t per_seq = (int64_t)p.prows * p.hqn;
  if (wid >= (int64_t)p.sn * per_seq) return;
  const int sl = (int)(wid / per_seq);
  const int64_t rem = wid - sl * per_seq;
  const int il = (int)(rem / p.hqn), hl = (int)(rem - (int64_t)il * p.hqn);
  const int s = p.s0 + sl;
  const int i = 2 * p.pj0 * p.TT + il;
  if (i >= q_len_of(a.seqs, s)) return;
  const int hq = p.hq0 + hl;
  const int64_t rg = row_base(a.seqs, s) + i;
  const int H = a.qo.n_heads, K = a.routes.K;
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const int ih = hq / (H / nih);
  const int32_t* cl = p.cidx + ((int64_t)ih * p.n_rows + rg) * K;
  const float* cb = p.cbias + ((int64_t)ih * p.n_rows + rg) * K;
  const int64_t pbase = (((int64_t)sl * p.prows + il) * p.hqn + hl) * (K + 1);
  const bool has_bias = a.routes.bias != nullptr;
  // log2-domain weights of the slots: routed partial + its bias, window
  float lv[(kPlanMaxSlots + 1 + 31) / 32];
  int npart = 0;
  float mx = -INFINITY;
#pragma unroll
  for (int u = 0; u < (kPlanMaxSlots + 1 + 31) / 32; ++u) {
    const int j = lane + 32 * u;
    float v = -INFINITY;
    if (j < K) {
      if (cl[j] >= 0) {
        v = p.part_lse[pbase + j];
        if (has_bias) v += cb[j] * LOG2E;
        ++npart;
      }
    } else if (j == K) {
      v = p.part_lse[pbase + K];
    }
    lv[u] = v;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    npart += __shfl_xor_sync(0xffffffffu, npart, o);
  }
  // every key masked (all weights 0): keep the weights finite
  if (mx == -INFINITY) mx = 0.0f;
  float den = 0.0f;
#pragma unroll
  for (int u = 0; u < (kPlanMaxSlots + 1 + 31) / 32; ++u) {
    const int j = lane + 32 * u;
    if (j <= K) {
      const float w = exp2f(lv[u] - mx);
      s_w[wl][j] = w;
      den += w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  __syncwarp();
  // weighted sum over t = 0..npart (t < npart: routed slot t; t = npart: the
  // window slot K), eight 256-byte partial rows in flight per step
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const uint2* po = reinterpret_cast<const uint2*>(p.part_o);
  for (int t0 = 0; t0 <= npart; t0 += 8) {
    uint2 v[8];
    float w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = t0 + u;
      const int j = t < npart ? t : K;
      const bool ok = t <= npart;
      w[u] = ok ? s_w[wl][j] : 0.0f;
      v[u] = ok ? po[(pbase + j) * (HD / 4) + lane] : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float2 f0 = unpack2(v[u].x, (T*)nullptr), f1 = unpack2(v[u].y, (T*)nullptr);
      acc[0] = fmaf(w[u], f0.x, acc[0]);
      acc[1] = fmaf(w[u], f0.y, acc[1]);
      acc[2] = fmaf(w[u], f1.x, acc[2]);
      acc[3] = fmaf(w[u], f1.y, acc[3]);
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
  const uint2 ov = make_uint2(pack2(acc[0] * inv, acc[1] * inv, (T*)nullptr),
                              pack2(acc[2] * inv, acc[3] * inv, (T*)nullptr));
  const int64_t ooff = (a.seqs.q_start ? rg * a.qo.o_stride_tok
                                       : (int64_t)s * a.qo.o_stride_seq + (int64_t)i * a.qo.o_stride_tok) +
                       (int64_t)hq * a.qo.o_stride_head;
  T* op = reinterpret_cast<T*>(a.qo.out) + ooff;
  reinterpret_cast<uint2*>(op)[lane] = ov;
  // fused output gather: the same row into every peer rank's copy of the
  // output (posted P2P stores over NVLink; same strides, same offset)
  for (int pr = 0; pr < a.n_peers; ++pr)
    reinterpret_cast<uint2*>(reinterpret_cast<T*>(a.out_peers[pr]) + ooff)[lane] = ov;
  if (lane == 0 && a.qo.lse) {
    const float lse = den > 0.0f ? (mx + log2f(den)) * 0.6931471805599453f : -INFINITY;
    a.qo.lse[(a.seqs.q_start ? rg * a.qo.lse_stride_tok
                             : (int64_t)s * a.qo.lse_stride_seq + (int64_t)i * a.qo.lse_stride_tok) +
             (int64_t)hq * a.qo.lse_stride_head] = lse;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

static PFN_cuTensorMapEncodeTiled_v12000 routed_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// The queries as a 2-D tensor of 128-element rows for the TMA row gather:
// possible when every q stride is a whole number of rows (the [B, H, T, D],
// [B, T, H, D] and packed [T, H, D] layouts).  Returns false otherwise (the
// loaders then copy rows with cp.async).
static bool make_q_rows_map(CUtensorMap* map, const DashPrefillArgs& c) {
  auto enc = routed_encode_fn();
  const DashQO& qo = c.qo;
  if (!enc || (reinterpret_cast<uintptr_t>(qo.q) & 15) != 0) return false;
  const bool packed = c.seqs.q_start != nullptr;
  if (qo.q_stride_tok < 0 || qo.q_stride_head < 0 || qo.q_stride_tok % 128 || qo.q_stride_head % 128) return false;
  if (!packed && (qo.q_stride_seq < 0 || qo.q_stride_seq % 128)) return false;
  const int64_t rows_of_seq = packed ? (int64_t)c.seqs.q_len_fixed : (int64_t)c.seqs.max_q_len;
  if (rows_of_seq <= 0 || c.seqs.n_seq <= 0 || qo.n_heads <= 0) return false;
  const int64_t max_off = (packed ? 0 : (int64_t)(c.seqs.n_seq - 1) * qo.q_stride_seq) +
                          (rows_of_seq - 1) * qo.q_stride_tok + (int64_t)(qo.n_heads - 1) * qo.q_stride_head;
  const int64_t rows = max_off / 128 + 1;
  if (rows >= ((int64_t)1 << 31)) return false;
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, 1};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, c.kv.dtype == DASH_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(qo.q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, bool PAGED, int BS>
static int launch_routed_typed(const DashPrefillArgs& c, const PrefillPlan& p, const CUtensorMap& mk,
                               const CUtensorMap& mv, int hcn, cudaStream_t st) {
  CUtensorMap mq;
  memset(&mq, 0, sizeof(mq));
  const int qmap = make_q_rows_map(&mq, c) ? 1 : 0;
  auto kern = prefill_routed_kernel<T, PAGED, BS>;
  constexpr int smem = RLayout<BS>::SMEM;
  static_assert(smem <= 232448, "shared memory budget");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "cudaFuncSetAttribute(prefill_routed_kernel) failed");
  // persistent: one CTA per SM walks the (sequence, block, kv head) items
  const int64_t items = (int64_t)p.sn * p.nblk_cap * hcn;
  const unsigned grid = (unsigned)(items < sm_count() ? items : sm_count());
  kern<<<grid, kThreads, smem, st>>>(mk, mv, mq, c, p, hcn, qmap);
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

int launch_prefill_merge(const DashPrefillArgs& c, const PrefillPlan& p, cudaStream_t st) {
  const int64_t warps = (int64_t)p.sn * p.prows * p.hqn;
  const unsigned grid = (unsigned)((warps + kMergeWarps - 1) / kMergeWarps);
  if (c.kv.dtype == DASH_DTYPE_BF16) prefill_merge_kernel<__nv_bfloat16><<<grid, kMergeWarps * 32, 0, st>>>(c, p);
  else prefill_merge_kernel<__half><<<grid, kMergeWarps * 32, 0, st>>>(c, p);
  count_launch();
  return check_launch("prefill_merge_kernel");
}

}  // namespace dash
