// dash_backward_tc.cu -- training backward of the DASH gather attention on
// sm_100a tensor cores (bf16 / fp16 inputs, fp32 accumulation).
//
// Same semantics as the CUDA-core kernels of dash_backward.cu
// (sparse_gather_e2e_triton.py:118-262), key-tile major with gathered query
// rows, so no query row is multiplied against a block it did not route:
//
// Work unit: one CTA per (128-key tile, kv head, sequence).  The tile's rows
// are the query rows that routed one of its (at most four) blocks with a key
// below their local window (per-block row bitmask of bwd_flags_kernel) plus
// the rows whose window reaches a key of the tile.  They are processed in
// batches of 128 slots (a slot = a query row x one of the G query heads of
// this kv head):
//   producer warp 9  enumerates the next batch's rows and loads its per-slot
//                    lse / delta / routed flags / biases (double-buffered)
//   math warps 0-7   gather the slots' q and dout rows into shared memory
//                    (cp.async, 128-byte swizzle, K-major)
//   MMA warp 8       S^T  = K  Q^T        (M = 128 keys, N = 128 slots, K = d)
//                    dP^T = V  dO^T
//   math warps       thread = (key, slot half): P^T = exp(s*scale + bias - lse) on the kept
//                    keys, dS^T = P^T (dP^T - delta); P^T and dS^T (bf16)
//                    back into TMEM over S^T / dP^T, dS^T also into shared
//                    memory (MN-major); per-slot column sums of the remote
//                    dS^T (butterfly reduce-scatter) -> slot-bias gradient
//   MMA warp         dV += P^T dO,  dK += dS^T Q   (A from TMEM)
//                    dQ  = dS K                    (A and B MN-major, shared)
//   math warps       thread = slot: dQ rows from TMEM -> fp32 reductions
//                    (red.global.add.v4.f32, nothing returned)
// After the last batch dK (x scale) and dV leave TMEM, one row per thread.
// TMEM: S^T | dP^T | dV | dK, 128 columns each; after the softmax P^T and
// dS^T (packed bf16) take the S^T columns and dQ the dP^T columns.
// Every wait is bounded (abort flag + time limit, DASH_DEV_TIMEOUT).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <climits>
#include <cstring>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {
namespace {

constexpr int TK = 128;                  // keys per CTA
constexpr int NS = 128;                  // slots per batch
constexpr int kMath = 256;               // 8 math warps (two warpgroups)
constexpr int kMmaWarp = 8;
constexpr int kProdWarp = 9;
constexpr int kTcThreads = kMath + 64;   // + MMA warp + producer warp
constexpr int OFF_K = 0;                 // [2 halves][128 keys][128 B]
constexpr int OFF_V = 32768;
constexpr int OFF_Q = 65536;             // [2 halves][128 slots][128 B]
constexpr int OFF_DO = 98304;
constexpr int OFF_DS = 131072;           // dS^T MN-major: [2 slot halves][128 keys][128 B]
constexpr int OFF_META = 163840;
// A tile of 128 keys holds up to QB blocks (block sizes are multiples of 32,
// so every 32-key warp quarter lies in one block).
constexpr int QB = 4;
// Per-batch slot meta, double-buffered (the producer fills batch b+1 while
// batch b is computed): a = {pos, routed bits (one per tile block) | seg << 4,
// cloc, delta} and b = the remote logit offset of each tile block (read by
// the softmax), global row, query head, routed-list slot of each tile block.
struct SlotMeta {
  int4 a[NS];
  float4 b[NS];
  int row[NS];
  int hq[NS];
  int4 sl[NS];
  int ns;
  int pad[3];
};
constexpr int META_BYTES = 2 * (int)sizeof(SlotMeta) + 4 * NS * 4;   // + dsum [4][NS]
constexpr int OFF_BAR = (OFF_META + META_BYTES + 15) & ~15;
// dQ staging: per math warp, 32 slots x 32 fp32 (one quarter of a row)
constexpr int OFF_DQSTG = (OFF_BAR + 128 + 127) & ~127;   // [8 warps][32 slots][128 B]
constexpr int SMEM_TC = OFF_DQSTG + 8 * 4096 + 1024;       // + alignment slack
static_assert(SMEM_TC <= 232448, "shared memory budget");
constexpr uint32_t TMEM_COLS = 512;

template <typename E> struct Fmt;
template <> struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t v = 1;
  static __device__ __forceinline__ float tof(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};
template <> struct Fmt<__half> {
  static constexpr uint32_t v = 0;
  static __device__ __forceinline__ float tof(__half x) { return __half2float(x); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ void st(__half* p, float x) { *p = __float2half_rn(x); }
};

__device__ __forceinline__ void math_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// barrier of the 8 math warps that also ANDs a predicate over them: every
// math warp leaves a failed wait together (none is left at a later barrier)
__device__ __forceinline__ bool math_all(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 1, 256, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p)
      : "memory");
  return r != 0;
}

// one 256-byte row (128 x 16-bit) -> K-major 128-byte-swizzled buffer of 128 rows
__device__ __forceinline__ void st_row_sw128(uint8_t* buf, int row, const uint4* src, bool zero) {
#pragma unroll
  for (int cc = 0; cc < 16; ++cc) {
    const uint4 v = zero ? make_uint4(0, 0, 0, 0) : src[cc];
    const int region = cc >> 3, c8 = cc & 7;
    *reinterpret_cast<uint4*>(buf + region * 16384 + row * 128 + ((c8 ^ (row & 7)) << 4)) = v;
  }
}

// the same row copied with cp.async (no register staging); the caller waits
// with cp_async_wait_all() before handing the buffer to the tensor cores
__device__ __forceinline__ void cp_row_sw128(uint8_t* buf, int row, const uint4* src, bool zero) {
#pragma unroll
  for (int cc = 0; cc < 16; ++cc) {
    const int region = cc >> 3, c8 = cc & 7;
    uint8_t* dst = buf + region * 16384 + row * 128 + ((c8 ^ (row & 7)) << 4);
    if (zero)
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    else
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src + cc) : "memory");
  }
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ uint64_t kmaj_desc(uint32_t base, int kk) {
  return sw128_desc(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mn_desc(uint32_t base, int kk) {
  return sw128_desc(base + kk * 2048, 16384, 1024);
}

// 32 values per lane -> lane c holds the sum over the warp of value c
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = lane & off;
#pragma unroll
    for (int k = 0; k < off; ++k) {
      const float send = up ? v[k] : v[k + off];
      const float keep = up ? v[k + off] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// SEG: rows carry segment starts (packed sequences); without them the key >=
// segment test is compiled out
template <typename E, bool SEG>
__global__ void __launch_bounds__(kTcThreads, 1)
    bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                  const DashAttnBwdArgs a, int nblk, int words, int ntiles, float* dq_acc, const int qmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  SlotMeta* meta = reinterpret_cast<SlotMeta*>(sm + OFF_META);   // [2], batch b uses meta[b & 1]
  float* m_dsum = reinterpret_cast<float*>(meta + 2);            // [4][NS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* rows_full = bars + 0;
  uint64_t* s_full = bars + 1;
  uint64_t* p_full = bars + 2;
  uint64_t* pv_done = bars + 3;
  uint64_t* fin = bars + 4;
  uint64_t* meta_full = bars + 5;      // [2]
  uint64_t* meta_empty = bars + 7;     // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 10);
  DeviceError* derr = a.device_error;

  const int T = a.seq_len, HQ = a.n_heads, H = a.n_kv_heads, G = HQ / H;
  const int s = blockIdx.x / ntiles, tl = blockIdx.x - s * ntiles;
  const int h = blockIdx.y;
  const int key0 = tl * TK;
  const int bs = a.block_size, LW = a.local_window;
  const int bA = key0 / bs;                                  // first block of the tile
  const int nbt = min(key0 + TK - 1, T - 1) / bs - bA + 1;  // blocks in the tile (<= QB)
  // index head of this kv head; its routes are rows (s*HI + ih)*T + t
  const int HI = a.n_index_heads > 1 ? a.n_index_heads : 1;
  const int ih = h * HI / H;
  const int64_t rr_shift = ((int64_t)s * (HI - 1) + ih) * T;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t kv_row = (int64_t)H * 128;
  const int64_t kvoff = ((int64_t)s * T * H + h) * 128;
  const float LOG2E = 1.4426950408889634f;

  if (tid == 0) {
    mbar_init(rows_full, 8);
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
    mbar_init(fin, 1);
    mbar_init(meta_full + 0, 1);
    mbar_init(meta_full + 1, 1);
    mbar_init(meta_empty + 0, 8);
    mbar_init(meta_empty + 1, 8);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == kMmaWarp) { tmem_alloc(tmem_holder, TMEM_COLS); tmem_relinquish(); }
  if (tid < 2 * TK) {            // threads 0-127: K rows, 128-255: V rows
    const int r = tid & (TK - 1);
    const int key = key0 + r;
    const bool z = key >= T;
    const void* base = tid < TK ? a.k : a.v;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(base) + kvoff + (int64_t)(z ? 0 : key) * kv_row);
    st_row_sw128(sm + (tid < TK ? OFF_K : OFF_V), r, src, z);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;
  constexpr uint32_t fmt = Fmt<E>::v;

  if (warp == kProdWarp) {
    // ===================== producer: slot lists + per-slot meta =====================
    const uint32_t* fl0 = a.flags + (((int64_t)s * HI + ih) * nblk + bA) * words;   // block bA + q at + q*words
    const int64_t loc_end = min((int64_t)key0 + TK - 1 + LW - 1, (int64_t)T - 1);
    int next_row = key0;                 // first row not yet taken (uniform)
    for (int b = 0;; ++b) {
      SlotMeta& M = meta[b & 1];
      if (b >= 2 && !mbar_wait_warp(meta_empty + (b & 1), ((b >> 1) - 1) & 1, abort_flag, derr, 85)) break;
      // rows: 32 bitmask words per step, one per lane
      int cnt = 0;
      const int cap = NS / G;
      while (cnt < cap && next_row < T) {
        const int w = (next_row >> 5) + lane;
        uint32_t m = 0u;
        if (w < words) {
          for (int q = 0; q < nbt; ++q) m |= fl0[(int64_t)q * words + w];
          const int64_t r0 = (int64_t)w * 32;
          const int64_t lo = max(r0, (int64_t)key0), hi = min(r0 + 31, loc_end);
          if (lo <= hi) {
            const int nbits = (int)(hi - lo + 1);
            m |= (nbits == 32 ? 0xffffffffu : ((1u << nbits) - 1u)) << (int)(lo - r0);
          }
          if (lane == 0) m &= 0xffffffffu << (next_row & 31);
          if (r0 + 32 > T) m &= (T - r0 >= 32) ? 0xffffffffu : ((1u << (T - r0)) - 1u);
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
          const int r = cnt + excl + k;
          for (int g = 0; g < G; ++g) { M.row[r * G + g] = w * 32 + bit; M.hq[r * G + g] = h * G + g; }
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
      const int ns = cnt * G;
      __syncwarp();
      // per-slot meta, four slots per lane
#pragma unroll 1
      for (int q = 0; q < NS / 32; ++q) {
        const int n = lane + 32 * q;
        const bool live = n < ns;
        const int i = live ? M.row[n] : 0;
        const int hq = live ? M.hq[n] : 0;
        const int64_t row = (int64_t)s * T + i;
        const int64_t rr = row + rr_shift;     // row of this index head's routes
        int routed = 0;
        int slot[QB] = {-1, -1, -1, -1};
        float bias[QB] = {0.f, 0.f, 0.f, 0.f};
        float lse = 0.f, delta = 0.f;
        if (live) {
          lse = a.lse[row * HQ + hq];
          delta = a.delta[row * HQ + hq];
#pragma unroll
          for (int q = 0; q < QB; ++q)
            if (q < nbt && ((fl0[(int64_t)q * words + (i >> 5)] >> (i & 31)) & 1u)) routed |= 1 << q;
          // first slot of each routed tile block: 16 independent loads per step
          const int32_t* ids = a.idx + rr * a.K;
          int found = 0;
          for (int j0 = 0; j0 < a.K && found != routed; j0 += 16) {
            int v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = j0 + u < a.K ? ids[j0 + u] : -1;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int q = v[u] - bA;
#pragma unroll
              for (int qq = 0; qq < QB; ++qq)
                if (q == qq && ((routed >> qq) & 1) && !((found >> qq) & 1)) { slot[qq] = j0 + u; found |= 1 << qq; }
            }
          }
          if (a.bias) {
#pragma unroll
            for (int q = 0; q < QB; ++q)
              if (slot[q] >= 0) bias[q] = a.bias[rr * a.K + slot[q]];
          }
        }
        M.row[n] = (int)row;
        M.hq[n] = hq;
        M.sl[n] = make_int4(slot[0], slot[1], slot[2], slot[3]);
        // a padding slot's position keeps every key out
        const int seg = (live && a.seg_start) ? a.seg_start[row] : 0;
        M.a[n] = make_int4(live ? i : INT_MIN / 2, routed | (seg << 4), __float_as_int(-lse * LOG2E),
                           __float_as_int(delta));
        M.b[n] = make_float4((bias[0] - lse) * LOG2E, (bias[1] - lse) * LOG2E, (bias[2] - lse) * LOG2E,
                             (bias[3] - lse) * LOG2E);
      }
      if (lane == 0) M.ns = ns;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_full + (b & 1));
      if (ns == 0) break;
    }
  } else if (warp == kMmaWarp) {
    // ============================ MMA issuer ============================
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc(fmt, 0, 0, TK, NS);
      constexpr uint32_t idesc_acc = make_idesc(fmt, 0, 1, TK, 128);
      constexpr uint32_t idesc_dq = make_idesc(fmt, 1, 1, NS, 128);
      const uint32_t sK = smem_u32(sm + OFF_K), sV = smem_u32(sm + OFF_V);
      const uint32_t sQ = smem_u32(sm + OFF_Q), sDO = smem_u32(sm + OFF_DO), sDS = smem_u32(sm + OFF_DS);
      for (int b = 0;; ++b) {
        if (!mbar_wait(rows_full, b & 1, abort_flag, derr, 80)) break;
        tc_fence_after();
        if (*reinterpret_cast<volatile int*>(&meta[b & 1].ns) == 0) break;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ss(tS, kmaj_desc(sK, kk), kmaj_desc(sQ, kk), idesc_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ss(tDP, kmaj_desc(sV, kk), kmaj_desc(sDO, kk), idesc_s, kk > 0);
        umma_commit(s_full);
        if (!mbar_wait(p_full, b & 1, abort_flag, derr, 81)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ts(tDV, tS + kk * 8, mn_desc(sDO, kk), idesc_acc, (b > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ts(tDK, tS + 64 + kk * 8, mn_desc(sQ, kk), idesc_acc, (b > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_ss(tDP, mn_desc(sDS, kk), mn_desc(sK, kk), idesc_dq, kk > 0);
        umma_commit(pv_done);
      }
      // every MMA of this CTA completes before TMEM is released
      umma_commit(fin);
      volatile int no_abort = 0;
      mbar_wait(fin, 0, &no_abort, nullptr, 82);
    }
    __syncwarp();
  } else {
    // ============================ math warps ============================
    // warp w: TMEM lane quarter wq (keys, or slots for dQ) and column half sh
    const int wq = warp & 3, sh = warp >> 2;
    const int kl = wq * 32 + lane;               // this thread's TMEM lane
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float sl2 = a.scale * LOG2E;
    const int key = key0 + kl;
    const int kb = min(key, T - 1) / bs - bA;     // this key's block within the tile
    const int rmask = 1 << kb;
    int nb = 0;
    bool alive = true;
    while (alive) {
      if (nb > 0) {
        // ---- dQ of batch nb-1 -> fp32 accumulator (lanes = slots, d half sh) ----
        if (!math_all(mbar_wait_warp(pv_done, (nb - 1) & 1, abort_flag, derr, 83))) { alive = false; break; }
        tc_fence_after();
        const SlotMeta& P = meta[(nb - 1) & 1];
        const int ns_prev = P.ns;
        uint8_t* dstg = sm + OFF_DQSTG + warp * 4096;
#pragma unroll 1
        for (int q2 = 0; q2 < 2; ++q2) {
          float v[32];
          tmem_ld32f(tDP + sh * 64 + q2 * 32 + lane_base, v);
          tmem_ld_wait();
          // through shared memory (16-byte chunk c of slot `lane` at
          // ((c ^ (lane & 7)) << 4)): the warp then reduces its 32 slots'
          // 128-byte pieces four per instruction (8 lanes each) instead of
          // 32 scattered 16-byte pieces
#pragma unroll
          for (int c = 0; c < 8; ++c)
            *reinterpret_cast<float4*>(dstg + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int rr = 4 * j + (lane >> 3), cc = lane & 7;
            const int slot = wq * 32 + rr;
            if (slot < ns_prev) {
              const float4 w = *reinterpret_cast<const float4*>(dstg + rr * 128 + ((cc ^ (rr & 7)) << 4));
              float* dst = dq_acc + ((int64_t)P.row[slot] * HQ + P.hq[slot]) * 128 + sh * 64 + q2 * 32 + cc * 4;
              red_add_v4(dst, w.x, w.y, w.z, w.w);
            }
          }
          __syncwarp();
        }
        // the producer may refill this meta buffer
        __syncwarp();
        if (lane == 0) mbar_arrive(meta_empty + ((nb - 1) & 1));
      }
      if (!math_all(mbar_wait_warp(meta_full + (nb & 1), (nb >> 1) & 1, abort_flag, derr, 86))) { alive = false; break; }
      const SlotMeta& M = meta[nb & 1];
      const int ns = M.ns;
      if (ns == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(rows_full);
        break;
      }
      // ---- gather slot n: threads 0-127 its q row, 128-255 its dout row ----
      if (qmap) {
        // TMA row gather: lane l < 16 of warp w brings slots (w&3)*32 + 4(l&7)
        // .. +3, column half l>>3, of q (warps 0-3) or dout (warps 4-7).  A
        // padding slot reads row 0: its position keeps every key out, so its
        // P and dS are 0 whatever the row holds.
        const int wq4 = warp & 3;
        const bool isdo = warp >= 4;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(rows_full, 32 * 256);
        __syncwarp();
        if (lane < 16) {
          const int quad = lane & 7, hf = lane >> 3;
          const int n0 = wq4 * 32 + 4 * quad;
          int r[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) r[j] = n0 + j < ns ? M.row[n0 + j] * HQ + M.hq[n0 + j] : 0;
          tma_gather4(sm + (isdo ? OFF_DO : OFF_Q) + hf * 16384 + n0 * 128, isdo ? &tmDO : &tmQ, rows_full,
                      hf * 64, r[0], r[1], r[2], r[3]);
        }
      } else {
        const int n = tid & (NS - 1);
        const bool live = n < ns;
        const int64_t off = ((int64_t)(live ? M.row[n] : 0) * HQ + (live ? M.hq[n] : 0)) * 128;
        if (tid >= NS)
          cp_row_sw128(sm + OFF_DO, n, reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(a.dout) + off), !live);
        else
          cp_row_sw128(sm + OFF_Q, n, reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(a.q) + off), !live);
        cp_async_wait_all();
        fence_proxy_async_smem();
        math_bar();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(rows_full);
      }
      // ---- P^T and dS^T for key `key` (TMEM lane kl), slots sh*64 .. +63 ----
      if (!math_all(mbar_wait_warp(s_full, nb & 1, abort_flag, derr, 84))) { alive = false; break; }
      tc_fence_after();
      {
        const int h2 = sh;
        uint32_t pkP[32], pkD[32];
#pragma unroll
        for (int c32 = 0; c32 < 2; ++c32) {
          float x[32], y[32], rs[32];
          const uint32_t col = h2 * 64 + c32 * 32;
          tmem_ld32f(tS + col + lane_base, x);
          tmem_ld32f(tDP + col + lane_base, y);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float pv[2], dv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int n = col + e + u;
              const int4 ma = M.a[n];
              const float mb = reinterpret_cast<const float*>(M.b)[n * QB + kb];
              const int d = ma.x - key;
              const bool inseg = !SEG || key >= (ma.y >> 4);
              const bool local = d >= 0 && d < LW && inseg;
              const bool remote = d >= LW && (ma.y & rmask) && inseg;
              const float c = remote ? mb : __int_as_float(ma.z);
              const float p = (local || remote) ? fast_exp2(fmaf(x[e + u], sl2, c)) : 0.f;
              const float ds = (local || remote) ? p * (y[e + u] - __int_as_float(ma.w)) : 0.f;
              pv[u] = p;
              dv[u] = ds;
              rs[e + u] = remote ? ds : 0.f;
            }
            pkP[c32 * 16 + e / 2] = Fmt<E>::pack(pv[0], pv[1]);
            pkD[c32 * 16 + e / 2] = Fmt<E>::pack(dv[0], dv[1]);
          }
          m_dsum[wq * NS + col + lane] = reduce_scatter32(rs, lane);
        }
        // P^T / dS^T of slot half h2 go to S^T columns h2*32 / 64 + h2*32,
        // which both warpgroups read as S^T: store after both have read
        math_bar();
        tmem_st32(tS + h2 * 32 + lane_base, pkP);
        tmem_st32(tS + 64 + h2 * 32 + lane_base, pkD);
        // dS^T row kl (slots h2*64 .. +63) -> MN-major shared buffer
        uint8_t* drow = sm + OFF_DS + h2 * 16384 + kl * 128;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8)
          *reinterpret_cast<uint4*>(drow + ((c8 ^ (kl & 7)) << 4)) =
              make_uint4(pkD[4 * c8], pkD[4 * c8 + 1], pkD[4 * c8 + 2], pkD[4 * c8 + 3]);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      math_bar();
      // ---- slot-bias gradient of slot tid ----
      if (tid < ns && a.d_bias) {
        // warp quarter w (keys key0 + 32w ..) lies in tile block qb(w)
        float sum[QB] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int qb = min(key0 + 32 * w, T - 1) / bs - bA;
          const float v = m_dsum[w * NS + tid];
#pragma unroll
          for (int q = 0; q < QB; ++q) sum[q] += q == qb ? v : 0.f;
        }
        const int64_t row = M.row[tid] + rr_shift;
        const int4 sl = M.sl[tid];
        const int slq[QB] = {sl.x, sl.y, sl.z, sl.w};
#pragma unroll
        for (int q = 0; q < QB; ++q)
          if (slq[q] >= 0) red_add(a.d_bias + row * a.K + slq[q], sum[q]);
      }
      ++nb;
    }
    // ---- dK, dV of key kl, d half sh ----
    // (alive is uniform over the math warps; the TMEM loads are warp-collective,
    // so every lane issues them and only the stores depend on the key)
    if (alive) {
      const bool kv_ok = key < T;
      E* dkp = reinterpret_cast<E*>(a.dk) + kvoff + (int64_t)(kv_ok ? key : 0) * kv_row + sh * 64;
      E* dvp = reinterpret_cast<E*>(a.dv) + kvoff + (int64_t)(kv_ok ? key : 0) * kv_row + sh * 64;
#pragma unroll 1
      for (int q4 = 0; q4 < 2; ++q4) {
        float kv[32], vv[32];
        tmem_ld32f(tDK + sh * 64 + q4 * 32 + lane_base, kv);
        tmem_ld32f(tDV + sh * 64 + q4 * 32 + lane_base, vv);
        tmem_ld_wait();
        if (!kv_ok) continue;
        uint32_t pk[16], pv[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          pk[c] = nb > 0 ? Fmt<E>::pack(kv[2 * c] * a.scale, kv[2 * c + 1] * a.scale) : 0u;
          pv[c] = nb > 0 ? Fmt<E>::pack(vv[2 * c], vv[2 * c + 1]) : 0u;
        }
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          *reinterpret_cast<uint4*>(dkp + q4 * 32 + v4 * 8) = make_uint4(pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2], pk[4 * v4 + 3]);
          *reinterpret_cast<uint4*>(dvp + q4 * 32 + v4 * 8) = make_uint4(pv[4 * v4], pv[4 * v4 + 1], pv[4 * v4 + 2], pv[4 * v4 + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, TMEM_COLS);
}

// delta[row, h] = sum_d o * dout (one warp per (row, head))
template <typename E>
__global__ void __launch_bounds__(256) bwd_delta_kernel(DashAttnBwdArgs a, int64_t n) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const E* o = reinterpret_cast<const E*>(a.o) + w * 128 + lane * 4;
  const E* d = reinterpret_cast<const E*>(a.dout) + w * 128 + lane * 4;
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) acc = fmaf(Fmt<E>::tof(o[c]), Fmt<E>::tof(d[c]), acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) a.delta[w] = acc;
}

// dq = scale * acc, converted
template <typename E>
__global__ void __launch_bounds__(256) bwd_dq_convert_kernel(const float* acc, E* dq, float scale, int64_t n4) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n4) return;
  const float4 v = reinterpret_cast<const float4*>(acc)[i];
  uint2 r;
  r.x = Fmt<E>::pack(v.x * scale, v.y * scale);
  r.y = Fmt<E>::pack(v.z * scale, v.w * scale);
  reinterpret_cast<uint2*>(dq)[i] = r;
}

static PFN_cuTensorMapEncodeTiled_v12000 bwd_encode_fn() {
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

// q or dout [n_seq, seq_len, n_heads, 128] as a 2-D tensor of 128-element
// rows for the TMA row gather (box: one row x 64 columns, 128-byte swizzle).
// Returns false when the rows do not fit the gather's int coordinates; the
// kernel then copies rows with cp.async.
static bool make_rows_map(CUtensorMap* map, const void* base, const DashAttnBwdArgs& a) {
  auto enc = bwd_encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  const int64_t rows = (int64_t)a.n_seq * a.seq_len * a.n_heads;
  if (rows <= 0 || rows >= ((int64_t)1 << 31)) return false;
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, 1};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, a.dtype == DASH_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename E>
int launch_tc_typed(const DashAttnBwdArgs& a, int nblk, int words, float* dq_acc, cudaStream_t st) {
  const int64_t rows = (int64_t)a.n_seq * a.seq_len;
  const int64_t nrh = rows * a.n_heads;
  bwd_delta_kernel<E><<<(unsigned)((nrh + 7) / 8), 256, 0, st>>>(a, nrh);
  count_launch();
  int rc = check_launch("bwd_delta_kernel");
  if (rc) return rc;
  const int ntiles = (a.seq_len + TK - 1) / TK;
  const dim3 grid((unsigned)(a.n_seq * ntiles), (unsigned)a.n_kv_heads);
  CUtensorMap mq, mdo;
  memset(&mq, 0, sizeof(mq));
  memset(&mdo, 0, sizeof(mdo));
  const int qmap = make_rows_map(&mq, a.q, a) && make_rows_map(&mdo, a.dout, a) ? 1 : 0;
  if (a.seg_start) {
    cudaFuncSetAttribute(bwd_tc_kernel<E, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TC);
    bwd_tc_kernel<E, true><<<grid, kTcThreads, SMEM_TC, st>>>(mq, mdo, a, nblk, words, ntiles, dq_acc, qmap);
  } else {
    cudaFuncSetAttribute(bwd_tc_kernel<E, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TC);
    bwd_tc_kernel<E, false><<<grid, kTcThreads, SMEM_TC, st>>>(mq, mdo, a, nblk, words, ntiles, dq_acc, qmap);
  }
  count_launch();
  rc = check_launch("bwd_tc_kernel");
  if (rc) return rc;
  const int64_t n4 = nrh * 32;
  bwd_dq_convert_kernel<E><<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(dq_acc, reinterpret_cast<E*>(a.dq), a.scale, n4);
  count_launch();
  return check_launch("bwd_dq_convert_kernel");
}

}  // namespace

size_t attn_bwd_tc_acc_bytes(const DashAttnBwdArgs& a) {
  if (a.dtype != DASH_DTYPE_BF16 && a.dtype != DASH_DTYPE_F16) return 0;
  return (size_t)a.n_seq * a.seq_len * a.n_heads * 128 * 4;
}

int launch_attn_bwd_tc(const DashAttnBwdArgs& a, int nblk, int words, cudaStream_t st) {
  float* dq_acc = a.dq_acc;
  if (cudaMemsetAsync(dq_acc, 0, attn_bwd_tc_acc_bytes(a), st) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "memset of the dq accumulator failed");
  if (a.dtype == DASH_DTYPE_BF16) return launch_tc_typed<__nv_bfloat16>(a, nblk, words, dq_acc, st);
  return launch_tc_typed<__half>(a, nblk, words, dq_acc, st);
}

}  // namespace dash
