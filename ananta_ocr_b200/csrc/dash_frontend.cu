// dash_frontend.cu -- router front end on tcgen05: the two index projections
// (hidden x [W_q ; W_k]^T) for 256 tokens per CTA as two M=128 x N=256 MMA
// chains sharing every weight tile, with the RMSNorm + RoPE epilogue read
// straight from TMEM and the index-K rows written to their destination (dense,
// or the paged index cache slot).
//
// Bytes: the hidden rows are read once (HBM); the weights (2 x 128 x hidden
// bf16) are re-read by every CTA from L2, so 256 tokens per CTA halve that
// L2 -> SM traffic against 128 (the mainloop is bound by it, not by HBM).
//
// Roles (576 threads, one CTA per 256 tokens):
//   warp 0       TMA producer: per 64-wide slice of the hidden dimension, the
//                two hidden tiles [128 x 64] and the two weight tiles
//                [128 x 64] (SWIZZLE_128B), into a 3-stage ring (64 KB each)
//   warp 1       TMEM allocation (512 columns) and the MMA issuer (one thread):
//                per stage 2 accumulators x 4 tcgen05.mma (K = 16), fp32
//   warps 2-17   epilogue, one (accumulator, projection, row) per thread: TMEM
//                lane = token row (warp w reads lane quarter w % 4), columns
//                [0,128) of an accumulator are q, [128,256) are k.  The thread
//                rounds its row to bf16 (the reference's Linear output), takes
//                the mean square, normalises, applies the rotate-half RoPE with
//                the reference's per-operation bf16 rounding and stages the
//                (bf16-exact) results in the freed stage buffers; the tile is
//                then written with coalesced row stores.
// Every wait is bounded (mbar_wait); on a timeout the CTA raises its abort
// flag, records DASH_DEV_TIMEOUT, drains its TMA copies and MMAs and frees TMEM.
#include <cudaTypedefs.h>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {
namespace fe {
constexpr int BM = 256;                      // token rows per CTA (two accumulators)
constexpr int BK = 64;                       // hidden columns per stage (128 B of bf16)
constexpr int D = 128;                       // index dim
constexpr int BN = 2 * D;                    // q | k
constexpr int NST = 3;
constexpr int A_BYTES = 128 * BK * 2;        // 16 KB per 128-row hidden tile
constexpr int W_BYTES = D * BK * 2;          // 16 KB per weight tile
constexpr int STAGE = 2 * A_BYTES + 2 * W_BYTES;   // 64 KB
constexpr int OFF_NORM = NST * STAGE;        // (1 + w_q), (1 + w_k): fp32 [2][128]
constexpr int OFF_BAR = OFF_NORM + 2 * D * 4;
constexpr int SMEM_BYTES = OFF_BAR + 128 + 1024;   // barriers + alignment slack
constexpr int EPI_WARPS = 16;
constexpr int NTHREADS = (2 + EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int ST_LD = D + 8;                 // bf16 staging row pitch (272 B)
constexpr int UNIT_BYTES = 128 * ST_LD * 2;  // one (accumulator, projection) tile
static_assert(4 * UNIT_BYTES <= OFF_NORM, "epilogue staging must fit the stage buffers");
}  // namespace fe

// fp32 -> bf16 -> fp32, round to nearest even, on the integer pipe (the
// rounding the reference's bf16 tensors apply; non-finite values keep their
// class: inf stays inf, a quiet NaN stays NaN)
__device__ __forceinline__ uint32_t bf16r_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
}
__device__ __forceinline__ float bf16r(float x) { return __uint_as_float(bf16r_bits(x)); }
// two fp32 -> packed bf16x2 (lo, hi), rounded to nearest even on the integer pipe
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return __byte_perm(bf16r_bits(lo), bf16r_bits(hi), 0x7632);
}

// y = bf16(x * inv * w1) (w1 = 1 + w); the clamped variant zeroes non-finite x
// and clamps both products to +-1e4 (dash_attention.py:680-700)
__device__ __forceinline__ float rms_scale(float x, float inv, float w1, bool clamp) {
  if (clamp) {
    if (!isfinite(x)) x = 0.0f;
    const float y = clamp_act(__fmul_rn(x, inv));
    return bf16r(clamp_act(__fmul_rn(y, w1)));
  }
  return bf16r(__fmul_rn(__fmul_rn(x, inv), w1));
}

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(fe::EPI_WARPS * 32) : "memory");
}

// AND of `v` over the epilogue warps (a named-barrier reduction)
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)v), "r"(fe::EPI_WARPS * 32)
      : "memory");
  return out != 0;
}

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// One projection of this thread's row: TMEM columns [tcol, tcol + 128) hold
// x.  Pass 1 reads TMEM once, stores the bf16-rounded row in the staging row
// `srow` and sums the squares; pass 2 reads the row back from shared memory and
// overwrites it with the (bf16-exact) outputs.
__device__ __forceinline__ void epilogue_unit(uint32_t tcol, const float* w1s,
                                              const uint4* cos_row, const uint4* sin_row,
                                              float eps, bool clamp, __nv_bfloat16* srow) {
  float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    float v[64];
    tmem_ld32f(tcol + c * 64, v);
    tmem_ld32f(tcol + c * 64 + 32, v + 32);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 64; j += 8) {
      uint32_t p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x0 = bf16r(v[j + 2 * e]), x1 = bf16r(v[j + 2 * e + 1]);
        if (clamp) {
          if (!isfinite(x0)) x0 = 0.0f;
          if (!isfinite(x1)) x1 = 0.0f;
        }
        ss[e] = __fadd_rn(ss[e], __fmul_rn(x0, x0));
        ss[e] = __fadd_rn(ss[e], __fmul_rn(x1, x1));
        p[e] = __byte_perm(__float_as_uint(x0), __float_as_uint(x1), 0x7632);
      }
      *reinterpret_cast<uint4*>(srow + c * 64 + j) = make_uint4(p[0], p[1], p[2], p[3]);
    }
  }
  const float tot = __fadd_rn(__fadd_rn(ss[0], ss[1]), __fadd_rn(ss[2], ss[3]));
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / 128.0f), eps));
  // pass 2: columns j and j + 64 together (rotate-half partners), 8 at a time
#pragma unroll 2
  for (int g = 0; g < 8; ++g) {
    const uint4 xa4 = *reinterpret_cast<const uint4*>(srow + g * 8);
    const uint4 xb4 = *reinterpret_cast<const uint4*>(srow + 64 + g * 8);
    uint4 ca, sa, cb, sb;
    if (cos_row) {
      ca = __ldg(cos_row + g);
      sa = __ldg(sin_row + g);
      cb = __ldg(cos_row + 8 + g);
      sb = __ldg(sin_row + 8 + g);
    }
    const uint32_t xav[4] = {xa4.x, xa4.y, xa4.z, xa4.w}, xbv[4] = {xb4.x, xb4.y, xb4.z, xb4.w};
    const uint32_t cav[4] = {ca.x, ca.y, ca.z, ca.w}, sav[4] = {sa.x, sa.y, sa.z, sa.w};
    const uint32_t cbv[4] = {cb.x, cb.y, cb.z, cb.w}, sbv[4] = {sb.x, sb.y, sb.z, sb.w};
    uint32_t pa[4], pb[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float oa[2], ob[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = g * 8 + 2 * e + h;
        const float xa = h ? bf_hi(xav[e]) : bf_lo(xav[e]);
        const float xb = h ? bf_hi(xbv[e]) : bf_lo(xbv[e]);
        const float ya = rms_scale(xa, inv, w1s[j], clamp);
        const float yb = rms_scale(xb, inv, w1s[j + 64], clamp);
        oa[h] = ya;
        ob[h] = yb;
        if (cos_row) {
          const float c_a = h ? bf_hi(cav[e]) : bf_lo(cav[e]);
          const float s_a = h ? bf_hi(sav[e]) : bf_lo(sav[e]);
          const float c_b = h ? bf_hi(cbv[e]) : bf_lo(cbv[e]);
          const float s_b = h ? bf_hi(sbv[e]) : bf_lo(sbv[e]);
          // rot = (-y_hi, y_lo); every product and the sum rounded to bf16
          oa[h] = __fadd_rn(bf16r(__fmul_rn(ya, c_a)), -bf16r(__fmul_rn(yb, s_a)));
          ob[h] = __fadd_rn(bf16r(__fmul_rn(yb, c_b)), bf16r(__fmul_rn(ya, s_b)));
        }
      }
      pa[e] = pack_bf16x2(oa[0], oa[1]);
      pb[e] = pack_bf16x2(ob[0], ob[1]);
    }
    *reinterpret_cast<uint4*>(srow + g * 8) = make_uint4(pa[0], pa[1], pa[2], pa[3]);
    *reinterpret_cast<uint4*>(srow + 64 + g * 8) = make_uint4(pb[0], pb[1], pb[2], pb[3]);
  }
}

// k-bar of one page by one warp, in the arithmetic order of kbar_pool_kernel
// (dash_router.cu): per key a sequential FMA chain over the feature index,
// clamp, max, det_expf, a sequential sum, IEEE division, then per feature a
// sequential FMA chain over the keys; non-finite -> 0.
__device__ __noinline__ void kbar_refresh_warp(const DashIndexProjArgs& a, int64_t page, int n, int lane) {
  if (n <= 0) return;
  constexpr int D = 128, MAXJ = 8;                 // up to 256 keys per page
  const bool b16 = a.k_dtype == DASH_DTYPE_BF16;
  auto key = [&](int j, int c) -> float {
    const int64_t row = page * a.kbar_block_size + j;
    return b16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.idx_k)[row * a.k_stride + c])
               : reinterpret_cast<const float*>(a.idx_k)[row * a.k_stride + c];
  };
  const float inv_sqrt_d = (float)(1.0 / sqrt((double)D));
  float e[MAXJ];
  float lmax = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXJ; ++i) {
    const int j = lane + 32 * i;
    e[i] = 0.0f;
    if (j < n) {
      float acc = 0.0f;
      for (int c = 0; c < D; ++c) acc = __fmaf_rn(key(j, c), a.kbar_head_cls ? a.kbar_head_cls[c] : 0.0f, acc);
      e[i] = clamp_act(__fmul_rn(acc, inv_sqrt_d));
      lmax = fmaxf(lmax, e[i]);
    }
  }
  for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
#pragma unroll
  for (int i = 0; i < MAXJ; ++i)
    if (lane + 32 * i < n) e[i] = det_expf(__fsub_rn(e[i], lmax));
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXJ; ++i)
    for (int l = 0; l < 32; ++l) {
      const float v = __shfl_sync(0xffffffffu, e[i], l);
      if (32 * i + l < n) sum = __fadd_rn(sum, v);
    }
  const float den = sum > 1e-6f ? sum : 1e-6f;
#pragma unroll
  for (int i = 0; i < MAXJ; ++i) e[i] = __fdiv_rn(e[i], den);
  float acc[D / 32];
#pragma unroll
  for (int q = 0; q < D / 32; ++q) acc[q] = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXJ; ++i)
    for (int l = 0; l < 32; ++l) {
      const int j = 32 * i + l;
      if (j >= n) break;
      const float w = __shfl_sync(0xffffffffu, e[i], l);
#pragma unroll
      for (int q = 0; q < D / 32; ++q) acc[q] = __fmaf_rn(w, key(j, lane + 32 * q), acc[q]);
    }
#pragma unroll
  for (int q = 0; q < D / 32; ++q) {
    float v = acc[q];
    if (!(v == v) || isinf(v)) v = 0.0f;
    a.kbar[page * a.kbar_row_stride + lane + 32 * q] = v;
  }
}

__global__ void __launch_bounds__(fe::NTHREADS, 1)
    index_proj_kernel(const __grid_constant__ CUtensorMap tmH,
                      const __grid_constant__ CUtensorMap tmWq,
                      const __grid_constant__ CUtensorMap tmWk, const DashIndexProjArgs a) {
  using namespace fe;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* w1s = reinterpret_cast<float*>(sm + OFF_NORM);       // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* full = bars;                 // [NST] TMA -> MMA
  uint64_t* empty = bars + NST;          // [NST] MMA -> TMA
  uint64_t* acc_full = bars + 2 * NST;   // MMA -> epilogue
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * NST + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * NST + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * BM;
  const int nk = a.hidden_dim / BK;
  DeviceError* derr = a.device_error;

  if (tid == 0) {
    for (int k = 0; k < NST; ++k) {
      mbar_init(full + k, 1);
      mbar_init(empty + k, 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (tid >= 64 && tid < 64 + 2 * D) {   // (1 + w) of both norms, fp32
    const int j = tid - 64;
    w1s[j] = __fadd_rn(1.0f, j < D ? a.norm_q[j] : a.norm_k[j - D]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // =================== TMA producer ===================
    if (lane == 0) {
      prefetch_tmap(&tmH);
      prefetch_tmap(&tmWq);
      prefetch_tmap(&tmWk);
      int ks = 0;
      for (; ks < nk; ++ks) {
        const int st = ks % NST;
        if (ks >= NST && !mbar_wait(empty + st, ((ks / NST) - 1) & 1, abort_flag, derr, 70)) break;
        uint8_t* dA = sm + st * STAGE;
        mbar_arrive_expect_tx(full + st, STAGE);
        tma_load_2d(dA, &tmH, full + st, ks * BK, m0);
        tma_load_2d(dA + A_BYTES, &tmH, full + st, ks * BK, m0 + 128);
        tma_load_2d(dA + 2 * A_BYTES, &tmWq, full + st, ks * BK, 0);
        tma_load_2d(dA + 2 * A_BYTES + W_BYTES, &tmWk, full + st, ks * BK, 0);
      }
      // drain: never leave the CTA with bulk copies in flight
      for (int k = max(0, ks - NST); k < ks; ++k) {
        volatile int no_abort = 0;
        mbar_wait(full + (k % NST), (k / NST) & 1, &no_abort, nullptr, 71);
      }
    }
  } else if (warp == 1) {
    // =================== MMA issuer ===================
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(1, 0, 0, 128, BN);   // bf16 x bf16 -> fp32
      for (int ks = 0; ks < nk; ++ks) {
        const int st = ks % NST;
        if (!mbar_wait(full + st, (ks / NST) & 1, abort_flag, derr, 72)) break;
        tc_fence_after();
        const uint32_t sA = smem_u32(sm + st * STAGE);
        const uint32_t sB = sA + 2 * A_BYTES;   // q rows 0..127, then k rows 128..255
#pragma unroll
        for (int acc = 0; acc < 2; ++acc) {
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sw128_desc(sA + acc * A_BYTES + kk * 32, 16, 1024);
            const uint64_t bd = sw128_desc(sB + kk * 32, 16, 1024);
            umma_ss(tmem + acc * BN, ad, bd, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(empty + st);
      }
      // issued MMAs complete before the epilogue (and the dealloc) proceed
      umma_commit(acc_full);
      volatile int no_abort = 0;
      mbar_wait(acc_full, 0, &no_abort, nullptr, 75);
    }
  } else {
    // ===== epilogue: thread = (accumulator, projection, row); TMEM lane = row =====
    const int ew = warp - 2;                         // 0..15
    const int q4 = warp & 3;                         // TMEM lane quarter of this warp
    const int unit = ew >> 2;                        // 0..3
    const int acc = unit >> 1, proj = unit & 1;
    const int r = q4 * 32 + lane;                    // row within the accumulator
    const int64_t t = (int64_t)m0 + acc * 128 + r;
    const bool live = t < a.T;
    const bool rope = a.cos != nullptr;
    const uint4* cr = nullptr;
    const uint4* sr = nullptr;
    if (rope) {
      const int64_t tt = live ? t : 0;
      cr = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.cos) + tt * a.cs_stride);
      sr = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.sin) + tt * a.cs_stride);
    }
    // (an aborted CTA still commits acc_full; its partial sums are not stored)
    const bool ok = mbar_wait_warp(acc_full, 0, abort_flag, derr, 73) &&
                    __all_sync(0xffffffffu, *abort_flag == 0);
    tc_fence_after();
    if (epi_all(ok)) {
      // the stage buffers are free: every MMA that read them has completed
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(sm + unit * UNIT_BYTES);
      const uint32_t tcol = tmem + acc * BN + proj * D + ((uint32_t)(q4 * 32) << 16);
      epilogue_unit(tcol, w1s + proj * D, cr, sr, a.eps, a.norm_clamp != 0, stage + r * ST_LD);
      epi_bar();
      // coalesced write-out: 4 units x 128 rows, warp ew takes rows ew, ew + 16, ...
      const bool kb16 = a.k_dtype == DASH_DTYPE_BF16;
      for (int rr = ew; rr < 4 * 128; rr += EPI_WARPS) {
        const int u = rr >> 7, row = rr & 127;
        const int64_t tk = (int64_t)m0 + (u >> 1) * 128 + row;
        if (tk >= a.T) continue;
        const uint2 v = *reinterpret_cast<const uint2*>(
            reinterpret_cast<const __nv_bfloat16*>(sm + u * UNIT_BYTES) + row * ST_LD + 4 * lane);
        if ((u & 1) == 0) {
          float4 f = make_float4(bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y));
          reinterpret_cast<float4*>(a.idx_q + tk * a.q_stride)[lane] = f;
        } else {
          int64_t krow = tk;
          if (a.slot_mapping) {
            krow = a.slot_mapping[tk];
            if (krow < 0 || krow >= a.k_rows) {
              if (lane == 0) record_error(derr, DASH_DEV_BAD_PAGE, 74, krow);
              continue;
            }
          }
          if (kb16) {
            reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.idx_k) + krow * a.k_stride)[lane] = v;
          } else {
            float4 f = make_float4(bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y));
            reinterpret_cast<float4*>(reinterpret_cast<float*>(a.idx_k) + krow * a.k_stride)[lane] = f;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
  // fused k-bar refresh: the barrier above made this CTA's idx_k rows visible
  // to all its threads; a warp per token naming a page
  if (a.kbar_page) {
    const int nwarps = NTHREADS / 32;
    for (int tl = warp; tl < 2 * 128; tl += nwarps) {
      const int64_t t = (int64_t)m0 + tl;
      if (t >= a.T) break;
      const int64_t page = a.kbar_page[t];
      if (page < 0) continue;
      kbar_refresh_warp(a, page, min(a.kbar_ntok[t], a.kbar_block_size), lane);
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 fe_encode() {
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

// 2-D bf16 map of [rows, cols] (row stride in elements), box {64, 128}, SW128
static int make_rows_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                         int64_t stride) {
  auto enc = fe_encode();
  if (!enc) return set_error(DASH_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)fe::BK, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DASH_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DASH_OK;
}

int launch_index_proj(const DashIndexProjArgs& a, cudaStream_t st) {
  if (a.T == 0) return DASH_OK;
  CUtensorMap mh, mq, mk;
  int rc = make_rows_map(&mh, a.hidden, a.T, a.hidden_dim, a.hidden_stride);
  if (!rc) rc = make_rows_map(&mq, a.w_q, fe::D, a.hidden_dim, a.w_stride);
  if (!rc) rc = make_rows_map(&mk, a.w_k, fe::D, a.hidden_dim, a.w_stride);
  if (rc) return rc;
  cudaFuncSetAttribute(index_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fe::SMEM_BYTES);
  const unsigned grid = (unsigned)((a.T + fe::BM - 1) / fe::BM);
  index_proj_kernel<<<grid, fe::NTHREADS, fe::SMEM_BYTES, st>>>(mh, mq, mk, a);
  count_launch();
  return check_launch("index_proj_kernel");
}

}  // namespace dash

namespace dash {

// ---------------------------------------------------------------------------
// rope_kv_kernel: one CTA per token; thread work item = 8 columns of a head
// row plus their rotate-half partners (q and k), or 8 columns of v.  HBM-bound
// elementwise pass: q read + written, k and v read and written once into the
// cache rows, cos/sin read once per token.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 rope8(uint4 x, uint4 xp, uint4 c, uint4 s, bool lo_half) {
  // lo_half: x holds columns j < 64 (rot = -x_partner), else rot = +x_partner
  const uint32_t xv[4] = {x.x, x.y, x.z, x.w}, pv[4] = {xp.x, xp.y, xp.z, xp.w};
  const uint32_t cv[4] = {c.x, c.y, c.z, c.w}, sv[4] = {s.x, s.y, s.z, s.w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float r[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float xf = h ? bf_hi(xv[e]) : bf_lo(xv[e]);
      float pf = h ? bf_hi(pv[e]) : bf_lo(pv[e]);
      if (lo_half) pf = -pf;
      const float cf = h ? bf_hi(cv[e]) : bf_lo(cv[e]);
      const float sf = h ? bf_hi(sv[e]) : bf_lo(sv[e]);
      r[h] = __fadd_rn(bf16r(__fmul_rn(xf, cf)), bf16r(__fmul_rn(pf, sf)));
    }
    o[e] = pack_bf16x2(r[0], r[1]);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(256) rope_kv_kernel(DashRopeKVArgs a) {
  const int64_t t = blockIdx.x;
  const int nq = a.n_q_heads, nkv = a.n_kv_heads;
  const uint4* cs = a.cos ? reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.cos) + t * a.cs_stride) : nullptr;
  const uint4* sn = a.cos ? reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.sin) + t * a.cs_stride) : nullptr;
  const int64_t slot = a.slot_mapping ? a.slot_mapping[t] : t;
  const bool slot_ok = slot >= 0 && slot < a.num_slots;
  if (!slot_ok && threadIdx.x == 0) record_error(a.device_error, DASH_DEV_BAD_PAGE, 80, slot);
  // work items: q pair-chunks (nq * 8), k pair-chunks (nkv * 8), v chunks (nkv * 16)
  const int n_items = nq * 8 + nkv * 8 + (a.v ? nkv * 16 : 0);
  for (int it = threadIdx.x; it < n_items; it += blockDim.x) {
    if (it < nq * 8 + nkv * 8) {
      const bool is_q = it < nq * 8;
      const int i = is_q ? it : it - nq * 8;
      const int head = i >> 3, ch = i & 7;                 // columns [8ch, 8ch+8) and +64
      const uint4* src = reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(is_q ? a.q : a.k) + t * (is_q ? a.q_stride : a.k_stride)) + head * 16;
      const uint4 lo = src[ch], hi = src[8 + ch];
      uint4 olo = lo, ohi = hi;
      if (cs) {
        olo = rope8(lo, hi, __ldg(cs + ch), __ldg(sn + ch), true);
        ohi = rope8(hi, lo, __ldg(cs + 8 + ch), __ldg(sn + 8 + ch), false);
      }
      uint4* dst;
      if (is_q) {
        dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.q_out) + t * a.q_out_stride) + head * 16;
      } else {
        if (!slot_ok) continue;
        dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.k_cache) + slot * a.cache_row_stride) + head * 16;
      }
      dst[ch] = olo;
      dst[8 + ch] = ohi;
    } else {
      if (!slot_ok) continue;
      const int i = it - nq * 8 - nkv * 8;                  // v: head i / 16, chunk i % 16
      const uint4* src = reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(a.v) + t * a.v_stride);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.v_cache) + slot * a.cache_row_stride);
      dst[i] = src[i];
    }
  }
}

int launch_rope_kv(const DashRopeKVArgs& a, cudaStream_t st) {
  if (a.T == 0) return DASH_OK;
  rope_kv_kernel<<<(unsigned)a.T, 256, 0, st>>>(a);
  count_launch();
  return check_launch("rope_kv_kernel");
}

}  // namespace dash
