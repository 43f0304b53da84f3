// dash_common.cuh -- shared device helpers for the DASH sm_100a kernels.
//
// Contents: status codes and the device error word, bounded mbarrier waits,
// TMA tile loads, tcgen05 (TMEM alloc / MMA / commit / ld / st) wrappers, the
// fixed-order fp32 helpers the router shares with the CPU oracle.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/dash_b200.h"

namespace dash {

// ---------------------------------------------------------------------------
// Device error word.  Kernels never trap: a failed bounds check or a wait
// that ran past its limit records the first error code here and the kernel
// returns.  The host reads it with dash_device_error().
// ---------------------------------------------------------------------------
using DeviceError = DashDeviceError;

__device__ __forceinline__ void record_error(DeviceError* e, int code, int where,
                                             long long info) {
  if (e && atomicCAS(reinterpret_cast<int*>(&e->code), 0, code) == 0) {
    e->where = where;
    e->info = info;
  }
}

// ---------------------------------------------------------------------------
// Image-page membership of block descriptor i: page q lies in [lo, hi] and,
// with a page bit set, bit (q - lo) is set (exact set instead of range).
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool page_desc_holds(const int32_t* lo_a, const int32_t* hi_a,
                                                const uint32_t* bits, int words, int64_t i,
                                                int q) {
  const int lo = lo_a[i];
  if (q < 0 || lo < 0 || q < lo || q > hi_a[i]) return false;
  if (!bits) return true;
  const int k = q - lo;
  if (k >= 32 * words) return false;
  return (bits[i * words + (k >> 5)] >> (k & 31)) & 1u;
}

// ---------------------------------------------------------------------------
// Fixed-order fp32 arithmetic shared with oracle/dash_oracle.c
// ---------------------------------------------------------------------------
__device__ __forceinline__ float clamp_act(float z) {
  // keeps NaN as NaN (torch.clamp semantics)
  if (z < -1.0e4f) return -1.0e4f;
  if (z > 1.0e4f) return 1.0e4f;
  return z;
}

// exp(x), x <= 0, Cody-Waite reduction + degree-7 Taylor polynomial; the same
// operation sequence as det_expf() of the CPU oracle, so results are bitwise
// equal to it.
__device__ __forceinline__ float det_expf(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  if (x > 0.0f) x = 0.0f;
  const float log2e = __uint_as_float(0x3FB8AA3Bu);
  const float ln2_hi = __uint_as_float(0x3F317200u);
  const float ln2_lo = __uint_as_float(0x35BFBE8Eu);
  float n = rintf(__fmul_rn(x, log2e));
  float r = __fmaf_rn(n, -ln2_hi, x);
  r = __fmaf_rn(n, -ln2_lo, r);
  float p = __uint_as_float(0x39500D01u);
  p = __fmaf_rn(p, r, __uint_as_float(0x3AB60B61u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3C088889u));
  p = __fmaf_rn(p, r, __uint_as_float(0x3D2AAAABu));
  p = __fmaf_rn(p, r, __uint_as_float(0x3E2AAAABu));
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  float s = __uint_as_float((uint32_t)(ni + 127) << 23);
  return __fmul_rn(p, s);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Four rows (any row indices) x 64 columns of a 2-D tensor into four
// consecutive 128-byte rows of shared memory, with the map's swizzle; the
// bytes complete on `bar`.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, uint64_t* bar, int col, int r0,
                                            int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may park the thread until the phase completes, for up to
// `hint_ns` (the hardware wakes it when the phase completes): a waiting warp
// does not spin on the issue slots its sub-partition shares with the others.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false when the CTA abort flag is up or the wait ran
// past `limit_ns`; in the latter case it raises the abort flag and records
// DASH_DEV_TIMEOUT in the device error word.  After 8 polls the thread
// parks in the hinted try_wait (20 us at most per try) instead of spinning.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, DeviceError* err,
                                          int where, uint64_t limit_ns = 2000000000ull) {
  for (int i = 0; i < 8; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      record_error(err, DASH_DEV_TIMEOUT, where, (long long)parity);
      return false;
    }
  }
}

// Warp-uniform variant: every lane waits, the warp proceeds only if all lanes
// saw the phase complete (keeps the following .sync.aligned tcgen05 ops
// converged even when the abort flag is raised mid-wait).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag, DeviceError* err,
                                               int where) {
  bool ok = mbar_wait(bar, parity, abort_flag, err, where);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA: tiled 4-D load global -> shared, completion on an mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// L2 prefetch of one tile of a tensor map (no shared-memory destination)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}

// fire-and-forget fp32 reductions into global memory (no value returned)
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void red_add(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
               "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/fp16 in, fp32 acc)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive once on `bar` when every tcgen05 op issued so far by this thread is done
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// columns [col, col+32) of TMEM lane (warp_quarter*32 + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
// same as tmem_ld32, straight into fp32 registers
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]),
        "=f"(r[7]), "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]),
        "=f"(r[13]), "=f"(r[14]), "=f"(r[15]), "=f"(r[16]), "=f"(r[17]), "=f"(r[18]),
        "=f"(r[19]), "=f"(r[20]), "=f"(r[21]), "=f"(r[22]), "=f"(r[23]), "=f"(r[24]),
        "=f"(r[25]), "=f"(r[26]), "=f"(r[27]), "=f"(r[28]), "=f"(r[29]), "=f"(r[30]),
        "=f"(r[31])
      : "r"(taddr));
}

// D (TMEM) (+)= A (TMEM, K-major, 128 lanes) x B (shared-memory descriptor).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Per-warpgroup register split (all four warps of the warpgroup execute it).
// The host checks the kernel's launch register count covers every split.
template <int N>
__device__ __forceinline__ void regs_grow() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_shrink() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (canonical UMMA layouts):
//   K-major : rows of 128 B, 8-row atoms stacked every `sbo` bytes
//   MN-major: 128 B of MN per row, K rows; 8-row K groups every `sbo` bytes,
//             64-element MN atoms every `lbo` bytes
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B type `ab_fmt`
// (0 = f16, 1 = bf16), a/b major (0 = K, 1 = MN), M x N.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_fmt, uint32_t a_mn, uint32_t b_mn,
                                                  uint32_t M, uint32_t N) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn << 15) | (b_mn << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Packed fp32x2 arithmetic (sm_100): one instruction for two lanes of data.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(a), "f"(b));
  return v;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t fadd2_rn(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^y for a pair of values on the FMA pipe (offloads the MUFU unit).
// Cody-Waite split y = j + f with j = round(y) taken by adding and removing
// 1.5 * 2^23, |f| <= 1/2 exact, then 2^f from a degree-3 polynomial whose
// constant term is fixed to 1; c1..c3 are a relative-error least-squares fit
// made for this kernel on [-1/2, 1/2] (max relative error 1.0e-4, under a
// tenth of a bf16 ulp), and 2^j enters through the exponent field.  y is
// clamped to [-127, 64]: at -127 the result is exactly +0 (the exponent of
// 1.0 minus 127), above 64 it stays >= 2^64, which callers treat as overflow.
__device__ __forceinline__ uint64_t exp2_poly2(float y0, float y1) {
  constexpr float kShift = 12582912.0f;   // 1.5 * 2^23
  constexpr float c1 = 0.6932829022407532f, c2 = 0.24220998585224152f, c3 = 0.055008433759212494f;
  y0 = fminf(fmaxf(y0, -127.0f), 64.0f);
  y1 = fminf(fmaxf(y1, -127.0f), 64.0f);
  const uint64_t yv = f2_pack(y0, y1);
  const uint64_t t = fadd2_rn(yv, f2_pack(kShift, kShift));
  const uint64_t jf = fadd2_rn(t, f2_pack(-kShift, -kShift));
  const uint64_t fr = ffma2(jf, f2_pack(-1.0f, -1.0f), yv);
  uint64_t pv = ffma2(fr, f2_pack(c3, c3), f2_pack(c2, c2));
  pv = ffma2(pv, fr, f2_pack(c1, c1));
  pv = ffma2(pv, fr, f2_pack(1.0f, 1.0f));
  float p0, p1, t0, t1;
  f2_unpack(pv, p0, p1);
  f2_unpack(t, t0, t1);
  // low bits of t hold j (the shifter's own bits vanish in the shift)
  const uint32_t r0 = __float_as_uint(p0) + (__float_as_uint(t0) << 23);
  const uint32_t r1 = __float_as_uint(p1) + (__float_as_uint(t1) << 23);
  return f2_pack(__uint_as_float(r0), __uint_as_float(r1));
}

template <typename T> struct DType;
template <> struct DType<__nv_bfloat16> { static constexpr uint32_t fmt = 1; };
template <> struct DType<__half> { static constexpr uint32_t fmt = 0; };

__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack2(uint32_t u, __nv_bfloat16*) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(h);
}
__device__ __forceinline__ float2 unpack2(uint32_t u, __half*) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

}  // namespace dash
