// dash_backward.cu -- training backward of the DASH gather attention and of
// the 1.5-entmax prior, CUDA cores, fp32 arithmetic.
//
// Semantics (sparse_gather_e2e_triton.py:118-262, _e2e_attn_bwd_dq_kernel /
// _e2e_attn_bwd_dkv_kernel; autograd wrapper :307-337): for query token t and
// head h with lse[t,h] from the forward,
//   s_tj  = scale * q_t . k_j,  p_tj = exp(s_tj + bias_tb(j) - lse)   (kept keys)
//   dp_tj = do_t . v_j,         ds_tj = p_tj (dp_tj - delta_t),  delta_t = o_t . do_t
//   dq_t  = scale * sum_j ds_tj k_j,  dk_j = scale * sum_t ds_tj q_t,  dv_j = sum_t p_tj do_t
//   d_bias[t, slot of b] = sum over all heads and the remote keys of b of ds_tj
// Kept keys of row t: the local window (t - LW, t] (no bias) and, of every
// routed block b (first occurrence of an id, 0 <= b < blocks), the keys below
// t - LW + 1 (bias of b's slot); everything causal.
//
// Kernels:
//   bwd_flags_kernel   per (sequence, block) bitmask of the query rows that
//                      routed the block with at least one remote key
//   bwd_dq_kernel      one CTA per (token, kv head): delta, dq of the G query
//                      heads, d_bias (one atomic per 64-key tile and kv head)
//   bwd_dkv_kernel     one CTA per (64-key tile, kv head): walks the rows that
//                      routed the tile's block or reach it through their local
//                      window; dk and dv accumulate in registers, no atomics
// K/V tiles are staged in shared memory as fp32 rows of 132 floats (16-byte
// aligned rows; float4 reads of 8 consecutive rows fall in distinct banks).
//
// The entmax kernels restate dash_attention.py:637-658 (_Entmax15): forward
// z = (x - max)/2, tau solving sum relu(z - tau)^2 = 1 (support found by
// bisection, tau then from the closed form over the support), y = relu(z-tau)^2;
// backward g = sqrt(y), dx = dy*g - g * sum(dy*g) / max(sum g, 1e-12).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <climits>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {
namespace {

constexpr int BD = 128;       // head dim
constexpr int KT = 64;        // keys per tile
constexpr int KS = 132;       // fp32 row stride of a staged K/V tile
constexpr int kThreads = 128;

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ void st(float* p, float x) { *p = x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float4 ld4(const __half* p) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ float ld(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void st(__half* p, float x) { *p = __float2half_rn(x); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// rows [key0, key0 + KT) of one kv head -> fp32 tile; rows outside [0, nvalid) are 0
template <typename T>
__device__ __forceinline__ void stage_tile(float* dst, const T* base, int64_t row_stride, int key0,
                                           int nvalid) {
  for (int c = threadIdx.x; c < KT * (BD / 4); c += kThreads) {
    const int r = c >> 5, c4 = c & 31;
    const int key = key0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (key >= 0 && key < nvalid) v = Elem<T>::ld4(base + (int64_t)key * row_stride + 4 * c4);
    *reinterpret_cast<float4*>(dst + r * KS + 4 * c4) = v;
  }
}

// s and dp partial dot products of key j (thread tid & 63) over half
// (tid >> 6) of the head dim, for the G query rows in Qs / Ds
template <int G>
__device__ __forceinline__ void partial_scores(const float* Ks, const float* Vs, const float* Qs,
                                               const float* Ds, float* part) {
  const int j = threadIdx.x & (KT - 1), half = threadIdx.x >> 6;
  const float* kr = Ks + j * KS + half * 64;
  const float* vr = Vs + j * KS + half * 64;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float* qr = Qs + g * BD + half * 64;
    const float* dr = Ds + g * BD + half * 64;
    float as = 0.f, ap = 0.f;
#pragma unroll 4
    for (int c = 0; c < 64; c += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
      const float4 q4 = *reinterpret_cast<const float4*>(qr + c);
      const float4 v4 = *reinterpret_cast<const float4*>(vr + c);
      const float4 d4 = *reinterpret_cast<const float4*>(dr + c);
      as = fmaf(q4.x, k4.x, as); as = fmaf(q4.y, k4.y, as);
      as = fmaf(q4.z, k4.z, as); as = fmaf(q4.w, k4.w, as);
      ap = fmaf(d4.x, v4.x, ap); ap = fmaf(d4.y, v4.y, ap);
      ap = fmaf(d4.z, v4.z, ap); ap = fmaf(d4.w, v4.w, ap);
    }
    part[(0 * 2 + half) * G * KT + g * KT + j] = as;
    part[(1 * 2 + half) * G * KT + g * KT + j] = ap;
  }
}

// ---------------------------------------------------------------------------
// (with several index heads: one bitmask per (sequence, index head, block);
// with segment starts: blocks holding a key in [seg_start, remote bound))
__global__ void __launch_bounds__(kThreads) bwd_flags_kernel(DashAttnBwdArgs a, int nblk, int words) {
  const int64_t row = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int T = a.seq_len;
  if (row >= (int64_t)a.n_seq * T) return;
  const int s = (int)(row / T), t = (int)(row - (int64_t)s * T);
  const int HI = a.n_index_heads > 1 ? a.n_index_heads : 1;
  const int64_t seg = a.seg_start ? (int64_t)a.seg_start[row] : 0;
  const int64_t ls = max((int64_t)t - a.local_window + 1, seg);
  for (int ih = 0; ih < HI; ++ih) {
    const int64_t rr = ((int64_t)s * HI + ih) * T + t;
    const int32_t* ids = a.idx + rr * a.K;
    for (int j = 0; j < a.K; ++j) {
      const int b = ids[j];
      if (b < 0 || b >= nblk || (int64_t)b * a.block_size >= ls || (int64_t)(b + 1) * a.block_size <= seg) continue;
      bool dup = false;
      for (int j2 = 0; j2 < j && !dup; ++j2) dup = ids[j2] == b;
      if (dup) continue;
      atomicOr(a.flags + (((int64_t)s * HI + ih) * nblk + b) * words + (t >> 5), 1u << (t & 31));
    }
  }
}

// ---------------------------------------------------------------------------
template <typename E, int G>
__global__ void __launch_bounds__(kThreads) bwd_dq_kernel(DashAttnBwdArgs a, int nblk) {
  extern __shared__ float4 smem_f4[];
  float* Ks = reinterpret_cast<float*>(smem_f4);
  float* Vs = Ks + KT * KS;
  float* Qs = Vs + KT * KS;            // [G][BD]
  float* Ds = Qs + G * BD;             // [G][BD]
  float* part = Ds + G * BD;           // [2][2][G][KT]
  float* DSs = part + 4 * G * KT;      // [G][KT]
  float* red = DSs + G * KT;           // [4 warps][G]
  float* lse_s = red + 4 * G;          // [G]
  float* del_s = lse_s + G;            // [G]
  float* sbias = del_s + G;            // [K]
  int* sblk = reinterpret_cast<int*>(sbias + a.K);   // [K] kept block per slot, -1 dropped

  const int T = a.seq_len, HQ = a.n_heads, H = a.n_kv_heads;
  const int64_t row = blockIdx.x;
  const int h = blockIdx.y;
  const int s = (int)(row / T), t = (int)(row - (int64_t)s * T);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const E* qb = reinterpret_cast<const E*>(a.q);
  const E* ob = reinterpret_cast<const E*>(a.o);
  const E* dob = reinterpret_cast<const E*>(a.dout);
  const E* kb = reinterpret_cast<const E*>(a.k) + ((int64_t)s * T * H + h) * BD;
  const E* vb = reinterpret_cast<const E*>(a.v) + ((int64_t)s * T * H + h) * BD;
  const int64_t kv_row = (int64_t)H * BD;

  // ---- the G query rows, delta, lse, kept slots ----
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int64_t off = (row * HQ + h * G + g) * BD + tid;
    const float dv = Elem<E>::ld(dob + off);
    Qs[g * BD + tid] = Elem<E>::ld(qb + off);
    Ds[g * BD + tid] = dv;
    const float od = warp_sum(Elem<E>::ld(ob + off) * dv);
    if (lane == 0) red[warp * G + g] = od;
  }
  const int64_t ls = (int64_t)t - a.local_window + 1;
  for (int j = tid; j < a.K; j += kThreads) {
    const int32_t* ids = a.idx + row * a.K;
    const int b = ids[j];
    bool keep = b >= 0 && b < nblk && (int64_t)b * a.block_size < ls;
    for (int j2 = 0; j2 < j && keep; ++j2) keep = ids[j2] != b;
    sblk[j] = keep ? b : -1;
    sbias[j] = a.bias ? a.bias[row * a.K + j] : 0.f;
  }
  __syncthreads();
  if (tid < G) {
    const float d = red[tid] + red[G + tid] + red[2 * G + tid] + red[3 * G + tid];
    del_s[tid] = d;
    lse_s[tid] = a.lse[row * HQ + h * G + tid];
    a.delta[row * HQ + h * G + tid] = d;
  }
  __syncthreads();

  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.f;

  // one 64-key tile: keys [lo, hi] of the tile starting at key0 are kept
  auto tile = [&](int key0, int lo, int hi, float bias, int slot) {
    __syncthreads();
    stage_tile<E>(Ks, kb, kv_row, key0, hi + 1);
    stage_tile<E>(Vs, vb, kv_row, key0, hi + 1);
    __syncthreads();
    partial_scores<G>(Ks, Vs, Qs, Ds, part);
    __syncthreads();
    if (tid < KT) {
      const int key = key0 + tid;
      const bool kept = key >= lo && key <= hi;
      float dsum = 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float sc = part[g * KT + tid] + part[G * KT + g * KT + tid];
        const float dp = part[2 * G * KT + g * KT + tid] + part[3 * G * KT + g * KT + tid];
        const float p = kept ? expf(fmaf(sc, a.scale, bias) - lse_s[g]) : 0.f;
        const float ds = p * (dp - del_s[g]);
        DSs[g * KT + tid] = ds;
        dsum += ds;
      }
      if (slot >= 0 && a.d_bias) {
        dsum = warp_sum(dsum);
        if (lane == 0) red_add(a.d_bias + row * a.K + slot, dsum);
      }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float* dsr = DSs + g * KT;
      float v = acc[g];
#pragma unroll 8
      for (int j = 0; j < KT; ++j) v = fmaf(dsr[j], Ks[j * KS + tid], v);
      acc[g] = v;
    }
  };

  // routed blocks, slot order: keys of block b below the local window
  const int bs = a.block_size;
  for (int j = 0; j < a.K; ++j) {
    const int b = sblk[j];
    if (b < 0) continue;
    const int64_t bend = min((int64_t)(b + 1) * bs, ls);   // exclusive
    for (int64_t k0 = (int64_t)b * bs; k0 < bend; k0 += KT)
      tile((int)k0, (int)k0, (int)min(k0 + KT, bend) - 1, sbias[j], j);
  }
  // local window (t - LW, t]
  for (int64_t k0 = max(ls, (int64_t)0); k0 <= t; k0 += KT)
    tile((int)k0, (int)k0, (int)min(k0 + KT - 1, (int64_t)t), 0.f, -1);

  E* dqb = reinterpret_cast<E*>(a.dq);
#pragma unroll
  for (int g = 0; g < G; ++g) Elem<E>::st(dqb + (row * HQ + h * G + g) * BD + tid, acc[g] * a.scale);
}

// ---------------------------------------------------------------------------
template <typename E, int G>
__global__ void __launch_bounds__(kThreads) bwd_dkv_kernel(DashAttnBwdArgs a, int nblk, int words,
                                                           int ntiles) {
  extern __shared__ float4 smem_f4[];
  float* Ks = reinterpret_cast<float*>(smem_f4);
  float* Vs = Ks + KT * KS;
  float* Qs = Vs + KT * KS;            // [G][BD]
  float* Ds = Qs + G * BD;             // [G][BD]
  float* part = Ds + G * BD;           // [2][2][G][KT]
  float* Ps = part + 4 * G * KT;       // [G][KT]
  float* DSs = Ps + G * KT;            // [G][KT]
  float* lse_s = DSs + G * KT;         // [G]
  float* del_s = lse_s + G;            // [G]
  float* misc = del_s + G;             // [0] bias of the row's slot of this block

  const int T = a.seq_len, HQ = a.n_heads, H = a.n_kv_heads;
  const int s = blockIdx.x / ntiles, tl = blockIdx.x - s * ntiles;
  const int h = blockIdx.y;
  const int key0 = tl * KT;
  const int b = key0 / a.block_size;
  const int tid = threadIdx.x, lane = tid & 31;
  const int j = tid & (KT - 1), half = tid >> 6;
  const int LW = a.local_window;
  const int64_t kvoff = ((int64_t)s * T * H + h) * BD;
  const E* qb = reinterpret_cast<const E*>(a.q);
  const E* dob = reinterpret_cast<const E*>(a.dout);
  const int64_t kv_row = (int64_t)H * BD;
  stage_tile<E>(Ks, reinterpret_cast<const E*>(a.k) + kvoff, kv_row, key0, T);
  stage_tile<E>(Vs, reinterpret_cast<const E*>(a.v) + kvoff, kv_row, key0, T);

  float dk[64], dv[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) { dk[c] = 0.f; dv[c] = 0.f; }

  // a 64-key tile holds at most two blocks (block sizes are multiples of 32):
  // b and b2 (= b when the tile lies in one block); keys from j2 on are b2's
  const int b2 = min(key0 + KT - 1, T - 1) / a.block_size;
  const int j2 = b2 != b ? b2 * a.block_size - key0 : KT;
  const uint32_t* fl = a.flags + ((int64_t)s * nblk + b) * words;
  const uint32_t* fl2 = a.flags + ((int64_t)s * nblk + b2) * words;
  // rows whose window reaches a key of the tile: [key0, key0 + KT - 1 + LW - 1]
  const int64_t loc_end = min((int64_t)key0 + KT - 1 + LW - 1, (int64_t)T - 1);
  for (int w = key0 >> 5; w < words; ++w) {
    uint32_t m = fl[w] | fl2[w];
    const int64_t r0 = (int64_t)w * 32;
    if (r0 <= loc_end) {
      const int64_t lo = max(r0, (int64_t)key0), hi = min(r0 + 31, loc_end);
      if (lo <= hi) {
        const int nb = (int)(hi - lo + 1);
        const uint32_t span = nb == 32 ? 0xffffffffu : ((1u << nb) - 1u);
        m |= span << (int)(lo - r0);
      }
    }
    m &= (r0 + 31 < key0) ? 0u : (key0 > r0 ? ~((1u << (key0 - r0)) - 1u) : 0xffffffffu);
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      const int i = (int)(r0 + bit);
      if (i >= T) break;
      const bool routed = (fl[w] >> bit) & 1u;
      const bool routed2 = b2 != b && ((fl2[w] >> bit) & 1u);
      const int64_t row = (int64_t)s * T + i;
      __syncthreads();
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int64_t off = (row * HQ + h * G + g) * BD + tid;
        Qs[g * BD + tid] = Elem<E>::ld(qb + off);
        Ds[g * BD + tid] = Elem<E>::ld(dob + off);
      }
      if (tid < G) {
        lse_s[tid] = a.lse[row * HQ + h * G + tid];
        del_s[tid] = a.delta[row * HQ + h * G + tid];
      }
      if (tid < 64) {
        // bias of the first slot holding b (warp 0) / b2 (warp 1)
        const int bb = tid < 32 ? b : b2;
        const bool rt = tid < 32 ? routed : routed2;
        float bias = 0.f;
        if (rt && a.bias) {
          int first = INT_MAX;
          for (int jj = lane; jj < a.K; jj += 32)
            if (a.idx[row * a.K + jj] == bb) { first = jj; break; }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
          if (first != INT_MAX) bias = a.bias[row * a.K + first];
        }
        if (lane == 0) misc[tid >> 5] = bias;
      }
      __syncthreads();
      partial_scores<G>(Ks, Vs, Qs, Ds, part);
      __syncthreads();
      if (tid < KT) {
        const int key = key0 + tid;
        const int64_t ls = (int64_t)i - LW + 1;
        const bool second = tid >= j2;
        const bool local = key < T && key <= i && key >= ls;
        const bool remote = (second ? routed2 : routed) && key < T && key < ls;
        const float bias = remote ? misc[second ? 1 : 0] : 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float sc = part[g * KT + tid] + part[G * KT + g * KT + tid];
          const float dp = part[2 * G * KT + g * KT + tid] + part[3 * G * KT + g * KT + tid];
          const float p = (local || remote) ? expf(fmaf(sc, a.scale, bias) - lse_s[g]) : 0.f;
          Ps[g * KT + tid] = p;
          DSs[g * KT + tid] = p * (dp - del_s[g]);
        }
      }
      __syncthreads();
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = Ps[g * KT + j], dsj = DSs[g * KT + j];
        const float* qr = Qs + g * BD + half * 64;
        const float* dr = Ds + g * BD + half * 64;
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          const float4 q4 = *reinterpret_cast<const float4*>(qr + c);
          const float4 d4 = *reinterpret_cast<const float4*>(dr + c);
          dk[c] = fmaf(dsj, q4.x, dk[c]); dk[c + 1] = fmaf(dsj, q4.y, dk[c + 1]);
          dk[c + 2] = fmaf(dsj, q4.z, dk[c + 2]); dk[c + 3] = fmaf(dsj, q4.w, dk[c + 3]);
          dv[c] = fmaf(pj, d4.x, dv[c]); dv[c + 1] = fmaf(pj, d4.y, dv[c + 1]);
          dv[c + 2] = fmaf(pj, d4.z, dv[c + 2]); dv[c + 3] = fmaf(pj, d4.w, dv[c + 3]);
        }
      }
    }
  }
  const int key = key0 + j;
  if (key < T) {
    E* dkb = reinterpret_cast<E*>(a.dk) + kvoff + (int64_t)key * kv_row + half * 64;
    E* dvb = reinterpret_cast<E*>(a.dv) + kvoff + (int64_t)key * kv_row + half * 64;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      Elem<E>::st(dkb + c, dk[c] * a.scale);
      Elem<E>::st(dvb + c, dv[c]);
    }
  }
}

// ---------------------------------------------------------------------------
// 1.5-entmax, one warp per row
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) entmax15_fwd_kernel(DashEntmaxArgs a) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  const float* x = a.x + row * a.stride;
  float* y = a.y + row * a.stride;
  const int n = a.n;
  float mx = -INFINITY;
  for (int i = lane; i < n; i += 32) mx = fmaxf(mx, x[i]);
  mx = warp_max(mx);
  // z = (x - max)/2 <= 0 and sum relu(z - tau)^2 is 0 at tau = 0 and >= 1 at
  // tau = -1: bisection keeps f(lo) >= 1 > f(hi)
  float lo = -1.f, hi = 0.f;
  for (int it = 0; it < 32; ++it) {
    const float mid = 0.5f * (lo + hi);
    float f = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float d = (x[i] - mx) * 0.5f - mid;
      if (d > 0.f) f = fmaf(d, d, f);
    }
    f = warp_sum(f);
    if (f >= 1.f) lo = mid; else hi = mid;
  }
  // closed form over the support {z > lo} (an element at tau itself adds 0)
  float k = 0.f, s1 = 0.f, s2 = 0.f;
  for (int i = lane; i < n; i += 32) {
    const float z = (x[i] - mx) * 0.5f;
    if (z > lo) { k += 1.f; s1 += z; s2 = fmaf(z, z, s2); }
  }
  k = warp_sum(k); s1 = warp_sum(s1); s2 = warp_sum(s2);
  k = fmaxf(k, 1.f);
  const float mean = s1 / k, mean_sq = s2 / k;
  const float ss = k * (mean_sq - mean * mean);
  const float tau = mean - sqrtf(fmaxf((1.f - ss) / k, 0.f));
  for (int i = lane; i < n; i += 32) {
    const float d = fmaxf((x[i] - mx) * 0.5f - tau, 0.f);
    y[i] = d * d;
  }
}

__global__ void __launch_bounds__(256) entmax15_bwd_kernel(DashEntmaxArgs a) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  const float* y = a.y + row * a.stride;
  const float* dy = a.dy + row * a.stride;
  float* dx = a.dx + row * a.stride;
  float sdx = 0.f, sg = 0.f;
  for (int i = lane; i < a.n; i += 32) {
    const float g = sqrtf(y[i]);
    sdx = fmaf(dy[i], g, sdx);
    sg += g;
  }
  sdx = warp_sum(sdx);
  sg = warp_sum(sg);
  const float q = sdx / fmaxf(sg, 1e-12f);
  for (int i = lane; i < a.n; i += 32) {
    const float g = sqrtf(y[i]);
    dx[i] = dy[i] * g - q * g;
  }
}

size_t dq_smem(int G, int K) {
  return (size_t)(2 * KT * KS + 2 * G * BD + 5 * G * KT + 6 * G) * 4 + (size_t)K * 8;
}
size_t dkv_smem(int G) {
  return (size_t)(2 * KT * KS + 2 * G * BD + 6 * G * KT + 2 * G + 4) * 4;
}

template <typename E, int G>
int launch_bwd_typed(const DashAttnBwdArgs& a, int nblk, int words, cudaStream_t st) {
  const size_t sq = dq_smem(G, a.K), skv = dkv_smem(G);
  // per device and function; cheap, and allowed while a graph is captured
  cudaFuncSetAttribute(bwd_dq_kernel<E, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sq);
  cudaFuncSetAttribute(bwd_dkv_kernel<E, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)skv);
  const int64_t rows = (int64_t)a.n_seq * a.seq_len;
  bwd_dq_kernel<E, G><<<dim3((unsigned)rows, (unsigned)a.n_kv_heads), kThreads, sq, st>>>(a, nblk);
  count_launch();
  int rc = check_launch("bwd_dq_kernel");
  if (rc) return rc;
  const int ntiles = (a.seq_len + KT - 1) / KT;
  bwd_dkv_kernel<E, G><<<dim3((unsigned)(a.n_seq * ntiles), (unsigned)a.n_kv_heads), kThreads, skv, st>>>(
      a, nblk, words, ntiles);
  count_launch();
  return check_launch("bwd_dkv_kernel");
}

template <typename E>
int launch_bwd_g(const DashAttnBwdArgs& a, int G, int nblk, int words, cudaStream_t st) {
  switch (G) {
    case 1: return launch_bwd_typed<E, 1>(a, nblk, words, st);
    case 2: return launch_bwd_typed<E, 2>(a, nblk, words, st);
    case 4: return launch_bwd_typed<E, 4>(a, nblk, words, st);
    case 8: return launch_bwd_typed<E, 8>(a, nblk, words, st);
    default: return set_error(DASH_ERR_UNSUPPORTED, "query heads per kv head %d not in {1,2,4,8}", G);
  }
}

}  // namespace

size_t attn_bwd_flag_words(const DashAttnBwdArgs& a) {
  const int64_t nblk = (a.seq_len + a.block_size - 1) / a.block_size;
  const int64_t words = (a.seq_len + 31) / 32;
  const int64_t HI = a.n_index_heads > 1 ? a.n_index_heads : 1;
  return (size_t)(a.n_seq * HI * nblk * words);
}

int launch_attn_bwd(const DashAttnBwdArgs& a, cudaStream_t st) {
  const int64_t rows = (int64_t)a.n_seq * a.seq_len;
  if (rows == 0) return DASH_OK;
  const int nblk = (a.seq_len + a.block_size - 1) / a.block_size;
  const int words = (a.seq_len + 31) / 32;
  if (cudaMemsetAsync(a.flags, 0, attn_bwd_flag_words(a) * 4, st) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "memset of the row flags failed");
  if (a.d_bias && cudaMemsetAsync(a.d_bias, 0, (size_t)rows * (a.n_index_heads > 1 ? a.n_index_heads : 1) * a.K * 4, st) != cudaSuccess)
    return set_error(DASH_ERR_CUDA, "memset of d_bias failed");
  bwd_flags_kernel<<<(unsigned)((rows + kThreads - 1) / kThreads), kThreads, 0, st>>>(a, nblk, words);
  count_launch();
  int rc = check_launch("bwd_flags_kernel");
  if (rc) return rc;
  // 16-bit inputs: tensor cores (dash_backward_tc.cu); fp32: the kernels above
  if (a.dtype == DASH_DTYPE_BF16 || a.dtype == DASH_DTYPE_F16) return launch_attn_bwd_tc(a, nblk, words, st);
  return launch_bwd_g<float>(a, a.n_heads / a.n_kv_heads, nblk, words, st);
}

int launch_entmax15(const DashEntmaxArgs& a, bool backward, cudaStream_t st) {
  if (a.rows == 0 || a.n == 0) return DASH_OK;
  const unsigned grid = (unsigned)((a.rows + 7) / 8);
  if (backward) entmax15_bwd_kernel<<<grid, 256, 0, st>>>(a);
  else entmax15_fwd_kernel<<<grid, 256, 0, st>>>(a);
  count_launch();
  return check_launch(backward ? "entmax15_bwd_kernel" : "entmax15_fwd_kernel");
}

}  // namespace dash
