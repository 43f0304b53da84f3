// dash_prefill_f32.cu -- DASH prefill gather attention in fp32 on CUDA cores.
//
// For fp32 q/k/v (the reference computes its fp32 path with tl.dot at tf32 or
// better, sparse_gather_e2e_triton.py:77,85, and its dense torch path in
// fp32): every product and sum here is an fp32 FMA, so results match an fp32
// reference to ~1e-6 relative instead of bf16's 2e-2.  Contiguous K/V only
// (the paged serving caches are bf16/fp16).
//
// One warp per query row (token, query head); 8 warps per CTA take 8
// consecutive rows of one head.  The row's keys are its local window
// (max(pos - LW + 1, seg) .. pos, no bias) and, for each block of its
// canonical routed list (plan_kernel: deduplicated, ascending, only blocks
// with a key below the window), the block's keys below the window (+ bias).
// Keys go 32 at a time: lane j scores key j (full 128-dim dot product, q
// staged in shared memory, K row read with 16-byte loads), the warp takes the
// chunk max and rescales its running sums (online softmax in the exp2
// domain), then every lane accumulates 4 output dims over the chunk's keys
// (P broadcast by shuffles, V rows read coalesced).
//
// Semantics: sparse_gather_e2e_triton.py:34-115 (per-row key rule and bias),
// dash_attention.py:980-1006 (_forward_dense, the fp32 torch form).
#include <cmath>

#include "dash_common.cuh"
#include "dash_internal.h"
#include "dash_prefill_plan.cuh"

namespace dash {

constexpr int kF32Warps = 8;
constexpr int kF32D = 128;

// sequence of a flat query row: fixed layout by division, packed layout by a
// binary search of the row starts
__device__ __forceinline__ int seq_of_row(const DashSeqs& q, int64_t r) {
  if (!q.q_start) return (int)(r / (q.q_len_fixed > 0 ? q.q_len_fixed : 1));
  int lo = 0, hi = q.n_seq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q.q_start[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kF32Warps * 32) prefill_f32_kernel(const DashPrefillArgs a,
                                                                     const PrefillPlan p) {
  __shared__ __align__(16) float s_q[kF32Warps][kF32D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kF32Warps + warp;
  if (r >= p.n_rows) return;                       // whole warps leave together
  const int hq = blockIdx.y;
  const int hk = hq / p.G;
  const int H = a.qo.n_heads;
  const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
  const int ih = (hk * p.G) / (H / nih);
  const int s = seq_of_row(a.seqs, r);
  const int i = (int)(r - row_base(a.seqs, s));
  const int kvl = kv_len_of(a.seqs, s);
  const int pos = pos0_of(a.seqs, s) + i;
  const int seg = a.seg_start ? a.seg_start[r] : 0;
  const int lstart = pos - a.local_window + 1;
  const float LOG2E = 1.4426950408889634f;
  const float sl2 = a.scale * LOG2E;

  const float* qrow = reinterpret_cast<const float*>(a.qo.q) +
                      (a.seqs.q_start ? r * a.qo.q_stride_tok
                                      : (int64_t)s * a.qo.q_stride_seq + (int64_t)i * a.qo.q_stride_tok) +
                      (int64_t)hq * a.qo.q_stride_head;
  {
    const float4 v = reinterpret_cast<const float4*>(qrow)[lane];
    reinterpret_cast<float4*>(s_q[warp])[lane] = make_float4(v.x * sl2, v.y * sl2, v.z * sl2, v.w * sl2);
  }
  __syncwarp();
  const float* kbase = reinterpret_cast<const float*>(a.kv.k) + (int64_t)s * a.kv.stride_seq +
                       (int64_t)hk * a.kv.stride_head;
  const float* vbase = reinterpret_cast<const float*>(a.kv.v) + (int64_t)s * a.kv.stride_seq +
                       (int64_t)hk * a.kv.stride_head;
  const float4* sq4 = reinterpret_cast<const float4*>(s_q[warp]);

  float m_run = -INFINITY, l_lane = 0.0f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  // keys [k0, k1) with additive term add (log2 domain)
  auto run = [&](int k0, int k1, float add) {
    for (int kk = k0; kk < k1; kk += 32) {
      const int key = kk + lane;
      float x = -INFINITY;
      if (key < k1) {
        const float4* kr = reinterpret_cast<const float4*>(kbase + (int64_t)key * a.kv.stride_tok);
        float acc = 0.0f;
#pragma unroll 8
        for (int c = 0; c < kF32D / 4; ++c) {
          const float4 kv = kr[c], qv = sq4[c];
          acc = fmaf(qv.x, kv.x, acc);
          acc = fmaf(qv.y, kv.y, acc);
          acc = fmaf(qv.z, kv.z, acc);
          acc = fmaf(qv.w, kv.w, acc);
        }
        x = acc + add;
      }
      float mc = x;
      for (int off = 16; off > 0; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
      const float m_new = fmaxf(m_run, mc);
      if (m_new == -INFINITY) continue;              // nothing kept yet (uniform per warp)
      const float alpha = exp2f(m_run - m_new);      // exp2(-inf) = 0 on the first chunk
      l_lane *= alpha;
      o.x *= alpha; o.y *= alpha; o.z *= alpha; o.w *= alpha;
      m_run = m_new;
      const float pj = exp2f(x - m_new);
      l_lane += pj;
      const int n = min(32, k1 - kk);
      for (int t = 0; t < n; ++t) {
        const float pt = __shfl_sync(0xffffffffu, pj, t);
        const float4 vv = reinterpret_cast<const float4*>(vbase + (int64_t)(kk + t) * a.kv.stride_tok)[lane];
        o.x = fmaf(pt, vv.x, o.x);
        o.y = fmaf(pt, vv.y, o.y);
        o.z = fmaf(pt, vv.z, o.z);
        o.w = fmaf(pt, vv.w, o.w);
      }
    }
  };
  // routed blocks below the window, then the window
  const int K = a.routes.K;
  const int64_t lrow = (int64_t)ih * p.n_rows + r;
  const int32_t* rl = p.cidx + lrow * K;
  const float* rb = p.cbias + lrow * K;
  const int bs = a.block_size;
  for (int j = 0; j < K; ++j) {
    const int b = rl[j];
    if (b < 0) break;
    const int k0 = max(b * bs, seg);
    const int k1 = min(min((b + 1) * bs, lstart), kvl);
    if (k0 < k1) run(k0, k1, rb[j] * LOG2E);
  }
  run(max(max(lstart, seg), 0), min(pos + 1, kvl), 0.0f);

  float l = l_lane;
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  float* orow = reinterpret_cast<float*>(a.qo.out) +
                (a.seqs.q_start ? r * a.qo.o_stride_tok
                                : (int64_t)s * a.qo.o_stride_seq + (int64_t)i * a.qo.o_stride_tok) +
                (int64_t)hq * a.qo.o_stride_head;
  reinterpret_cast<float4*>(orow)[lane] = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
  if (lane == 0 && a.qo.lse) {
    const float lse = l > 0.0f ? (m_run + log2f(l)) * 0.6931471805599453f : -INFINITY;
    a.qo.lse[(a.seqs.q_start ? r * a.qo.lse_stride_tok
                             : (int64_t)s * a.qo.lse_stride_seq + (int64_t)i * a.qo.lse_stride_tok) +
             (int64_t)hq * a.qo.lse_stride_head] = lse;
  }
}

int launch_prefill_f32(const DashPrefillArgs& a, const PrefillPlan& p, cudaStream_t st) {
  dim3 grid((unsigned)((p.n_rows + kF32Warps - 1) / kF32Warps), a.qo.n_heads);
  prefill_f32_kernel<<<grid, kF32Warps * 32, 0, st>>>(a, p);
  count_launch();
  return check_launch("prefill_f32_kernel");
}

}  // namespace dash
