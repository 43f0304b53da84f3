// dash_router.cu -- DASH router kernels (CUDA cores, fp32):
//   kbar_pool_kernel   stage-0 head_cls pooling of index keys (k-bar)
//   route_rows_kernel  block scores + candidate mask + 1.5-entmax + top-K + bias
//   block_max_kernel   indexer-mode stage-0 block-max scores
//
// Bit-exactness: every dot product is a sequential __fmaf_rn chain over the
// feature index and every other rounding step is spelled out, in the same
// order as oracle/dash_oracle.c, so k-bar, block scores and the selected block
// lists are bitwise equal to the CPU oracle.
#include <cooperative_groups.h>
#include <type_traits>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {

namespace cg = cooperative_groups;

constexpr float kScoreNeg = -1.0e9f;
constexpr float kEntmaxNeg = -1.0e4f;

// ---------------------------------------------------------------------------
// k-bar pooling: one CTA per block (contiguous) or plan entry (paged).
// Restates dash_attention.py:863-888 / route_triton.py:36-72.
// DC > 0 fixes the index dim at compile time (loops unroll, shared-memory
// operands are fetched ahead of the fixed-order FMA chains); VEC stages the
// keys with 16-byte loads.  The arithmetic order is the same in every form.
// ---------------------------------------------------------------------------
// One k-bar row: the first n tokens at element offset `base` of a.keys ->
// a.kbar row out_row.  All 128 threads of the CTA take part (barriers).
template <typename KT, int DC, bool VEC>
__device__ __forceinline__ void kbar_pool_body(const DashKbarArgs& a, float* sm, int n, int64_t base,
                                               int64_t out_row) {
  const int d = DC > 0 ? DC : a.d;
  const int ld = d + 1;                       // padded row, conflict-free column reads
  float* sk = sm;                             // [bs][d+1]
  float* shc = sk + a.block_size * ld;        // [d]
  float* se = shc + d;                        // [bs]
  float* sred = se + a.block_size;            // [4]
  const KT* keys = reinterpret_cast<const KT*>(a.keys);
  if constexpr (VEC) {
    // 16-byte vectors of W elements; every load of a thread is issued before
    // its first shared-memory store
    constexpr int W = 16 / (int)sizeof(KT);
    const int dv = d / W;
    const int tot = n * dv;
#pragma unroll 16
    for (int e = threadIdx.x; e < tot; e += 128) {
      const int j = e / dv, cv = e - j * dv;
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(keys + base + (int64_t)j * a.tok_stride) + cv);
      const KT* v = reinterpret_cast<const KT*>(&raw);
#pragma unroll
      for (int k = 0; k < W; ++k) sk[j * ld + cv * W + k] = (float)v[k];
    }
  } else {
#pragma unroll 8
    for (int e = threadIdx.x; e < n * d; e += 128) {
      int j = e / d, c = e - j * d;
      sk[j * ld + c] = (float)__ldg(keys + base + (int64_t)j * a.tok_stride + c);
    }
  }
  for (int c = threadIdx.x; c < d; c += blockDim.x) shc[c] = a.head_cls ? a.head_cls[c] : 0.0f;
  __syncthreads();
  const float inv_sqrt_d = (float)(1.0 / sqrt((double)d));
  float lmax = -INFINITY;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    float acc = 0.0f;
#pragma unroll 16
    for (int c = 0; c < d; ++c) acc = __fmaf_rn(sk[j * ld + c], shc[c], acc);
    float aw = clamp_act(__fmul_rn(acc, inv_sqrt_d));
    se[j] = aw;
    lmax = fmaxf(lmax, aw);
  }
  for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
  if ((threadIdx.x & 31) == 0) sred[threadIdx.x >> 5] = lmax;
  __syncthreads();
  float rmax = fmaxf(fmaxf(sred[0], sred[1]), fmaxf(sred[2], sred[3]));
  if (n <= 0) rmax = 0.0f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) se[j] = det_expf(__fsub_rn(se[j], rmax));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
#pragma unroll 16
    for (int j = 0; j < n; ++j) sum = __fadd_rn(sum, se[j]);
    sred[0] = sum > 1e-6f ? sum : 1e-6f;
  }
  __syncthreads();
  const float den = sred[0];
  for (int j = threadIdx.x; j < n; j += blockDim.x) se[j] = __fdiv_rn(se[j], den);
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.0f;
#pragma unroll 16
    for (int j = 0; j < n; ++j) acc = __fmaf_rn(se[j], sk[j * ld + c], acc);
    if (!(acc == acc) || isinf(acc)) acc = 0.0f;
    a.kbar[out_row * a.kbar_row_stride + c] = acc;
  }
}

// Shared memory of kbar_pool_body, in floats.
__host__ __device__ inline size_t kbar_pool_smem_floats(int block_size, int d) {
  return (size_t)block_size * (d + 1) + d + block_size + 4;
}

// Plan entry i of a paged pool: false when it is not a page slot (ntok <= 0,
// route_triton.py:69-72).
__device__ __forceinline__ bool kbar_paged_entry(const DashKbarArgs& a, int i, int& n, int64_t& base,
                                                 int64_t& out_row) {
  n = a.ntok[i];
  if (n <= 0) return false;
  if (n > a.block_size) n = a.block_size;
  base = a.pages[i] * a.page_stride;
  out_row = a.pages[i];
  return true;
}

template <typename KT, int DC, bool VEC>
__global__ void __launch_bounds__(128) kbar_pool_kernel(const __grid_constant__ DashKbarArgs a) {
  extern __shared__ float sm[];
  int n;
  int64_t base, out_row;
  if (a.pages == nullptr) {
    int b = blockIdx.x, s = blockIdx.y;
    n = a.seq_len - b * a.block_size;
    if (n > a.block_size) n = a.block_size;
    base = (int64_t)s * a.seq_stride + (int64_t)b * a.block_size * a.tok_stride;
    out_row = (int64_t)s * a.kbar_seq_rows + b;
  } else if (!kbar_paged_entry(a, blockIdx.x, n, base, out_row)) {
    return;
  }
  kbar_pool_body<KT, DC, VEC>(a, sm, n, base, out_row);
}

// ---------------------------------------------------------------------------
// Row -> (sequence, position) for the DashSeqs packing.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void row_to_seq(const DashSeqs& q, int64_t r, int& s, int& i) {
  if (q.q_start == nullptr) {
    s = (int)(r / q.q_len_fixed);
    i = (int)(r - (int64_t)s * q.q_len_fixed);
    return;
  }
  int lo = 0, hi = q.n_seq - 1;                 // last s with q_start[s] <= r
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (q.q_start[mid] <= r) lo = mid; else hi = mid - 1;
  }
  s = lo;
  i = (int)(r - q.q_start[lo]);
}
__device__ __forceinline__ int seq_kv_len(const DashSeqs& q, int s) {
  return q.kv_len ? q.kv_len[s] : q.kv_len_fixed;
}
__device__ __forceinline__ int seq_q_len(const DashSeqs& q, int s) {
  return q.q_start ? (q.q_start[s + 1] - q.q_start[s]) : q.q_len_fixed;
}
__device__ __forceinline__ int64_t seq_pos(const DashSeqs& q, int s, int i) {
  int p0 = q.pos0 ? q.pos0[s] : seq_kv_len(q, s) - seq_q_len(q, s);
  return (int64_t)p0 + i;
}

__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------
// Routing: one warp per query row.
// Restates modeling_deepseekv2.py:309-333 + 351-388 (and WHL dash_router.py
// route_and_select): cand = remote & mask (fallback remote); x = cand ? z*scale
// : -1e4; top-M by (x desc, id asc) via a radix select on the order-preserving
// key; entmax tau by the sort-based formula over the ranked top-M; first K by
// rank; bias = (log max(p,floor) - mean)/sigma
// over the valid (candidate) slots; ascending pack with -1 tail.
// ---------------------------------------------------------------------------
constexpr int kRouteWarps = 4;
constexpr int kMaxM = 256;

// Scores of blocks b = t0, t0+step, ... of one row into sx.  Four blocks are
// in flight per thread (four independent accumulators); each dot product is
// still one sequential __fmaf_rn chain over the feature index.
__device__ __forceinline__ void score_blocks(const DashRouteArgs& a, const float* sq, float* sx,
                                             int s, int64_t qblk, int kvl, int t0, int step) {
  const int W = a.width;
  const float inv_sqrt_d = (float)(1.0 / sqrt((double)a.d));
  for (int b0 = t0; b0 < W; b0 += 4 * step) {
    const float4* kb[4];
    bool live[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + u * step;
      live[u] = b < W && (int64_t)b <= qblk - a.local_blocks && (int64_t)b * a.block_size < kvl;
      kb[u] = nullptr;
      if (live[u]) {
        int64_t kr = a.block_table ? (int64_t)a.block_table[(int64_t)s * a.bt_stride + b]
                                   : (int64_t)s * a.kbar_seq_rows + b;
        if (kr < 0 || kr >= a.num_kbar_rows) {
          record_error(a.device_error, DASH_DEV_BAD_PAGE, 10, kr);
          live[u] = false;
        } else {
          kb[u] = reinterpret_cast<const float4*>(a.kbar + kr * a.kbar_row_stride);
        }
      }
    }
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c4 = 0; c4 < a.d / 4; ++c4) {
      const float q0 = sq[4 * c4 + 0], q1 = sq[4 * c4 + 1], q2 = sq[4 * c4 + 2], q3 = sq[4 * c4 + 3];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!live[u]) continue;
        const float4 k4 = __ldg(kb[u] + c4);
        acc[u] = __fmaf_rn(q0, k4.x, acc[u]);
        acc[u] = __fmaf_rn(q1, k4.y, acc[u]);
        acc[u] = __fmaf_rn(q2, k4.z, acc[u]);
        acc[u] = __fmaf_rn(q3, k4.w, acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + u * step;
      if (b < W) sx[b] = live[u] ? clamp_act(__fmul_rn(acc[u], inv_sqrt_d)) : kScoreNeg;
    }
  }
}

// Largest T with #{key >= T} >= M, decided bit by bit from the top.  The scan
// stops once exactly M keys are >= T: the top-M set is then fixed and has no
// partial tie at its boundary.  Keys are order_key(x); padding keys are 0,
// below every real key.
template <int KW>
__device__ __forceinline__ uint32_t radix_threshold(const uint32_t (&kr)[KW], int M) {
  uint32_t T = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t trial = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int u = 0; u < KW; ++u) c += kr[u] >= trial ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= M) {
      T = trial;
      if (c == M) break;
    }
  }
  return T;
}

__device__ __forceinline__ uint32_t radix_threshold_smem(const float* sx, int W, int M, int lane) {
  uint32_t T = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t trial = T | (1u << bit);
    int c = 0;
    for (int b = lane; b < W; b += 32) c += order_key(sx[b]) >= trial ? 1 : 0;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= M) {
      T = trial;
      if (c == M) break;
    }
  }
  return T;
}

// Selection for one row whose W scores are in sx, by one warp: candidates,
// x = score*scale, top-M (x desc, id asc), 1.5-entmax over the top-M, first K
// by rank, bias, ascending pack.  KW > 0: W <= 32*KW and the x / keys of
// block lane + 32u live in registers; KW == 0: they stay in sx (overwritten).
//
// The entmax threshold is the sort-based formula of
// modeling_deepseekv2.py:_infer_route_select (via entmax15): for every rank k
// of the sorted z = (x - max)/2, tau_k = mean_k - sqrt(max((1 - ss_k)/k, 0))
// from prefix sums taken sequentially in rank order; support = #{k : tau_k <=
// z_k}; tau = tau_support.  Each step is one correctly rounded operation in
// the order of the CPU restatement, so tau is bitwise the restatement's.
//
// Per-warp scratch: mid_ (block id by slot; slots ascend by id), mx (x by
// slot, then z by rank, then log-prior by rank), mval (valid flag by rank).
// Page-aware candidacy of block b for a row of sequence s whose query page is
// qp (descriptor of a physical block through the block table, or row-major
// per sequence).
__device__ __forceinline__ bool page_block_holds(const DashRouteArgs& a, int qp, int s, int b) {
  if (qp < 0) return false;
  const int64_t i = a.block_table ? (int64_t)a.block_table[(int64_t)s * a.bt_stride + b]
                                  : (int64_t)s * a.page_seq_rows + b;
  if (i < 0 || i >= a.num_page_desc) {
    record_error(a.device_error, DASH_DEV_BAD_PAGE, 13, i);
    return false;
  }
  return page_desc_holds(a.page_lo, a.page_hi, a.page_bits, a.page_bits_words, i, qp);
}

// Second half of a row's selection, by one warp: the M top-M items are in
// slots (mid_ = block id, mx = x) in ascending id order; ranks by (x desc, id
// asc), the sort-based entmax threshold, the log prior of the first K ranks,
// bias and the ascending pack.  scand holds the row's candidate bits.
template <int PER>
__device__ __forceinline__ void select_tail(const DashRouteArgs& a, const uint32_t* scand, const int* mid_,
                                            float* mx, int* mval, int M, int64_t r, int lane) {
  const uint32_t lt_mask = (1u << lane) - 1u;
  auto is_cand = [&](int b) -> bool { return (scand[b >> 5] >> (b & 31)) & 1u; };
  // ---- rank of slot t = lane + 32u by (x desc, id asc); PER >= ceil(M / 32) ----
  const int nper = (M + 31) >> 5;
  float xt[PER];
  int rk[PER];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int t = lane + 32 * u;
    xt[u] = (u < nper && t < M) ? mx[t] : -INFINITY;
    rk[u] = 0;
  }
#pragma unroll 8
  for (int v = 0; v < M; ++v) {
    const float xv = mx[v];
#pragma unroll
    for (int u = 0; u < PER; ++u)
      if (u < nper) rk[u] += (xv > xt[u] || (xv == xt[u] && v < lane + 32 * u)) ? 1 : 0;
  }
  float xmax = -INFINITY;
#pragma unroll
  for (int u = 0; u < PER; ++u) xmax = fmaxf(xmax, xt[u]);
  for (int o = 16; o > 0; o >>= 1) xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
  int Kc = min(a.K, M);
  if (Kc < 1) Kc = 1;
  bool valid[PER];
  __syncwarp();  // every lane has read mx by slot
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int t = lane + 32 * u;
    valid[u] = false;
    if (u < nper && t < M) {
      valid[u] = rk[u] < Kc && is_cand(mid_[t]);
      mx[rk[u]] = __fmul_rn(__fsub_rn(xt[u], xmax), 0.5f);   // z by rank (x/2 exactly)
      mval[rk[u]] = valid[u] ? 1 : 0;
    }
  }
  __syncwarp();

  // ---- tau_k for rank k = lane + 32u; support; tau ----
  float cs = 0.0f, cs2 = 0.0f;
  float tau_r[PER];
  int support = 0;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    tau_r[u] = 0.0f;
    if (u < nper) {
      const int k = lane + 32 * u;
      // add z_j for j = previous k + 1 .. k in ascending order (u = 0: 0 .. k)
      const int jstart = u == 0 ? 32 - min(M, 32) : 0;
#pragma unroll 8
      for (int jj = jstart; jj < 32; ++jj) {
        const int j = k - 31 + jj;
        const float zj = mx[max(j, 0)];
        if (j >= 0) {
          cs = __fadd_rn(cs, zj);
          cs2 = __fadd_rn(cs2, __fmul_rn(zj, zj));
        }
      }
      bool in_support = false;
      if (k < M) {
        const float rho = (float)(k + 1);
        const float mean = __fdiv_rn(cs, rho);
        const float mean_sq = __fdiv_rn(cs2, rho);
        const float ss = __fmul_rn(rho, __fsub_rn(mean_sq, __fmul_rn(mean, mean)));
        const float delta = __fdiv_rn(__fsub_rn(1.0f, ss), rho);
        const float tau = __fsub_rn(mean, __fsqrt_rn(delta > 0.0f ? delta : 0.0f));
        tau_r[u] = tau;
        in_support = tau <= mx[k];
      }
      support += __popc(__ballot_sync(0xffffffffu, in_support));
    }
  }
  if (support < 1) support = 1;
  float tsel = 0.0f;
#pragma unroll
  for (int u = 0; u < PER; ++u)
    if (u == ((support - 1) >> 5)) tsel = tau_r[u];
  const float tau = __shfl_sync(0xffffffffu, tsel, (support - 1) & 31);

  // ---- log prior of the first Kc ranks; mean over the valid ones ----
  __syncwarp();  // every lane has read z by rank
  for (int k = lane; k < Kc; k += 32) {
    float t = __fsub_rn(mx[k], tau);
    t = t > 0.0f ? t : 0.0f;
    const float p = __fmul_rn(t, t);
    mx[k] = logf(p > a.prior_floor ? p : a.prior_floor);
  }
  __syncwarp();
  float lsum = 0.0f;
  int cnt = 0;
#pragma unroll 8
  for (int k = 0; k < Kc; ++k)
    if (mval[k]) {
      lsum = __fadd_rn(lsum, mx[k]);
      ++cnt;
    }
  const float mu = __fdiv_rn(lsum, (float)(cnt > 0 ? cnt : 1));

  // ---- ascending pack (slots ascend by id) ----
  int32_t* oi = a.out_idx + r * a.out_stride;
  float* ob = a.out_bias + r * a.out_stride;
  int npos = 0;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    if (u < nper) {
      const uint32_t vb = __ballot_sync(0xffffffffu, valid[u]);
      if (valid[u]) {
        const int p = npos + __popc(vb & lt_mask);
        if (p < a.out_width) {
          oi[p] = mid_[lane + 32 * u];
          ob[p] = __fmul_rn(__fsub_rn(mx[rk[u]], mu), a.inv_sigma);
        }
      }
      npos += __popc(vb);
    }
  }
  for (int j = npos + lane; j < a.out_width; j += 32) {
    oi[j] = -1;
    ob[j] = 0.0f;
  }
  if (a.out_count && lane == 0) a.out_count[r] = min(npos, a.out_width);
}

template <int KW, int PER>
__device__ __noinline__ void select_row(const DashRouteArgs& a, float* sx, uint32_t* scand,
                                        int* mid_, float* mx, int* mval, int64_t r, int s,
                                        int lane, uint32_t* pc_cache) {
  const int W = a.width;
  const int Wp = (W + 31) & ~31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  // ---- candidates (with per-row fallback) ----
  const uint8_t* cm = nullptr;
  if (a.cand && !a.page_q) cm = a.cand + (a.cand_per_seq ? (int64_t)s : r) * a.cand_row_stride;
  const int qp = a.page_q ? a.page_q[r] : -1;
  // KW > 0: page candidacy of block lane + 32u in bit u, computed with
  // independent loads and, with a cache (rows of one sequence handled by this
  // warp), reused while the query page stays the same
  uint32_t pcm = 0;
  if constexpr (KW > 0) {
    if (a.page_q) {
      if (pc_cache && (int)pc_cache[32] == qp) {
        pcm = pc_cache[lane];
      } else {
#pragma unroll
        for (int u = 0; u < KW; ++u) {
          const int b = lane + 32 * u;
          if (b < W && page_block_holds(a, qp, s, b)) pcm |= 1u << u;
        }
        if (pc_cache) {
          __syncwarp();
          pc_cache[lane] = pcm;
          if (lane == 0) pc_cache[32] = (uint32_t)qp;
          __syncwarp();
        }
      }
    }
  }
  // KW > 0: the row's scores of blocks lane + 32u come into registers once;
  // candidate bit u of this lane in cbits
  float sv[KW > 0 ? KW : 1];
  uint32_t cbits = 0u;
  if constexpr (KW > 0) {
    uint32_t rbits = 0u;
#pragma unroll
    for (int u = 0; u < KW; ++u) {
      const int b = lane + 32 * u;
      sv[u] = b < W ? sx[b] : kScoreNeg;
      const bool remote = b < W && sv[u] > kScoreNeg * 0.5f;
      bool c = remote;
      if (a.page_q) c = remote && ((pcm >> u) & 1u) != 0;
      else if (cm) c = remote && cm[b] != 0;
      rbits |= (remote ? 1u : 0u) << u;
      cbits |= (c ? 1u : 0u) << u;
    }
    if (!__any_sync(0xffffffffu, cbits != 0u)) cbits = rbits;   // fallback: every remote block
#pragma unroll
    for (int u = 0; u < KW; ++u) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (cbits >> u) & 1u);
      if (lane == 0 && 32 * u < Wp) scand[u] = bal;
    }
    __syncwarp();
  } else {
    bool any = false;
    for (int b0 = 0; b0 < Wp; b0 += 32) {
      int b = b0 + lane;
      bool remote = b < W && sx[b] > kScoreNeg * 0.5f;
      bool c = remote;
      if (a.page_q) c = remote && page_block_holds(a, qp, s, b);
      else if (cm) c = remote && cm[b] != 0;
      uint32_t bal = __ballot_sync(0xffffffffu, c);
      if (lane == 0) scand[b0 >> 5] = bal;
      any |= bal != 0;
    }
    __syncwarp();
    if (!any) {
      for (int b0 = 0; b0 < Wp; b0 += 32) {
        int b = b0 + lane;
        bool remote = b < W && sx[b] > kScoreNeg * 0.5f;
        uint32_t bal = __ballot_sync(0xffffffffu, remote);
        if (lane == 0) scand[b0 >> 5] = bal;
      }
      __syncwarp();
    }
  }
  auto is_cand = [&](int b) -> bool { return (scand[b >> 5] >> (b & 31)) & 1u; };
  auto xform = [&](int b) -> float {
    float v = is_cand(b) ? __fmul_rn(sx[b], a.idx_scale) : kEntmaxNeg;
    if (!(v == v) || isinf(v)) v = kEntmaxNeg;
    return v;
  };

  // ---- top-M, gathered into slots in ascending id order ----
  int M = a.topm > 0 ? min(a.topm, W) : W;
  if (M < 1) M = 1;
  int n_items = 0;
  auto gather = [&](int b, float x, uint32_t k, uint32_t T, int& ties_left) {
    bool in = false, tie = false;
    if (b < W) {
      if (M >= W || k > T) in = true;
      else if (k == T) tie = true;
    }
    const uint32_t tb = __ballot_sync(0xffffffffu, tie);
    if (tie && __popc(tb & lt_mask) < ties_left) in = true;
    ties_left -= min(ties_left, __popc(tb));
    const uint32_t ib = __ballot_sync(0xffffffffu, in);
    if (in) {
      const int slot = n_items + __popc(ib & lt_mask);
      mid_[slot] = b;
      mx[slot] = x;
    }
    n_items += __popc(ib);
  };
  if constexpr (KW > 0) {
    float xr[KW];
    uint32_t kr[KW];
#pragma unroll
    for (int u = 0; u < KW; ++u) {
      const int b = lane + 32 * u;
      float v = ((cbits >> u) & 1u) ? __fmul_rn(sv[u], a.idx_scale) : kEntmaxNeg;
      if (!(v == v) || isinf(v)) v = kEntmaxNeg;
      xr[u] = b < W ? v : 0.0f;
      kr[u] = b < W ? order_key(xr[u]) : 0u;
    }
    uint32_t T = 0;
    int n_gt = 0;
    if (M < W) {
      // Every non-candidate has x = kEntmaxNeg.  When the candidates fit the
      // window and all lie above that value, the top-M is the candidates plus
      // the lowest-id non-candidates: the threshold is that value's key (no
      // select; rows restricted to a few blocks would otherwise resolve the
      // long tie digit by digit).
      int nc = 0;
      bool low = false;
#pragma unroll
      for (int u = 0; u < KW; ++u) {
        const int b = lane + 32 * u;
        if (b < W && ((cbits >> u) & 1u)) {
          ++nc;
          low |= !(xr[u] > kEntmaxNeg);
        }
      }
      nc = __reduce_add_sync(0xffffffffu, nc);
      if (nc <= M && !__any_sync(0xffffffffu, low)) {
        T = order_key(kEntmaxNeg);
        n_gt = nc;
      } else {
        T = radix_threshold<KW>(kr, M);
        int c = 0;
#pragma unroll
        for (int u = 0; u < KW; ++u) c += kr[u] > T ? 1 : 0;
        n_gt = __reduce_add_sync(0xffffffffu, c);
      }
    }
    int ties_left = M - n_gt;
#pragma unroll
    for (int u = 0; u < KW; ++u)
      if (32 * u < W) gather(lane + 32 * u, xr[u], kr[u], T, ties_left);
  } else {
    for (int b = lane; b < W; b += 32) sx[b] = xform(b);
    __syncwarp();
    uint32_t T = 0;
    int n_gt = 0;
    if (M < W) {
      T = radix_threshold_smem(sx, W, M, lane);
      int c = 0;
      for (int b = lane; b < W; b += 32) c += order_key(sx[b]) > T ? 1 : 0;
      n_gt = __reduce_add_sync(0xffffffffu, c);
    }
    int ties_left = M - n_gt;
    for (int b0 = 0; b0 < Wp; b0 += 32) {
      const int b = b0 + lane;
      const float x = b < W ? sx[b] : 0.0f;
      gather(b, x, b < W ? order_key(x) : 0u, T, ties_left);
    }
  }
  __syncwarp();
  M = n_items;  // == M

  select_tail<PER>(a, scand, mid_, mx, mval, M, r, lane);
}

template <int KW>
__device__ __forceinline__ void select_row_m(const DashRouteArgs& a, float* sx, uint32_t* scand,
                                             int* mid_, float* mx, int* mval, int64_t r, int s,
                                             int lane, uint32_t* pc_cache) {
  const int W = a.width;
  const int M = a.topm > 0 ? min(a.topm, W) : W;
  if (M <= 32) select_row<KW, 1>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else if (M <= 64) select_row<KW, 2>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else select_row<KW, kMaxM / 32>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
}

__device__ __forceinline__ void select_row_any(const DashRouteArgs& a, float* sx,
                                               uint32_t* scand, int* mid_, float* mx, int* mval,
                                               int64_t r, int s, int lane,
                                               uint32_t* pc_cache = nullptr) {
  const int W = a.width;
  if (W <= 160) select_row_m<5>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else if (W <= 256) select_row_m<8>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else if (W <= 512) select_row_m<16>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else if (W <= 1024) select_row_m<32>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
  else select_row_m<0>(a, sx, scand, mid_, mx, mval, r, s, lane, pc_cache);
}

// ---------------------------------------------------------------------------
// Tiled routing for many rows: a CTA scores 32 consecutive query rows of one
// sequence against 64-block chunks of k-bar staged in shared memory (each
// k-bar row is read from L2 once per 32 rows), then each warp selects for 4
// rows.  Every score is still one thread's sequential FMA chain.
// ---------------------------------------------------------------------------
constexpr int kTileRows = 32;
constexpr int kPcCache = 33;   // per warp: page-candidacy mask per lane + the query page
constexpr int kChunk = 64;
constexpr int kLd = 132;   // padded fp32 query row (conflict-free 16-byte loads by row)
constexpr int kKLd = 128;  // k-bar chunk row (read by broadcast: no padding)

// Per-warp selection scratch of a row: candidate bits [Wp / 32] and the
// top-M items (id, x, rank flag) [3 * Mp], Mp = M rounded up to 32.
__host__ __device__ inline int route_sel_floats(int W, int M) {
  return (W + 31) / 32 + 3 * ((M + 31) & ~31);
}
__host__ __device__ inline size_t route_tile_smem_floats(int W, int M) {
  const int Wp = (W + 31) & ~31;
  return (size_t)kTileRows * kLd + (size_t)kChunk * kKLd + kChunk + (size_t)kTileRows * Wp +
         8 * (size_t)route_sel_floats(W, M) + 8 * kPcCache;
}

__global__ void __launch_bounds__(256, 3) route_tile_kernel(const __grid_constant__ DashRouteArgs a, int tiles_per_seq) {
  extern __shared__ float smt[];
  const int W = a.width, Wp = (W + 31) & ~31;
  float* qs = smt;                                  // [32][kLd]
  float* kbs = qs + kTileRows * kLd;                // [64][kKLd]
  int* kbad = reinterpret_cast<int*>(kbs + kChunk * kKLd);  // [64]
  float* scs = reinterpret_cast<float*>(kbad + kChunk);     // [32][Wp]
  float* selbase = scs + kTileRows * Wp;            // per warp: cand | ids | x | ranks
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = blockIdx.x / tiles_per_seq, tb = blockIdx.x - s * tiles_per_seq;
  const int qlen = seq_q_len(a.seqs, s);
  const int i0 = tb * kTileRows;
  if (i0 >= qlen) return;
  const int nr = min(kTileRows, qlen - i0);
  const int kvl = seq_kv_len(a.seqs, s);
  const int64_t rbase = (a.seqs.q_start ? (int64_t)a.seqs.q_start[s] : (int64_t)s * a.seqs.q_len_fixed) + i0;
  const int64_t p0 = seq_pos(a.seqs, s, i0);
  const int bs = a.block_size;
  for (int e = tid; e < kTileRows * 32; e += 256) {
    const int rr = e >> 5, c4 = e & 31;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rr < nr) v = *reinterpret_cast<const float4*>(a.idx_q + (rbase + rr) * a.q_row_stride + 4 * c4);
    *reinterpret_cast<float4*>(qs + rr * kLd + 4 * c4) = v;
  }
  for (int e = tid; e < kTileRows * Wp; e += 256) scs[e] = kScoreNeg;
  int64_t bmax = (p0 + nr - 1) / bs - a.local_blocks;   // last block any row of the tile scores
  bmax = min(bmax, (int64_t)W - 1);
  bmax = min(bmax, (int64_t)(kvl - 1) / bs);
  const int rr = tid & 31;
  const int64_t qblk_r = (p0 + rr) / bs;
  const float inv_sqrt_d = (float)(1.0 / sqrt((double)a.d));
  __syncthreads();
  for (int64_t cb0 = 0; cb0 <= bmax; cb0 += kChunk) {
    for (int e = tid; e < kChunk * 32; e += 256) {
      const int bb = e >> 5, c4 = e & 31;
      const int64_t b = cb0 + bb;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      int bad = 1;
      if (b <= bmax) {
        const int64_t kr = a.block_table ? (int64_t)a.block_table[(int64_t)s * a.bt_stride + b]
                                         : (int64_t)s * a.kbar_seq_rows + b;
        if (kr < 0 || kr >= a.num_kbar_rows) {
          if (c4 == 0) record_error(a.device_error, DASH_DEV_BAD_PAGE, 11, kr);
        } else {
          v = __ldg(reinterpret_cast<const float4*>(a.kbar + kr * a.kbar_row_stride) + c4);
          bad = 0;
        }
      }
      *reinterpret_cast<float4*>(kbs + bb * kKLd + 4 * c4) = v;
      if (c4 == 0) kbad[bb] = bad;
    }
    __syncthreads();
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
    // blocks warp + 8k of the chunk that exist (warp-uniform): a chunk past
    // the tile's last block skips the rest
    const int64_t dlast = bmax - cb0 - warp;
    const int nk = dlast < 0 ? 0 : (int)min((int64_t)8, dlast / 8 + 1);
    if (nk == 8) {
      for (int c4 = 0; c4 < 32; ++c4) {
        const float4 q4 = *reinterpret_cast<const float4*>(qs + rr * kLd + 4 * c4);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 k4 = *reinterpret_cast<const float4*>(kbs + (warp + 8 * k) * kKLd + 4 * c4);
          acc[k] = __fmaf_rn(q4.x, k4.x, acc[k]);
          acc[k] = __fmaf_rn(q4.y, k4.y, acc[k]);
          acc[k] = __fmaf_rn(q4.z, k4.z, acc[k]);
          acc[k] = __fmaf_rn(q4.w, k4.w, acc[k]);
        }
      }
    } else if (nk > 0) {
      for (int c4 = 0; c4 < 32; ++c4) {
        const float4 q4 = *reinterpret_cast<const float4*>(qs + rr * kLd + 4 * c4);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k < nk) {
            const float4 k4 = *reinterpret_cast<const float4*>(kbs + (warp + 8 * k) * kKLd + 4 * c4);
            acc[k] = __fmaf_rn(q4.x, k4.x, acc[k]);
            acc[k] = __fmaf_rn(q4.y, k4.y, acc[k]);
            acc[k] = __fmaf_rn(q4.z, k4.z, acc[k]);
            acc[k] = __fmaf_rn(q4.w, k4.w, acc[k]);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int bb = warp + 8 * k;
      const int64_t b = cb0 + bb;
      if (rr < nr && b <= bmax && !kbad[bb] && b <= qblk_r - a.local_blocks && b * bs < kvl)
        scs[rr * Wp + b] = clamp_act(__fmul_rn(acc[k], inv_sqrt_d));
    }
    __syncthreads();
  }
  // selection scratch sized by the entmax window M (every index it takes is < M)
  const int Msel = a.topm > 0 ? min(a.topm, W) : W;
  const int Mp = (max(Msel, 1) + 31) & ~31;
  const int sel_floats = route_sel_floats(W, Msel);
  float* sel = selbase + warp * sel_floats;
  uint32_t* pc_cache = reinterpret_cast<uint32_t*>(selbase + 8 * sel_floats) + warp * kPcCache;
  if (lane == 0) pc_cache[32] = 0x80000000u;   // no page cached (pages are >= -1)
  __syncwarp();
  uint32_t* scand = reinterpret_cast<uint32_t*>(sel);
  int* mid_ = reinterpret_cast<int*>(scand + Wp / 32);
  float* mx = reinterpret_cast<float*>(mid_ + Mp);
  int* mrank = reinterpret_cast<int*>(mx + Mp);
  for (int r2 = warp; r2 < nr; r2 += 8) {
    const int64_t r = rbase + r2;
    float* sx = scs + r2 * Wp;
    if (a.scores_out)
      for (int b = lane; b < W; b += 32) a.scores_out[r * a.scores_out_stride + b] = sx[b];
    __syncwarp();
    select_row_any(a, sx, scand, mid_, mx, mrank, r, s, lane, pc_cache);
    __syncwarp();
  }
}

// CTA_ROW = false: one warp per row (many rows).  CTA_ROW = true: one CTA per
// row, all its threads score the row's blocks, warp 0 selects (few rows,
// e.g. decode).
template <bool CTA_ROW>
__global__ void __launch_bounds__(kRouteWarps * 32) route_rows_kernel(const __grid_constant__ DashRouteArgs a,
                                                                     int64_t n_rows) {
  extern __shared__ float smr[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = a.width;
  const int Wp = (W + 31) & ~31;
  // per-warp scratch: q [d] | x [Wp] | cand bits [Wp/32] | M items (id, x) | sel flags
  const int slot = CTA_ROW ? 0 : warp;
  float* sq = smr + slot * (a.d + Wp + Wp / 32 + 3 * kMaxM);
  float* sx = sq + a.d;
  uint32_t* scand = reinterpret_cast<uint32_t*>(sx + Wp);
  int* mid_ = reinterpret_cast<int*>(scand + Wp / 32);
  float* mx = reinterpret_cast<float*>(mid_ + kMaxM);
  int* mrank = reinterpret_cast<int*>(mx + kMaxM);

  const int64_t r = CTA_ROW ? (int64_t)blockIdx.x : (int64_t)blockIdx.x * kRouteWarps + warp;
  if (r >= n_rows) return;
  int s, i;
  row_to_seq(a.seqs, r, s, i);
  const int64_t pos = seq_pos(a.seqs, s, i);
  const int kvl = seq_kv_len(a.seqs, s);
  const int64_t qblk = pos >= 0 ? pos / a.block_size : -1;

  // ---- scores ----
  if (a.scores_in) {
    if (CTA_ROW && warp != 0) return;
    for (int b = lane; b < W; b += 32) sx[b] = a.scores_in[r * a.scores_in_stride + b];
  } else if (CTA_ROW) {
    for (int c = threadIdx.x; c < a.d; c += blockDim.x) sq[c] = a.idx_q[r * a.q_row_stride + c];
    __syncthreads();
    score_blocks(a, sq, sx, s, qblk, kvl, threadIdx.x, blockDim.x);
    __syncthreads();
    if (warp != 0) return;
  } else {
    for (int c = lane; c < a.d; c += 32) sq[c] = a.idx_q[r * a.q_row_stride + c];
    __syncwarp();
    score_blocks(a, sq, sx, s, qblk, kvl, lane, 32);
  }
  __syncwarp();
  if (a.scores_out)
    for (int b = lane; b < W; b += 32) a.scores_out[r * a.scores_out_stride + b] = sx[b];

  select_row_any(a, sx, scand, mid_, mx, mrank, r, s, lane);
}

// ---------------------------------------------------------------------------
// Few rows (decode): a cluster of kClusterCtas CTAs per row.  CTA c scores a
// contiguous slice of the row's blocks, one thread per block (its k-bar row is
// loaded whole, then the same sequential FMA chain as score_blocks, so scores
// are bitwise those of the other kernels).  After a cluster barrier CTA 0
// pulls the row's W scores out of the slices (distributed shared memory)
// straight into registers, EPT consecutive blocks per thread, and selects
// with all its threads (select_head_cta); warp 0 finishes (select_tail).
// The other CTAs are free after the barrier: with RK > 0 they refresh the
// k-bar rows of a paged plan meanwhile (the tail refresh of a decode step,
// folded into the routing launch).  A second, split barrier keeps every slice
// alive until CTA 0 has read it.  Rows wider than 128 * kClusterEpt blocks
// select with the one-warp select_row.
// ---------------------------------------------------------------------------
constexpr int kClusterCtas = 8;
constexpr int kClusterEpt = 8;        // CTA-wide selection up to 1024 blocks

__host__ __device__ inline int cluster_slice(int W) { return (W + kClusterCtas - 1) / kClusterCtas; }
// Shared memory, floats: q [128] | this CTA's slice | CTA 0's selection
// scratch, or a helper CTA's k-bar refresh scratch (the larger of the two).
__host__ __device__ inline size_t route_cluster_smem_floats(int W, size_t refresh_floats) {
  const int Wp = (W + 31) & ~31;
  const int per = (cluster_slice(W) + 31) & ~31;
  const size_t sel = (size_t)Wp + Wp / 32 + 3 * kMaxM + 256 + 16;
  return (size_t)128 + per + (sel > refresh_floats ? sel : refresh_floats);
}

// Blocks per thread of the CTA-wide selection: a power of two (a thread's
// candidate bits then lie in one 32-bit word), 0 when W is too wide.
__host__ __device__ inline int cluster_ept(int W) {
  const int need = (W + 127) / 128;
  return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : need <= kClusterEpt ? 8 : 0;
}

// CTA-wide first half of a row's selection (all 128 threads; the row's scores
// sc[e] of blocks b = EPT * tid + e, W <= 128 * EPT): candidates with the
// per-row fallback, x = z * scale, the exact M-th largest order key by an
// 8-bit radix over a shared histogram (stopping once a digit's keys are all
// taken), then the top-M by (x desc, id asc) gathered into slots in ascending
// id order through one packed (in, tie) prefix scan.  It takes the same set as
// select_row's warp form: keys above the threshold, and ties at it from the
// lowest id up.  Returns M.
template <int EPT>
__device__ int select_head_cta(const DashRouteArgs& a, const float (&sc)[EPT], int W, int64_t r, int s,
                               uint32_t* scand, int* mid_, float* mx, uint32_t* hist, uint32_t* sred) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b0 = tid * EPT;
  const int Wp = (W + 31) & ~31;
  // ---- candidates (with the per-row fallback to every remote block) ----
  const uint8_t* cm = nullptr;
  if (a.cand && !a.page_q) cm = a.cand + (a.cand_per_seq ? (int64_t)s : r) * a.cand_row_stride;
  const int qp = a.page_q ? a.page_q[r] : -1;
  uint32_t rem_bits = 0u, cand_bits = 0u;
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    const int b = b0 + e;
    const bool remote = b < W && sc[e] > kScoreNeg * 0.5f;
    bool c = remote;
    if (remote) {
      if (a.page_q) c = page_block_holds(a, qp, s, b);
      else if (cm) c = cm[b] != 0;
    }
    rem_bits |= (remote ? 1u : 0u) << e;
    cand_bits |= (c ? 1u : 0u) << e;
  }
  for (int w = tid; w < Wp / 32; w += blockDim.x) scand[w] = 0u;
  if (__syncthreads_or(cand_bits != 0u) == 0) cand_bits = rem_bits;
  if (cand_bits) atomicOr(scand + (b0 >> 5), cand_bits << (b0 & 31));

  // ---- x and order keys ----
  float x[EPT];
  uint32_t key[EPT];
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    float v = ((cand_bits >> e) & 1u) ? __fmul_rn(sc[e], a.idx_scale) : kEntmaxNeg;
    if (!(v == v) || isinf(v)) v = kEntmaxNeg;
    x[e] = v;
    key[e] = order_key(v);
  }
  int M = a.topm > 0 ? min(a.topm, W) : W;
  if (M < 1) M = 1;
  const bool all = M >= W;

  // ---- threshold T: keys > T are in, keys == T are ties ----
  uint32_t T = 0u;
  if (!all) {
    // bits every key shares are decided at once (scores of a row sit in a
    // narrow range, so their top bits agree): only the `lo` low bits below
    // the highest differing bit are resolved digit by digit
    uint32_t kand = 0xffffffffu, kor = 0u;
#pragma unroll
    for (int e = 0; e < EPT; ++e)
      if (b0 + e < W) {
        kand &= key[e];
        kor |= key[e];
      }
    kand = __reduce_and_sync(0xffffffffu, kand);
    kor = __reduce_or_sync(0xffffffffu, kor);
    if (lane == 0) {
      sred[8 + warp] = kand;
      sred[12 + warp] = kor;
    }
    __syncthreads();
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      kand &= sred[8 + w];
      kor |= sred[12 + w];
    }
    const uint32_t diff = kand ^ kor;
    int lo = diff ? 32 - __clz(diff) : 0;
    uint32_t prefix = lo >= 32 ? 0u : (kand & (0xffffffffu << lo));
    int need = M;                       // keys still to take among those matching prefix
    while (lo > 0) {
      const int shift = lo > 8 ? lo - 8 : 0;
      const uint32_t hmask = lo >= 32 ? 0u : (0xffffffffu << lo);
      const uint32_t dmask = (1u << (lo - shift)) - 1u;
      for (int j = tid; j < 256; j += blockDim.x) hist[j] = 0u;
      __syncthreads();
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
        const bool in = b0 + e < W && (key[e] & hmask) == prefix;
        const uint32_t dg = in ? (key[e] >> shift) & dmask : 0xffffffffu;
        // one increment per distinct digit of the warp
        const uint32_t same = __match_any_sync(0xffffffffu, dg);
        if (in && (same & ((1u << lane) - 1u)) == 0u) atomicAdd(hist + dg, (uint32_t)__popc(same));
      }
      __syncthreads();
      if (warp == 0) {
        // lane l holds digits 8l .. 8l+7; suf = keys with digit >= 8l
        uint32_t h[8], tot = 0u;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          h[k] = hist[lane * 8 + k];
          tot += h[k];
        }
        uint32_t suf = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += v;
        }
        const uint32_t above = suf - tot;          // keys with digit >= 8(l+1)
        // exactly one lane has above < need <= suf (suf of lane 0 = all >= need)
        if (above < (uint32_t)need && (uint32_t)need <= suf) {
          uint32_t acc = above, hsel = 0u;
          int dsel = lane * 8;
#pragma unroll
          for (int k = 7; k >= 0; --k) {
            if (hsel == 0u && acc + h[k] >= (uint32_t)need) {
              dsel = lane * 8 + k;
              hsel = h[k];
            } else if (hsel == 0u) {
              acc += h[k];
            }
          }
          const uint32_t left = (uint32_t)need - acc;   // 1 .. hsel
          sred[0] = prefix | ((uint32_t)dsel << shift);
          sred[1] = left;
          sred[2] = hsel == left ? 1u : 0u;             // every key of the digit is in
        }
      }
      __syncthreads();
      prefix = sred[0];
      need = (int)sred[1];
      lo = shift;
      if (sred[2]) break;
    }
    T = prefix;
  }

  // ---- gather: slot = #in with a lower id + #ties taken with a lower id ----
  uint32_t in_bits = 0u, tie_bits = 0u;
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    if (b0 + e < W) {
      if (all || key[e] > T) in_bits |= 1u << e;
      else if (key[e] == T) tie_bits |= 1u << e;
    }
  }
  const uint32_t v = ((uint32_t)__popc(in_bits) << 16) | (uint32_t)__popc(tie_bits);
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) sred[4 + warp] = inc;
  __syncthreads();
  uint32_t before = inc - v, total = 0u;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    const uint32_t t = sred[4 + w];
    if (w < warp) before += t;
    total += t;
  }
  const int ties_left = M - (int)(total >> 16);
  int in_b = (int)(before >> 16), tie_b = (int)(before & 0xffffu);
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    int slot = -1;
    if ((in_bits >> e) & 1u) {
      slot = in_b + min(tie_b, ties_left);
      ++in_b;
    } else if ((tie_bits >> e) & 1u) {
      if (tie_b < ties_left) slot = in_b + tie_b;
      ++tie_b;
    }
    if (slot >= 0) {
      mid_[slot] = b0 + e;
      mx[slot] = x[e];
    }
  }
  __syncthreads();
  return M;
}

template <int PER>
__device__ __noinline__ void select_tail_warp(const DashRouteArgs& a, const uint32_t* scand, const int* mid_,
                                              float* mx, int* mval, int M, int64_t r, int lane) {
  select_tail<PER>(a, scand, mid_, mx, mval, M, r, lane);
}

// Scores of blocks [rank * per, rank * per + per) of the row into ssc.
__device__ __forceinline__ void cluster_score_slice(const DashRouteArgs& a, const float* sq, float* ssc,
                                                    int rank, int per, int s, int64_t qblk, int kvl) {
  const float inv_sqrt_d = (float)(1.0 / sqrt((double)a.d));
  const float4* sq4 = reinterpret_cast<const float4*>(sq);
  for (int t = threadIdx.x; t < per; t += blockDim.x) {
    const int b = rank * per + t;
    float sc = kScoreNeg;
    bool live = b < a.width && (int64_t)b <= qblk - a.local_blocks && (int64_t)b * a.block_size < kvl;
    int64_t kr = 0;
    if (live) {
      kr = a.block_table ? (int64_t)a.block_table[(int64_t)s * a.bt_stride + b]
                         : (int64_t)s * a.kbar_seq_rows + b;
      if (kr < 0 || kr >= a.num_kbar_rows) {
        record_error(a.device_error, DASH_DEV_BAD_PAGE, 12, kr);
        live = false;
      }
    }
    if (live) {
      const float4* kb = reinterpret_cast<const float4*>(a.kbar + kr * a.kbar_row_stride);
      float4 kv[32];
#pragma unroll
      for (int c4 = 0; c4 < 32; ++c4) kv[c4] = __ldg(kb + c4);
      float acc = 0.0f;
#pragma unroll
      for (int c4 = 0; c4 < 32; ++c4) {
        const float4 q4 = sq4[c4];
        acc = __fmaf_rn(q4.x, kv[c4].x, acc);
        acc = __fmaf_rn(q4.y, kv[c4].y, acc);
        acc = __fmaf_rn(q4.z, kv[c4].z, acc);
        acc = __fmaf_rn(q4.w, kv[c4].w, acc);
      }
      sc = clamp_act(__fmul_rn(acc, inv_sqrt_d));
    }
    ssc[t] = sc;
  }
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// RK: 0 no refresh; 1 / 2 refresh with fp32 / bf16 index keys (d = 128,
// 16-byte staging).  ka.n_plan entries spread over the helper CTAs (rank >= 1)
// of every cluster.
template <int RK>
__global__ void __launch_bounds__(128) route_cluster_kernel(const __grid_constant__ DashRouteArgs a,
                                                            const __grid_constant__ DashKbarArgs ka) {
  extern __shared__ __align__(16) float smc[];
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = a.width;
  const int Wp = (W + 31) & ~31;
  const int per = cluster_slice(W);
  const int perp = (per + 31) & ~31;
  float* sq = smc;                                   // [128] router query
  float* ssc = sq + 128;                             // [per] this CTA's slice of scores
  float* rest = ssc + perp;                          // CTA 0: selection; helpers: refresh

  const int64_t r = (int64_t)(blockIdx.x / kClusterCtas);
  int s, i;
  row_to_seq(a.seqs, r, s, i);
  const int64_t pos = seq_pos(a.seqs, s, i);
  const int kvl = seq_kv_len(a.seqs, s);
  const int64_t qblk = pos >= 0 ? pos / a.block_size : -1;
  sq[threadIdx.x] = a.idx_q[r * a.q_row_stride + threadIdx.x];
  __syncthreads();
  cluster_score_slice(a, sq, ssc, rank, per, s, qblk, kvl);
  cl.sync();                                  // every slice written

  if (rank != 0) {
    cluster_arrive_release();                 // nothing more for CTA 0 to wait on
    if constexpr (RK > 0) {
      using KT = typename std::conditional<RK == 1, float, __nv_bfloat16>::type;
      const int helpers = (int)(gridDim.x / kClusterCtas) * (kClusterCtas - 1);
      for (int e = (int)(blockIdx.x / kClusterCtas) * (kClusterCtas - 1) + rank - 1; e < ka.n_plan;
           e += helpers) {
        int n;
        int64_t base, out_row;
        if (kbar_paged_entry(ka, e, n, base, out_row)) kbar_pool_body<KT, 128, true>(ka, rest, n, base, out_row);
      }
    }
    cluster_wait_acquire();                   // CTA 0 has read this slice
    return;
  }

  // ---- CTA 0: the row's scores, then its selection ----
  uint32_t* scand = reinterpret_cast<uint32_t*>(rest);         // [Wp / 32]
  int* mid_ = reinterpret_cast<int*>(scand + Wp / 32);         // [kMaxM]
  float* mx = reinterpret_cast<float*>(mid_ + kMaxM);          // [kMaxM]
  int* mval = reinterpret_cast<int*>(mx + kMaxM);              // [kMaxM]
  uint32_t* hist = reinterpret_cast<uint32_t*>(mval + kMaxM);  // [256]
  uint32_t* sred = hist + 256;                                 // [16]
  float* sx = reinterpret_cast<float*>(sred + 16);             // [Wp] (rows wider than the CTA form)
  auto pull = [&](int b) -> float {
    const int src = b / per;
    return cl.map_shared_rank(ssc, src)[b - src * per];
  };
  int M = 0;
  auto cta_select = [&](auto ept_c) {
    constexpr int E = decltype(ept_c)::value;
    float sc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int b = (int)threadIdx.x * E + e;
      sc[e] = b < W ? pull(b) : kScoreNeg;
    }
    cluster_arrive_release();                 // every slice has been read
    if (a.scores_out) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int b = (int)threadIdx.x * E + e;
        if (b < W) a.scores_out[r * a.scores_out_stride + b] = sc[e];
      }
    }
    M = select_head_cta<E>(a, sc, W, r, s, scand, mid_, mx, hist, sred);
  };
  const int ept = cluster_ept(W);
  if (ept == 1) cta_select(std::integral_constant<int, 1>{});
  else if (ept == 2) cta_select(std::integral_constant<int, 2>{});
  else if (ept == 4) cta_select(std::integral_constant<int, 4>{});
  else if (ept == 8) cta_select(std::integral_constant<int, 8>{});
  if (ept > 0) {
    if (warp == 0) {
      if (M <= 32) select_tail_warp<1>(a, scand, mid_, mx, mval, M, r, lane);
      else if (M <= 64) select_tail_warp<2>(a, scand, mid_, mx, mval, M, r, lane);
      else select_tail_warp<kMaxM / 32>(a, scand, mid_, mx, mval, M, r, lane);
    }
  } else {
    for (int b = threadIdx.x; b < W; b += blockDim.x) sx[b] = pull(b);
    cluster_arrive_release();
    __syncthreads();
    if (warp == 0) {
      if (a.scores_out)
        for (int b = lane; b < W; b += 32) a.scores_out[r * a.scores_out_stride + b] = sx[b];
      __syncwarp();
      select_row_any(a, sx, scand, mid_, mx, mval, r, s, lane);
    }
  }
  cluster_wait_acquire();
}

// ---------------------------------------------------------------------------
// Indexer stage-0: block max of token scores over remote keys.
// One CTA per (32 query rows, key block, batch); thread (row, key lane).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) block_max_kernel(DashBlockMaxArgs a) {
  extern __shared__ float smb[];
  const int d = a.d, ld = d + 1;
  float* sq = smb;                 // [32][d+1]
  float* sk = sq + 32 * ld;        // [bs][d+1]
  float* sred = sk + a.block_size * ld;  // [4][32]
  const int c0 = blockIdx.x * 32, blk = blockIdx.y, b = blockIdx.z;
  const int j0 = blk * a.block_size;
  for (int e = threadIdx.x; e < 32 * d; e += blockDim.x) {
    int rr = e / d, c = e - rr * d;
    int cc = c0 + rr;
    sq[rr * ld + c] = cc < a.C ? a.q[b * a.q_stride_b + (int64_t)cc * a.q_stride_c + c] : 0.0f;
  }
  for (int e = threadIdx.x; e < a.block_size * d; e += blockDim.x) {
    int jj = e / d, c = e - jj * d;
    int j = j0 + jj;
    sk[jj * ld + c] = j < a.Sk ? a.k[b * a.k_stride_b + (int64_t)j * a.k_stride_j + c] : 0.0f;
  }
  __syncthreads();
  const int rr = threadIdx.x & 31, part = threadIdx.x >> 5;
  const int cc = c0 + rr;
  float m = a.empty;
  bool any = false;
  if (cc < a.C) {
    int64_t pos = a.pos[b * a.pos_stride_b + (int64_t)cc * a.pos_stride_c];
    int64_t seg = a.seg ? a.seg[b * a.seg_stride_b + (int64_t)cc * a.seg_stride_c] : 0;
    int64_t hi = pos - a.local_window;
    for (int jj = part; jj < a.block_size; jj += 4) {
      int64_t j = j0 + jj;
      if (j >= a.Sk || j > hi || j < seg) continue;
      float acc = 0.0f;
      for (int c = 0; c < d; ++c) acc = __fmaf_rn(sq[rr * ld + c], sk[jj * ld + c], acc);
      if (a.clamp) acc = clamp_act(acc);
      if (!any || acc > m || acc != acc) { m = acc; any = true; }
    }
  }
  sred[part * 32 + rr] = m;
  int* sany = reinterpret_cast<int*>(sred + 128);
  sany[part * 32 + rr] = any ? 1 : 0;
  __syncthreads();
  if (part == 0 && cc < a.C) {
    float best = a.empty;
    bool got = false;
    for (int p = 0; p < 4; ++p) {
      if (!sany[p * 32 + rr]) continue;
      float v = sred[p * 32 + rr];
      if (!got || v > best || v != v) { best = v; got = true; }
    }
    a.out[b * a.out_stride_b + (int64_t)cc * a.out_stride_c + blk] = best;
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
// The decode form: a cluster of CTAs per row (few rows, scored here).
static bool route_takes_cluster(const DashRouteArgs& a, int64_t n_rows) {
  return !a.scores_in && a.d == 128 && n_rows < 148 * 16;
}

// 16-byte staging of a k-bar pool needs every row start 16-byte aligned.
static bool kbar_vec_ok(const DashKbarArgs& a) {
  const int w = a.dtype == DASH_DTYPE_F32 ? 4 : 8;
  return (reinterpret_cast<uintptr_t>(a.keys) & 15) == 0 && a.d % w == 0 && a.tok_stride % w == 0 &&
         (a.pages == nullptr ? a.seq_stride % w == 0 : a.page_stride % w == 0);
}

// ka: optional paged k-bar plan refreshed by the helper CTAs (d = 128, 16-byte
// staging; the caller checked).
static int launch_route_cluster(const DashRouteArgs& a, int64_t n_rows, const DashKbarArgs* ka,
                                cudaStream_t st) {
  DashKbarArgs none = {};
  const int rk = ka == nullptr ? 0 : ka->dtype == DASH_DTYPE_F32 ? 1 : 2;
  const size_t rf = rk ? kbar_pool_smem_floats(ka->block_size, 128) : 0;
  const size_t smem = sizeof(float) * route_cluster_smem_floats(a.width, rf);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_rows * kClusterCtas));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto kern) -> cudaError_t {
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cudaLaunchKernelEx(&cfg, kern, a, ka ? *ka : none);
  };
  const cudaError_t e = rk == 0 ? go(route_cluster_kernel<0>) : rk == 1 ? go(route_cluster_kernel<1>)
                                                                        : go(route_cluster_kernel<2>);
  if (e != cudaSuccess) return set_error(DASH_ERR_CUDA, "route_cluster_kernel launch: %s", cudaGetErrorString(e));
  count_launch();
  return check_launch("route_cluster_kernel");
}

int launch_kbar(const DashKbarArgs& a, cudaStream_t st) {
  dim3 grid;
  if (a.pages == nullptr) {
    int nblk = (a.seq_len + a.block_size - 1) / a.block_size;
    grid = dim3(nblk, a.n_seq);
  } else {
    grid = dim3(a.n_plan);
  }
  if (grid.x == 0 || grid.y == 0) return DASH_OK;
  size_t smem = sizeof(float) * kbar_pool_smem_floats(a.block_size, a.d);
  const bool vec = kbar_vec_ok(a);
  auto go = [&](auto kern) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<grid, 128, smem, st>>>(a);
  };
  if (a.dtype == DASH_DTYPE_F32) {
    if (a.d == 128 && vec) go(kbar_pool_kernel<float, 128, true>);
    else if (vec) go(kbar_pool_kernel<float, 0, true>);
    else go(kbar_pool_kernel<float, 0, false>);
  } else {
    if (a.d == 128 && vec) go(kbar_pool_kernel<__nv_bfloat16, 128, true>);
    else if (vec) go(kbar_pool_kernel<__nv_bfloat16, 0, true>);
    else go(kbar_pool_kernel<__nv_bfloat16, 0, false>);
  }
  count_launch();
  return check_launch("kbar_pool_kernel");
}

int launch_route_refresh(const DashRouteArgs& a, int64_t n_rows, const DashKbarArgs& ka, cudaStream_t st) {
  if (ka.n_plan > 0 && ka.pages && n_rows > 0 && ka.d == 128 && kbar_vec_ok(ka) &&
      route_takes_cluster(a, n_rows))
    return launch_route_cluster(a, n_rows, &ka, st);
  // any other form: the refresh, then the routing (two launches)
  const int rc = ka.n_plan > 0 ? launch_kbar(ka, st) : DASH_OK;
  return rc != DASH_OK ? rc : launch_route(a, n_rows, st);
}

int launch_route(const DashRouteArgs& a, int64_t n_rows, cudaStream_t st) {
  if (n_rows == 0) return DASH_OK;
  int Wp = (a.width + 31) & ~31;
  size_t per_warp = sizeof(float) * ((size_t)a.d + Wp + Wp / 32 + 3 * kMaxM);
  // many rows of few sequences: tiled kernel (k-bar chunks shared by 32 rows)
  if (!a.scores_in && a.width <= 1024 && a.d == 128 && n_rows >= 148 * 16) {
    const int tiles = (a.seqs.max_q_len + kTileRows - 1) / kTileRows;
    const int M = a.topm > 0 ? (a.topm < a.width ? a.topm : a.width) : a.width;
    const size_t sm = sizeof(float) * route_tile_smem_floats(a.width, M);
    cudaFuncSetAttribute(route_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    route_tile_kernel<<<(unsigned)((int64_t)a.seqs.n_seq * tiles), 256, sm, st>>>(a, tiles);
    count_launch();
    return check_launch("route_tile_kernel");
  }
  // few rows (decode): a cluster of CTAs per row scores the blocks in parallel
  if (route_takes_cluster(a, n_rows)) return launch_route_cluster(a, n_rows, nullptr, st);
  // few rows otherwise: one CTA per row so all its threads score; else warp per row
  const bool cta_row = n_rows < 148 * 16;
  size_t smem = per_warp * (cta_row ? 1 : kRouteWarps);
  if (cta_row) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(route_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    route_rows_kernel<true><<<(unsigned)n_rows, kRouteWarps * 32, smem, st>>>(a, n_rows);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(route_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    int64_t grid = (n_rows + kRouteWarps - 1) / kRouteWarps;
    route_rows_kernel<false><<<(unsigned)grid, kRouteWarps * 32, smem, st>>>(a, n_rows);
  }
  count_launch();
  return check_launch("route_rows_kernel");
}

int launch_block_max(const DashBlockMaxArgs& a, cudaStream_t st) {
  dim3 grid((a.C + 31) / 32, a.nblk, a.B);
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return DASH_OK;
  size_t smem = sizeof(float) * ((size_t)(32 + a.block_size) * (a.d + 1) + 256);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(block_max_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  block_max_kernel<<<grid, 128, smem, st>>>(a);
  count_launch();
  return check_launch("block_max_kernel");
}

}  // namespace dash
