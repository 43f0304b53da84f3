// dash_decode.cu -- DASH decode attention over a block-paged KV cache.
//
// One CTA per (query row, query head, split).  The row's work list is its
// routed remote blocks (keys below the local window, + bias) followed by the
// blocks of its local window (no bias); split s takes a contiguous slice of
// that list.  Inside a CTA each warp walks whole blocks; a warp is 8 groups of
// 4 lanes, a group owns one key at a time and each lane of it 32 of the 128
// head dims (four 16-byte loads of K and of V per key).  Every group keeps its
// own online softmax (exp2 domain), merged by shuffles, then across warps in
// shared memory.  With several splits the CTA stores an unnormalised partial
// (o, m, l) in the workspace and bumps a per-(row, head) counter; the CTA that
// brings the counter to `splits` merges all partials and resets the counter,
// so no CTA waits for another.
//
// Semantics: WHL attend_triton.py:307-518 (_dash_sparse_decode_kernel) and
// WHL common.py:40-89 (split merge); modeling_deepseekv2.py:424-451.
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {

constexpr int kDecWarps = 4;
constexpr int kMaxDecItems = 512;   // remote slots + local blocks per row

struct DecItem {
  int32_t page_base_hi;  // unused padding for alignment
  int32_t key0, nkeys;   // first key (position) and count
  int32_t remote;        // 1: routed block (bias applies)
  float bias;            // natural-log bias
  int64_t base;          // element offset of key0 for this head
};

template <typename T>
__device__ __forceinline__ void load_row32(const T* p, float (&x)[32]) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 w = __ldg(p4 + u);
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = unpack2(ws[e], (T*)nullptr);
      x[u * 8 + 2 * e] = f.x;
      x[u * 8 + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void merge_state(float& m, float& l, float (&o)[32], float m2, float l2,
                                            const float (&o2)[32]) {
  float mn = fmaxf(m, m2);
  float a = (m == -INFINITY) ? 0.0f : fast_exp2(m - mn);
  float b = (m2 == -INFINITY) ? 0.0f : fast_exp2(m2 - mn);
#pragma unroll
  for (int c = 0; c < 32; ++c) o[c] = o[c] * a + o2[c] * b;
  l = l * a + l2 * b;
  m = mn;
}

template <typename T>
__global__ void __launch_bounds__(kDecWarps * 32) decode_kernel(DashDecodeArgs a, int splits,
                                                                float* part, int* counters) {
  __shared__ DecItem items[kMaxDecItems];
  __shared__ int s_nitems;
  __shared__ float s_m[kDecWarps], s_l[kDecWarps];
  __shared__ float s_o[kDecWarps][128];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x % splits;
  const int64_t r = blockIdx.x / splits;
  const int hq = blockIdx.y;
  const int H = a.qo.n_heads;
  const int G = H / a.kv.n_kv_heads;
  const int hk = hq / G;
  const int bs = a.block_size;

  int s, i;
  {
    const DashSeqs& q = a.seqs;
    if (q.q_start == nullptr) { s = (int)(r / q.q_len_fixed); i = (int)(r - (int64_t)s * q.q_len_fixed); }
    else {
      int lo = 0, hi = q.n_seq - 1;
      while (lo < hi) { int mid = (lo + hi + 1) >> 1; if (q.q_start[mid] <= r) lo = mid; else hi = mid - 1; }
      s = lo; i = (int)(r - q.q_start[lo]);
    }
  }
  const int kvl = a.seqs.kv_len ? a.seqs.kv_len[s] : a.seqs.kv_len_fixed;
  const int qlen = a.seqs.q_start ? a.seqs.q_start[s + 1] - a.seqs.q_start[s] : a.seqs.q_len_fixed;
  const int64_t pos = (int64_t)(a.seqs.pos0 ? a.seqs.pos0[s] : kvl - qlen) + i;
  const int64_t lstart = pos - a.local_window + 1 > 0 ? pos - a.local_window + 1 : 0;
  const int nblk_seq = (kvl + bs - 1) / bs;

  // ---- query (pre-scaled into the exp2 domain); loaded by every warp while
  // warp 0 builds the work list ----
  const int grp = lane >> 2, sub = lane & 3;
  const float sl2 = a.scale * 1.4426950408889634f;
  float q[32];
  {
    const T* qp = reinterpret_cast<const T*>(a.qo.q) +
                  (a.seqs.q_start ? (int64_t)(a.seqs.q_start[s] + i) * a.qo.q_stride_tok
                                  : (int64_t)s * a.qo.q_stride_seq + (int64_t)i * a.qo.q_stride_tok) +
                  (int64_t)hq * a.qo.q_stride_head + sub * 32;
    load_row32(qp, q);
#pragma unroll
    for (int c = 0; c < 32; ++c) q[c] *= sl2;
  }
  // ---- build the work list (warp 0, one routed slot per lane) ----
  if (warp == 0) {
    const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
    const int ih = hq / (H / nih);
    const int32_t* il = a.routes.idx + r * a.routes.row_stride + ih * a.routes.ihead_stride;
    const float* bl = a.routes.bias ? a.routes.bias + r * a.routes.row_stride + ih * a.routes.ihead_stride : nullptr;
    const int Kr = min(a.routes.K, kMaxDecItems - 32);
    int n = 0;
    for (int j0 = 0; j0 < Kr; j0 += 32) {
      const int j = j0 + lane;
      int b = j < Kr ? il[j] : -1;
      bool ok = b >= 0;
      if (ok && b >= nblk_seq) { record_error(a.device_error, DASH_DEV_BAD_BLOCK, 21, b); ok = false; }
      if (ok) {                                   // first occurrence of a duplicated id wins
#pragma unroll 8
        for (int u = 0; u < j; ++u) ok &= il[u] != b;
      }
      int64_t k0 = (int64_t)b * bs;
      int64_t k1 = min(min((int64_t)(b + 1) * bs, lstart), pos + 1);  // below the window
      ok &= k1 > k0;
      int64_t base = 0;
      if (ok) {
        if (a.kv.block_table) {
          int64_t p = a.kv.block_table[(int64_t)s * a.kv.bt_stride + b];
          if (p < 0 || p >= a.kv.num_pages) {
            record_error(a.device_error, DASH_DEV_BAD_PAGE, 20, p);
            ok = false;
          }
          base = p * a.kv.stride_seq + (int64_t)hk * a.kv.stride_head;
        } else {
          base = (int64_t)s * a.kv.stride_seq + k0 * a.kv.stride_tok + (int64_t)hk * a.kv.stride_head;
        }
      }
      uint32_t bal = __ballot_sync(0xffffffffu, ok);
      if (ok) {
        int slot = n + __popc(bal & ((1u << lane) - 1u));
        items[slot].key0 = (int)k0; items[slot].nkeys = (int)(k1 - k0);
        items[slot].remote = 1; items[slot].bias = bl ? bl[j] : 0.0f; items[slot].base = base;
      }
      n += __popc(bal);
    }
    // local window blocks: lane t takes block lstart/bs + t
    if (pos >= 0) {
      const int b0 = (int)(lstart / bs), b1 = (int)(pos / bs);
      for (int bb = b0; bb <= b1; bb += 32) {
        const int b = bb + lane;
        bool ok = b <= b1 && b < nblk_seq && n + lane < kMaxDecItems;
        int64_t k0 = max((int64_t)b * bs, lstart);
        int64_t k1 = min((int64_t)(b + 1) * bs, pos + 1);
        ok &= k1 > k0;
        int64_t base = 0;
        if (ok) {
          if (a.kv.block_table) {
            int64_t p = a.kv.block_table[(int64_t)s * a.kv.bt_stride + b];
            if (p < 0 || p >= a.kv.num_pages) {
              record_error(a.device_error, DASH_DEV_BAD_PAGE, 22, p);
              ok = false;
            }
            base = p * a.kv.stride_seq + (k0 - (int64_t)b * bs) * a.kv.stride_tok +
                   (int64_t)hk * a.kv.stride_head;
          } else {
            base = (int64_t)s * a.kv.stride_seq + k0 * a.kv.stride_tok + (int64_t)hk * a.kv.stride_head;
          }
        }
        uint32_t bal = __ballot_sync(0xffffffffu, ok);
        if (ok) {
          int slot = n + __popc(bal & ((1u << lane) - 1u));
          items[slot].key0 = (int)k0; items[slot].nkeys = (int)(k1 - k0);
          items[slot].remote = 0; items[slot].bias = 0.0f; items[slot].base = base;
        }
        n += __popc(bal);
      }
    }
    if (lane == 0) s_nitems = n;
  }
  __syncthreads();
  const int n_items = s_nitems;
  const int per = (n_items + splits - 1) / splits;
  const int it0 = split * per, it1 = min(n_items, it0 + per);

  float m = -INFINITY, l = 0.0f, o[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) o[c] = 0.0f;

  const T* kbase = reinterpret_cast<const T*>(a.kv.k);
  const T* vbase = reinterpret_cast<const T*>(a.kv.v);
  for (int it = it0 + warp; it < it1; it += kDecWarps) {
    const DecItem item = items[it];
    const float b2 = item.remote ? item.bias * 1.4426950408889634f : 0.0f;
    // Two keys per group per step (j, j+8): 16 loads of 16 B in flight per lane.
    // The trip count is the same for every lane of the warp (the shuffles
    // below need all 32 lanes); lanes past the end use key 0 and mask it.
    for (int j0 = 0; j0 < item.nkeys; j0 += 16) {
      const int j = j0 + grp;
      const bool one = j < item.nkeys;
      const bool two = j + 8 < item.nkeys;
      const int64_t off0 = item.base + (int64_t)(one ? j : 0) * a.kv.stride_tok + sub * 32;
      const int64_t off1 = item.base + (int64_t)(two ? j + 8 : 0) * a.kv.stride_tok + sub * 32;
      float k0[32], k1[32], v0[32], v1[32];
      load_row32(kbase + off0, k0);
      load_row32(kbase + off1, k1);
      load_row32(vbase + off0, v0);
      load_row32(vbase + off1, v1);
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
      for (int c = 0; c < 32; ++c) { s0 = fmaf(q[c], k0[c], s0); s1 = fmaf(q[c], k1[c], s1); }
      s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      s0 = one ? s0 + b2 : -INFINITY;
      s1 = two ? s1 + b2 : -INFINITY;
      const float mn = fmaxf(m, fmaxf(s0, s1));
      if (mn == -INFINITY) continue;                  // nothing valid yet for this group
      const float alpha = (m == -INFINITY) ? 0.0f : fast_exp2(m - mn);
      const float p0 = one ? fast_exp2(s0 - mn) : 0.0f;
      const float p1 = two ? fast_exp2(s1 - mn) : 0.0f;
      l = l * alpha + p0 + p1;
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = fmaf(p1, v1[c], fmaf(p0, v0[c], o[c] * alpha));
      m = mn;
    }
  }
  // ---- merge the 8 groups of the warp (lanes with the same `sub`) ----
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    float l2 = __shfl_xor_sync(0xffffffffu, l, off);
    float o2[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) o2[c] = __shfl_xor_sync(0xffffffffu, o[c], off);
    merge_state(m, l, o, m2, l2, o2);
  }
  if (grp == 0) {
#pragma unroll
    for (int c = 0; c < 32; ++c) s_o[warp][sub * 32 + c] = o[c];
    if (sub == 0) { s_m[warp] = m; s_l[warp] = l; }
  }
  __syncthreads();
  // ---- merge warps: thread t < 128 owns dim t ----
  float M = -INFINITY;
  for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, s_m[w]);
  float L = 0.0f, O = 0.0f;
  const int c = threadIdx.x;
  for (int w = 0; w < kDecWarps; ++w) {
    float f = (s_m[w] == -INFINITY) ? 0.0f : fast_exp2(s_m[w] - M);
    L += s_l[w] * f;
    O += s_o[w][c] * f;
  }
  const int64_t ob = (a.seqs.q_start ? (int64_t)(a.seqs.q_start[s] + i) * a.qo.o_stride_tok
                                     : (int64_t)s * a.qo.o_stride_seq + (int64_t)i * a.qo.o_stride_tok) +
                     (int64_t)hq * a.qo.o_stride_head;
  const int64_t lb = a.qo.lse ? (a.seqs.q_start ? (int64_t)(a.seqs.q_start[s] + i) * a.qo.lse_stride_tok
                                                : (int64_t)s * a.qo.lse_stride_seq + (int64_t)i * a.qo.lse_stride_tok) +
                                    (int64_t)hq * a.qo.lse_stride_head
                              : 0;
  T* out = reinterpret_cast<T*>(a.qo.out);
  if (splits == 1) {
    float v = L > 0.0f ? O / L : 0.0f;
    out[ob + c] = (T)v;
    if (a.qo.lse && c == 0) a.qo.lse[lb] = L > 0.0f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
    return;
  }
  // ---- split-KV: publish the partial, the last CTA merges ----
  const int64_t unit = r * H + hq;
  float* mypart = part + (unit * splits + split) * 130;
  mypart[c] = O;
  if (c == 0) { mypart[128] = M; mypart[129] = L; }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int old = atomicAdd(counters + unit, 1);
    s_last = (old == splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* up = part + unit * splits * 130;
  float MM = -INFINITY;
  for (int k = 0; k < splits; ++k) MM = fmaxf(MM, __ldcg(up + k * 130 + 128));
  float LL = 0.0f, OO = 0.0f;
  for (int k = 0; k < splits; ++k) {
    float mk = __ldcg(up + k * 130 + 128);
    float f = (mk == -INFINITY) ? 0.0f : fast_exp2(mk - MM);
    LL += __ldcg(up + k * 130 + 129) * f;
    OO += __ldcg(up + k * 130 + c) * f;
  }
  out[ob + c] = (T)(LL > 0.0f ? OO / LL : 0.0f);
  if (a.qo.lse && c == 0) a.qo.lse[lb] = LL > 0.0f ? (MM + log2f(LL)) * 0.6931471805599453f : -INFINITY;
  if (threadIdx.x == 0) counters[unit] = 0;
}

// CTA slots of the whole GPU for decode_kernel (resident CTAs per SM x SMs).
static int decode_slots() {
  static int slots[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148 * 4;
  if (slots[dev] == 0) {
    int sms = 0, per = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, decode_kernel<__nv_bfloat16>, kDecWarps * 32, 0);
    slots[dev] = (sms > 0 && per > 0) ? sms * per : 148 * 4;
  }
  return slots[dev];
}

// Split count minimising (waves of CTAs) x (per-CTA work): a row's work is its
// routed blocks plus window blocks; every CTA also pays a fixed prologue
// (work list, query) worth about 1.5 blocks.  Waves are counted whole, so the
// choice avoids a nearly empty last wave.
int decode_auto_splits(const DashDecodeArgs& a, int64_t n_rows) {
  const int64_t units = n_rows * a.qo.n_heads;
  const int items = a.routes.K + a.local_window / a.block_size + 1;
  const int64_t slots = decode_tma_supported(a) ? decode_tma_slots() : decode_slots();
  int best = 1;
  double best_cost = 1e300;
  for (int sp = 1; sp <= 16 && sp <= items; ++sp) {
    const double waves = (double)((units * sp + slots - 1) / slots);
    const double cost = waves * ((double)items / sp + 1.5);
    if (cost < best_cost * 0.999) { best_cost = cost; best = sp; }
  }
  return best;
}

size_t decode_workspace(const DashDecodeArgs& a, int64_t n_rows, int splits) {
  if (splits <= 1) return 0;
  int64_t units = n_rows * a.qo.n_heads;
  size_t part = (size_t)units * splits * 130 * sizeof(float);
  part = (part + 255) & ~(size_t)255;
  return part + (size_t)units * sizeof(int);
}

int launch_decode(const DashDecodeArgs& a, int64_t n_rows, int splits, cudaStream_t st) {
  if (n_rows == 0) return DASH_OK;
  float* part = nullptr;
  int* counters = nullptr;
  if (splits > 1) {
    int64_t units = n_rows * a.qo.n_heads;
    size_t p = (size_t)units * splits * 130 * sizeof(float);
    p = (p + 255) & ~(size_t)255;
    part = reinterpret_cast<float*>(a.workspace);
    counters = reinterpret_cast<int*>(reinterpret_cast<char*>(a.workspace) + p);
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)units * sizeof(int), st);
    if (e != cudaSuccess) return set_error(DASH_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }
  if (decode_tma_supported(a)) return launch_decode_tma(a, n_rows, splits, part, counters, st);
  dim3 grid((unsigned)(n_rows * splits), a.qo.n_heads);
  if (a.kv.dtype == DASH_DTYPE_BF16)
    decode_kernel<__nv_bfloat16><<<grid, kDecWarps * 32, 0, st>>>(a, splits, part, counters);
  else
    decode_kernel<__half><<<grid, kDecWarps * 32, 0, st>>>(a, splits, part, counters);
  count_launch();
  return check_launch("decode_kernel");
}

}  // namespace dash
