// dash_decode_tma.cu -- DASH decode attention over a block-paged KV cache,
// K/V streamed by TMA (sm_100a).
//
// One CTA per (query row, query head, split), as the register-staged kernel
// in dash_decode.cu, with the same work list (the row's routed remote blocks,
// keys below its local window, + bias; then its local-window blocks) and the
// same split merge.  The loads are decoupled from the math:
//
//   producer (warp 4)   builds the work list (ids de-duplicated with one
//                       match per 32 slots), then walks the split's blocks in
//                       16-key chunks: per chunk one 4-D TMA box
//                       {64 dims, 16 tokens, 1 head, 1 page} per half of K
//                       and of V (128-byte swizzle) into a ring of NST stages
//                       of 8 KB, completion on the stage's mbarrier
//   consumers (warps 0-3) chunk n goes to warp n % 4: a warp is 8 groups of 4
//                       lanes, group g takes keys g and g + 8 of the chunk,
//                       lane `sub` 32 of the 128 dims, read from the swizzled
//                       stage (conflict-free); online softmax in the exp2
//                       domain per group, merged by shuffles, then across
//                       warps in shared memory; the stage is released to the
//                       producer after its last read
//
// The ring keeps NST * 8 KB of K/V in flight per CTA all the time, where the
// register-staged kernel has loads in flight only between its compute phases.
// Rows past a page's end (a partial window block) arrive zero-filled and are
// masked like any key past the chunk's valid count.
//
// Semantics: WHL attend_triton.py:307-518 (_dash_sparse_decode_kernel) and
// WHL common.py:40-89 (split merge); modeling_deepseekv2.py:424-451.
#include <cudaTypedefs.h>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {
namespace {

constexpr int kTmaConsumers = 4;
constexpr int kTmaThreads = (kTmaConsumers + 1) * 32;
constexpr int kTmaStages = 8;
constexpr int kChunk = 16;                       // keys per stage
constexpr int kStageBytes = 2 * 2 * kChunk * 128;  // K and V, two 64-dim halves
constexpr int kTmaMaxItems = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct TmaSmem {
  uint8_t stage[kTmaStages][kStageBytes];        // 1024-byte aligned (swizzle atoms)
  int32_t item_page[kTmaMaxItems];
  int32_t item_tok[kTmaMaxItems];                // (token within the page << 16) | keys
  float item_b2[kTmaMaxItems];                   // bias * log2(e), 0 for window blocks
  int32_t chunk_nv[kTmaStages];                  // valid keys of the stage's chunk
  float chunk_b2[kTmaStages];
  uint64_t full[kTmaStages];
  uint64_t empty[kTmaStages];
  float s_o[kTmaConsumers][128];
  float s_m[kTmaConsumers], s_l[kTmaConsumers];
  int n_items, n_chunks, last, abort_flag;
};

__device__ __forceinline__ void unpack8(const uint4 w, float* x, const __nv_bfloat16*) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack2(ws[e], (__nv_bfloat16*)nullptr);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}
__device__ __forceinline__ void unpack8(const uint4 w, float* x, const __half*) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack2(ws[e], (__half*)nullptr);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}

// 32 dims [32 sub, 32 sub + 32) of row j of a swizzled 16-row half pair
// (half h at h * 2048; 16-byte chunk c of row j at ((c ^ (j & 7)) << 4)).
template <typename T>
__device__ __forceinline__ void lds_row32(const uint8_t* base, int j, int sub, float (&x)[32]) {
  const uint8_t* row = base + (sub >> 1) * (kChunk * 128) + j * 128;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int c = (sub & 1) * 4 + u;
    const uint4 w = *reinterpret_cast<const uint4*>(row + ((c ^ (j & 7)) << 4));
    unpack8(w, x + 8 * u, (const T*)nullptr);
  }
}

__device__ __forceinline__ void merge_state32(float& m, float& l, float (&o)[32], float m2, float l2,
                                              const float (&o2)[32]) {
  const float mn = fmaxf(m, m2);
  const float a = (m == -INFINITY) ? 0.0f : fast_exp2(m - mn);
  const float b = (m2 == -INFINITY) ? 0.0f : fast_exp2(m2 - mn);
#pragma unroll
  for (int c = 0; c < 32; ++c) o[c] = o[c] * a + o2[c] * b;
  l = l * a + l2 * b;
  m = mn;
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kTmaThreads) decode_tma_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                  const __grid_constant__ CUtensorMap tmV,
                                                                  const __grid_constant__ DashDecodeArgs a,
                                                                  int splits, float* part, int* counters) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  TmaSmem& S = *reinterpret_cast<TmaSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x % splits;
  const int64_t r = blockIdx.x / splits;
  const int hq = blockIdx.y;
  const int H = a.qo.n_heads;
  const int G = H / a.kv.n_kv_heads;
  const int hk = hq / G;
  const int bs = a.block_size;
  DeviceError* derr = a.device_error;

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
  const int64_t rowq = a.seqs.q_start ? (int64_t)(a.seqs.q_start[s] + i) : -1;

  const int grp = lane >> 2, sub = lane & 3;
  float q[32];
  if (warp < kTmaConsumers) {
    // query, pre-scaled into the exp2 domain (loaded while warp 4 builds the list)
    const T* qp = reinterpret_cast<const T*>(a.qo.q) +
                  (rowq >= 0 ? rowq * a.qo.q_stride_tok
                             : (int64_t)s * a.qo.q_stride_seq + (int64_t)i * a.qo.q_stride_tok) +
                  (int64_t)hq * a.qo.q_stride_head + sub * 32;
    const uint4* q4 = reinterpret_cast<const uint4*>(qp);
    const float sl2 = a.scale * kLog2e;
#pragma unroll
    for (int u = 0; u < 4; ++u) unpack8(__ldg(q4 + u), q + 8 * u, (const T*)nullptr);
#pragma unroll
    for (int c = 0; c < 32; ++c) q[c] *= sl2;
  } else {
    if (lane == 0) {
      for (int k = 0; k < kTmaStages; ++k) {
        mbar_init(&S.full[k], 1);
        mbar_init(&S.empty[k], 1);
      }
      S.abort_flag = 0;
      mbar_init_fence();
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
    }
    // ---- the work list: routed blocks (first occurrence of an id), then the window ----
    const int nih = a.routes.n_index_heads > 0 ? a.routes.n_index_heads : 1;
    const int ih = hq / (H / nih);
    const int32_t* il = a.routes.idx + r * a.routes.row_stride + ih * a.routes.ihead_stride;
    const float* bl = a.routes.bias ? a.routes.bias + r * a.routes.row_stride + ih * a.routes.ihead_stride : nullptr;
    const int Kr = min(a.routes.K, kTmaMaxItems - 32);
    const int32_t* btr = a.kv.block_table + (int64_t)s * a.kv.bt_stride;
    int n = 0;
    for (int j0 = 0; j0 < Kr; j0 += 32) {
      const int j = j0 + lane;
      const int b = j < Kr ? il[j] : -1;
      const float bias = (bl && j < Kr) ? bl[j] : 0.0f;
      bool ok = b >= 0;
      if (ok && b >= nblk_seq) { record_error(derr, DASH_DEV_BAD_BLOCK, 21, b); ok = false; }
      // first occurrence wins: the lowest lane of this slice holding b, and
      // no earlier slice
      const uint32_t same = __match_any_sync(0xffffffffu, b);
      ok &= (same & ((1u << lane) - 1u)) == 0u;
      for (int u = 0; ok && u < j0; ++u) ok &= il[u] != b;
      const int64_t k0 = (int64_t)b * bs;
      const int64_t k1 = min(min((int64_t)(b + 1) * bs, lstart), pos + 1);   // below the window
      ok &= k1 > k0;
      int64_t p = 0;
      if (ok) {
        p = btr[b];
        if (p < 0 || p >= a.kv.num_pages) { record_error(derr, DASH_DEV_BAD_PAGE, 20, p); ok = false; }
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, ok);
      if (ok) {
        const int slot = n + __popc(bal & ((1u << lane) - 1u));
        S.item_page[slot] = (int)p;
        S.item_tok[slot] = (int)(k1 - k0);
        S.item_b2[slot] = bias * kLog2e;
      }
      n += __popc(bal);
    }
    if (pos >= 0) {
      const int b0 = (int)(lstart / bs), b1 = (int)(pos / bs);
      for (int bb = b0; bb <= b1; bb += 32) {
        const int b = bb + lane;
        bool ok = b <= b1 && b < nblk_seq && n + lane < kTmaMaxItems;
        const int64_t k0 = max((int64_t)b * bs, lstart);
        const int64_t k1 = min((int64_t)(b + 1) * bs, pos + 1);
        ok &= k1 > k0;
        int64_t p = 0;
        if (ok) {
          p = btr[b];
          if (p < 0 || p >= a.kv.num_pages) { record_error(derr, DASH_DEV_BAD_PAGE, 22, p); ok = false; }
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, ok);
        if (ok) {
          const int slot = n + __popc(bal & ((1u << lane) - 1u));
          S.item_page[slot] = (int)p;
          S.item_tok[slot] = ((int)(k0 - (int64_t)b * bs) << 16) | (int)(k1 - k0);
          S.item_b2[slot] = 0.0f;
        }
        n += __popc(bal);
      }
    }
    __syncwarp();
    if (lane == 0) {
      const int per = (n + splits - 1) / splits;
      const int it0 = split * per, it1 = min(n, it0 + per);
      int c = 0;
      for (int it = it0; it < it1; ++it) c += ((S.item_tok[it] & 0xffff) + kChunk - 1) / kChunk;
      S.n_items = n;
      S.n_chunks = c;
    }
  }
  __syncthreads();
  const int n_items = S.n_items, n_chunks = S.n_chunks;
  const int per = (n_items + splits - 1) / splits;
  const int it0 = split * per, it1 = min(n_items, it0 + per);
  volatile int* abort_flag = &S.abort_flag;

  float m = -INFINITY, l = 0.0f, o[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) o[c] = 0.0f;

  if (warp == kTmaConsumers) {
    // ============================ producer ============================
    if (lane == 0) {
      int n = 0;
      bool alive = true;
      for (int it = it0; alive && it < it1; ++it) {
        const int page = S.item_page[it];
        const int tok = S.item_tok[it] >> 16, nk = S.item_tok[it] & 0xffff;
        const float b2 = S.item_b2[it];
        for (int c0 = 0; c0 < nk; c0 += kChunk, ++n) {
          const int st = n % kTmaStages;
          if (n >= kTmaStages &&
              !mbar_wait(&S.empty[st], (uint32_t)((n / kTmaStages) - 1) & 1u, abort_flag, derr, 30)) {
            alive = false;
            break;
          }
          S.chunk_nv[st] = min(kChunk, nk - c0);
          S.chunk_b2[st] = b2;
          mbar_arrive_expect_tx(&S.full[st], kStageBytes);
          uint8_t* dst = S.stage[st];
          tma_load_4d(dst, &tmK, &S.full[st], 0, tok + c0, hk, page);
          tma_load_4d(dst + kChunk * 128, &tmK, &S.full[st], 64, tok + c0, hk, page);
          tma_load_4d(dst + 2 * kChunk * 128, &tmV, &S.full[st], 0, tok + c0, hk, page);
          tma_load_4d(dst + 3 * kChunk * 128, &tmV, &S.full[st], 64, tok + c0, hk, page);
        }
      }
      // never leave the CTA with bulk copies in flight: the last chunk of
      // every stage has landed
      volatile int no_abort = 0;
      for (int k = n - 1; k >= 0 && k >= n - kTmaStages; --k)
        mbar_wait(&S.full[k % kTmaStages], (uint32_t)(k / kTmaStages) & 1u, &no_abort, nullptr, 31);
    }
    __syncwarp();
  } else {
    // ============================ consumers ============================
    for (int n = warp; n < n_chunks; n += kTmaConsumers) {
      const int st = n % kTmaStages;
      if (!mbar_wait_warp(&S.full[st], (uint32_t)(n / kTmaStages) & 1u, abort_flag, derr, 32)) break;
      const int nv = S.chunk_nv[st];
      const float b2 = S.chunk_b2[st];
      const uint8_t* sk = S.stage[st];
      const uint8_t* sv = sk + 2 * kChunk * 128;
      const bool one = grp < nv, two = grp + 8 < nv;
      // rows past the valid count (cache rows past the query's position, or
      // zero fill past the page) are never read: masked lanes read row 0
      const int j0 = one ? grp : 0, j1 = two ? grp + 8 : 0;
      float s0 = 0.0f, s1 = 0.0f;
      {
        float k0[32], k1[32];
        lds_row32<T>(sk, j0, sub, k0);
        lds_row32<T>(sk, j1, sub, k1);
#pragma unroll
        for (int c = 0; c < 32; ++c) { s0 = fmaf(q[c], k0[c], s0); s1 = fmaf(q[c], k1[c], s1); }
      }
      s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      s0 = one ? s0 + b2 : -INFINITY;
      s1 = two ? s1 + b2 : -INFINITY;
      const float mn = fmaxf(m, fmaxf(s0, s1));
      if (mn != -INFINITY) {
        const float alpha = (m == -INFINITY) ? 0.0f : fast_exp2(m - mn);
        const float p0 = one ? fast_exp2(s0 - mn) : 0.0f;
        const float p1 = two ? fast_exp2(s1 - mn) : 0.0f;
        float v0[32], v1[32];
        lds_row32<T>(sv, j0, sub, v0);
        lds_row32<T>(sv, j1, sub, v1);
        l = l * alpha + p0 + p1;
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = fmaf(p1, v1[c], fmaf(p0, v0[c], o[c] * alpha));
        m = mn;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[st]);
    }
    // ---- merge the 8 groups of the warp (lanes with the same `sub`) ----
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
      float o2[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) o2[c] = __shfl_xor_sync(0xffffffffu, o[c], off);
      merge_state32(m, l, o, m2, l2, o2);
    }
    if (grp == 0) {
#pragma unroll
      for (int c = 0; c < 32; ++c) S.s_o[warp][sub * 32 + c] = o[c];
      if (sub == 0) { S.s_m[warp] = m; S.s_l[warp] = l; }
    }
  }
  __syncthreads();
  // ---- merge the consumer warps: thread c < 128 owns dim c ----
  const int c = threadIdx.x;
  const bool dim_thread = c < 128;
  float M = -INFINITY, L = 0.0f, O = 0.0f;
  if (dim_thread) {
    for (int w = 0; w < kTmaConsumers; ++w) M = fmaxf(M, S.s_m[w]);
    for (int w = 0; w < kTmaConsumers; ++w) {
      const float f = (S.s_m[w] == -INFINITY) ? 0.0f : fast_exp2(S.s_m[w] - M);
      L += S.s_l[w] * f;
      O += S.s_o[w][c] * f;
    }
  }
  const int64_t ob = (rowq >= 0 ? rowq * a.qo.o_stride_tok
                                : (int64_t)s * a.qo.o_stride_seq + (int64_t)i * a.qo.o_stride_tok) +
                     (int64_t)hq * a.qo.o_stride_head;
  const int64_t lb = a.qo.lse ? (rowq >= 0 ? rowq * a.qo.lse_stride_tok
                                           : (int64_t)s * a.qo.lse_stride_seq + (int64_t)i * a.qo.lse_stride_tok) +
                                    (int64_t)hq * a.qo.lse_stride_head
                              : 0;
  T* out = reinterpret_cast<T*>(a.qo.out);
  if (splits == 1) {
    if (dim_thread) {
      out[ob + c] = (T)(L > 0.0f ? O / L : 0.0f);
      if (a.qo.lse && c == 0) a.qo.lse[lb] = L > 0.0f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
    }
    return;
  }
  // ---- split-KV: publish the partial, the last CTA of the (row, head) merges ----
  const int64_t unit = r * H + hq;
  float* mypart = part + (unit * splits + split) * 130;
  if (dim_thread) {
    mypart[c] = O;
    if (c == 0) { mypart[128] = M; mypart[129] = L; }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) S.last = atomicAdd(counters + unit, 1) == splits - 1;
  __syncthreads();
  if (!S.last || !dim_thread) return;
  __threadfence();
  const float* up = part + unit * splits * 130;
  float MM = -INFINITY;
  for (int k = 0; k < splits; ++k) MM = fmaxf(MM, __ldcg(up + k * 130 + 128));
  float LL = 0.0f, OO = 0.0f;
  for (int k = 0; k < splits; ++k) {
    const float mk = __ldcg(up + k * 130 + 128);
    const float f = (mk == -INFINITY) ? 0.0f : fast_exp2(mk - MM);
    LL += __ldcg(up + k * 130 + 129) * f;
    OO += __ldcg(up + k * 130 + c) * f;
  }
  out[ob + c] = (T)(LL > 0.0f ? OO / LL : 0.0f);
  if (a.qo.lse && c == 0) a.qo.lse[lb] = LL > 0.0f ? (MM + log2f(LL)) * 0.6931471805599453f : -INFINITY;
  if (c == 0) counters[unit] = 0;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 decode_encode_fn() {
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

static size_t decode_tma_smem() { return sizeof(TmaSmem) + 1024; }

bool decode_tma_supported(const DashDecodeArgs& a) {
  const int64_t e = 8;   // 16 bytes of bf16 / fp16
  return a.kv.block_table != nullptr && a.kv.head_dim == 128 &&
         (a.kv.dtype == DASH_DTYPE_BF16 || a.kv.dtype == DASH_DTYPE_F16) && a.block_size >= kChunk &&
         a.block_size <= 4096 && a.kv.num_pages > 0 && a.kv.num_pages < (int64_t)INT32_MAX &&
         a.kv.stride_tok > 0 && a.kv.stride_head > 0 && a.kv.stride_seq > 0 && a.kv.stride_tok % e == 0 &&
         a.kv.stride_head % e == 0 && a.kv.stride_seq % e == 0 &&
         (reinterpret_cast<uintptr_t>(a.kv.k) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.kv.v) & 15) == 0 &&
         decode_encode_fn() != nullptr;
}

// CTA slots of the whole GPU for decode_tma_kernel.
int decode_tma_slots() {
  static int slots[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148 * 3;
  if (slots[dev] == 0) {
    int sms = 0, per = 0;
    const int smem = (int)decode_tma_smem();
    cudaFuncSetAttribute(decode_tma_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, decode_tma_kernel<__nv_bfloat16>, kTmaThreads, smem);
    slots[dev] = (sms > 0 && per > 0) ? sms * per : 148 * 3;
  }
  return slots[dev];
}

static int make_page_map(CUtensorMap* map, const void* base, const DashDecodeArgs& a) {
  cuuint64_t dims[4] = {128, (cuuint64_t)a.block_size, (cuuint64_t)a.kv.n_kv_heads, (cuuint64_t)a.kv.num_pages};
  cuuint64_t strides[3] = {(cuuint64_t)a.kv.stride_tok * 2, (cuuint64_t)a.kv.stride_head * 2,
                           (cuuint64_t)a.kv.stride_seq * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)kChunk, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = decode_encode_fn()(
      map, a.kv.dtype == DASH_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
      const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DASH_ERR_CUDA, "cuTensorMapEncodeTiled (decode K/V) failed (%d)", (int)r);
  return DASH_OK;
}

int launch_decode_tma(const DashDecodeArgs& a, int64_t n_rows, int splits, float* part, int* counters,
                      cudaStream_t st) {
  CUtensorMap mk, mv;
  int rc = make_page_map(&mk, a.kv.k, a);
  if (rc == DASH_OK) rc = make_page_map(&mv, a.kv.v, a);
  if (rc != DASH_OK) return rc;
  const int smem = (int)decode_tma_smem();
  const dim3 grid((unsigned)(n_rows * splits), a.qo.n_heads);
  if (a.kv.dtype == DASH_DTYPE_BF16) {
    cudaFuncSetAttribute(decode_tma_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    decode_tma_kernel<__nv_bfloat16><<<grid, kTmaThreads, smem, st>>>(mk, mv, a, splits, part, counters);
  } else {
    cudaFuncSetAttribute(decode_tma_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    decode_tma_kernel<__half><<<grid, kTmaThreads, smem, st>>>(mk, mv, a, splits, part, counters);
  }
  count_launch();
  return check_launch("decode_tma_kernel");
}

}  // namespace dash
