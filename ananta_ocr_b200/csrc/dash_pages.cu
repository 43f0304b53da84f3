// dash_pages.cu -- page-aware candidate domains of the DASH router (image
// pages of an OCR document):
//   page_ids_kernel     token ids -> per-token image / query page ids and the
//                       per-block page descriptors, one 8-CTA cluster per row
//   page_state_kernel   per-slot page bookkeeping of a block-paged KV cache for
//                       one serving step (one CTA per request), refreshing the
//                       page bounds of the physical blocks the step wrote
//   page_allow_kernel   dense per-row candidate masks (one warp per row)
//   page_decode_kernel  decode-step query page of the contiguous decoder
//   block_any_kernel    any() of a token mask per block
//
// All of it is integer work over token ids (8 B per token in, a few bytes per
// token out): the kernels read the ids once with coalesced loads, turn them
// into 2-bit flags (image, page marker) staged in shared memory, and derive
// the prefix counts (markers, image tokens) with block scans; the page
// descriptors of a block come from the same staged tile, so nothing is
// re-read from HBM.
#include <climits>
#include <cooperative_groups.h>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {

namespace cg = cooperative_groups;

__device__ __forceinline__ uint32_t token_flags(int64_t id, int64_t img_id, int64_t mm_shift,
                                                int has_pg, int64_t pg_id) {
  const bool img = id == img_id || (mm_shift > 0 && id >= mm_shift);
  const bool mk = has_pg && id == pg_id;
  return (uint32_t)img | ((uint32_t)mk << 1);
}

__device__ __forceinline__ void store_page(void* base, int elem_bytes, int64_t i, int v) {
  if (elem_bytes == 8) reinterpret_cast<int64_t*>(base)[i] = v;
  else reinterpret_cast<int32_t*>(base)[i] = v;
}

__device__ __forceinline__ int64_t load_page(const void* base, int elem_bytes, int64_t i) {
  return elem_bytes == 8 ? reinterpret_cast<const int64_t*>(base)[i]
                         : (int64_t)reinterpret_cast<const int32_t*>(base)[i];
}

__device__ __forceinline__ uint32_t flag_at(uint2 f, int j) {
  return ((j < 4 ? f.x >> (8 * j) : f.y >> (8 * (j - 4)))) & 0xffu;
}

// Exclusive block scan of a sum; `total` receives the block total.  swarp:
// >= NT/32 words of shared memory.
template <int NT>
__device__ __forceinline__ uint32_t block_excl_sum(uint32_t v, uint32_t* swarp, uint32_t& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) swarp[w] = x;
  __syncthreads();
  if (w == 0) {
    uint32_t t = lane < NT / 32 ? swarp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < NT / 32) swarp[lane] = t;
  }
  __syncthreads();
  const uint32_t base = w > 0 ? swarp[w - 1] : 0u;
  total = swarp[NT / 32 - 1];
  __syncthreads();
  return base + x - v;
}

// Exclusive block max-scan of non-negative ints (identity 0).
template <int NT>
__device__ __forceinline__ int block_excl_max(int v, int* swarp, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x = max(x, y);
  }
  int ex = __shfl_up_sync(0xffffffffu, x, 1);
  if (lane == 0) ex = 0;
  if (lane == 31) swarp[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = lane < NT / 32 ? swarp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t = max(t, y);
    }
    if (lane < NT / 32) swarp[lane] = t;
  }
  __syncthreads();
  const int base = w > 0 ? swarp[w - 1] : 0;
  total = swarp[NT / 32 - 1];
  __syncthreads();
  return max(base, ex);
}

// ---------------------------------------------------------------------------
// page_ids_kernel: one cluster of kIdCluster CTAs per row.  The row is cut in
// tiles of kIdTile tokens, tile k owned by CTA k % kIdCluster.
//   phase 1: per tile, marker / image counts, last image token and markers up
//            to it -> a tile summary in the owner's shared memory;
//   cluster barrier; warp 0 of every CTA reads all summaries through
//            distributed shared memory, scans them (tile prefixes, the row's
//            last image token and pp); cluster barrier (summaries released);
//   phase 2: per tile, block scan of the flags, per-token pages, coalesced
//            stores, and the page descriptors of the tile's blocks.
// Restates _sparse_base_impl.py:2189-2260 (rule 0) and
// modeling_anantaocr.py:468-481 (rule 1).
// ---------------------------------------------------------------------------
constexpr int kIdThreads = 256;
constexpr int kIdPer = 8;
constexpr int kIdTile = kIdThreads * kIdPer;   // 2048 tokens
constexpr int kIdCluster = 8;
constexpr int kIdMaxTilesPerCta = 512;         // rows up to 8 * 512 * 2048 tokens

struct PgTile {
  int n_mark, n_img, last_img, mark_upto;      // last_img: position in the row or -1
};

__global__ void __cluster_dims__(kIdCluster, 1, 1) __launch_bounds__(kIdThreads)
    page_ids_kernel(DashPageIdsArgs a) {
  __shared__ __align__(16) uint8_t sflag[kIdTile];
  __shared__ int spage[kIdTile];
  __shared__ int sqp[kIdTile];
  __shared__ PgTile ssum[kIdMaxTilesPerCta];
  __shared__ int spre_m[kIdMaxTilesPerCta];
  __shared__ int spre_i[kIdMaxTilesPerCta];
  __shared__ uint32_t swarp[32];
  __shared__ int sred[32];
  __shared__ int srow[4];

  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int row = blockIdx.x / kIdCluster;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = a.key_length;
  const int n_tiles = (S + kIdTile - 1) / kIdTile;
  const int64_t* ids = a.token_ids + (int64_t)row * a.ids_stride;

  // Stages the flags of tile t0 (coalesced id loads) and returns this
  // thread's 8 consecutive flags.
  auto load_flags = [&](int t0) -> uint2 {
#pragma unroll
    for (int j = 0; j < kIdPer; ++j) {
      const int off = j * kIdThreads + tid;
      const int t = t0 + off;
      uint32_t f = 0;
      if (t < S) {
        const int64_t id = t < a.ids_len ? __ldg(ids + t) : (int64_t)-1;
        f = token_flags(id, a.image_token_id, a.mm_pad_shift, a.has_page_token, a.page_token_id);
      }
      sflag[off] = (uint8_t)f;
    }
    __syncthreads();
    return *reinterpret_cast<const uint2*>(sflag + tid * kIdPer);
  };

  if (rank == 0 && tid == 0 && a.n_query) a.n_query[row] = 0;

  // ---- phase 1: tile summaries ----
  for (int k = rank; k < n_tiles; k += kIdCluster) {
    const uint2 fl = load_flags(k * kIdTile);
    uint32_t cnt = 0;
    int last = -1;
#pragma unroll
    for (int j = 0; j < kIdPer; ++j) {
      const uint32_t f = flag_at(fl, j);
      cnt += ((f >> 1) << 16) | (f & 1u);
      if (f & 1u) last = tid * kIdPer + j;
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    last = __reduce_max_sync(0xffffffffu, last);
    if (lane == 0) {
      swarp[warp] = cnt;
      sred[warp] = last;
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t c = lane < kIdThreads / 32 ? swarp[lane] : 0u;
      int l = lane < kIdThreads / 32 ? sred[lane] : -1;
      c = __reduce_add_sync(0xffffffffu, c);
      l = __reduce_max_sync(0xffffffffu, l);
      if (lane == 0) {
        swarp[0] = c;
        sred[0] = l;
      }
    }
    __syncthreads();
    const uint32_t tile_cnt = swarp[0];
    const int tile_last = sred[0];
    __syncthreads();
    // markers at offsets <= the tile's last image token
    uint32_t mu = 0;
#pragma unroll
    for (int j = 0; j < kIdPer; ++j)
      mu += (flag_at(fl, j) >> 1) & (uint32_t)(tid * kIdPer + j <= tile_last);
    mu = __reduce_add_sync(0xffffffffu, mu);
    if (lane == 0) swarp[warp] = mu;
    __syncthreads();
    if (warp == 0) {
      uint32_t c = lane < kIdThreads / 32 ? swarp[lane] : 0u;
      c = __reduce_add_sync(0xffffffffu, c);
      if (lane == 0) {
        PgTile t;
        t.n_mark = (int)(tile_cnt >> 16);
        t.n_img = (int)(tile_cnt & 0xffffu);
        t.last_img = tile_last >= 0 ? k * kIdTile + tile_last : -1;
        t.mark_upto = (int)c;
        ssum[k / kIdCluster] = t;
      }
    }
    __syncthreads();
  }
  cl.sync();

  // ---- tile prefixes and row totals (warp 0 of every CTA) ----
  if (warp == 0) {
    int carry_m = 0, carry_i = 0, pp = 0, last = -1;
    for (int k0 = 0; k0 < n_tiles; k0 += 32) {
      const int k = k0 + lane;
      PgTile t = {0, 0, -1, 0};
      if (k < n_tiles) {
        const PgTile* rs = cl.map_shared_rank(ssum, k % kIdCluster);
        t = rs[k / kIdCluster];
      }
      int sm = t.n_mark, si = t.n_img;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int ym = __shfl_up_sync(0xffffffffu, sm, o);
        const int yi = __shfl_up_sync(0xffffffffu, si, o);
        if (lane >= o) {
          sm += ym;
          si += yi;
        }
      }
      const int ex_m = carry_m + sm - t.n_mark, ex_i = carry_i + si - t.n_img;
      if (k < n_tiles && k % kIdCluster == rank) {
        spre_m[k / kIdCluster] = ex_m;
        spre_i[k / kIdCluster] = ex_i;
      }
      const int best = __reduce_max_sync(0xffffffffu, (k < n_tiles && t.last_img >= 0) ? k : -1);
      const int v_last = __shfl_sync(0xffffffffu, t.last_img, best >= 0 ? best - k0 : 0);
      const int v_pp = __shfl_sync(0xffffffffu, ex_m + t.mark_upto, best >= 0 ? best - k0 : 0);
      if (best >= 0) {
        last = v_last;
        pp = v_pp;
      }
      carry_m += __shfl_sync(0xffffffffu, sm, 31);
      carry_i += __shfl_sync(0xffffffffu, si, 31);
    }
    if (lane == 0) {
      srow[0] = pp;
      srow[1] = last;
      if (rank == 0) {
        if (a.prompt_pages) a.prompt_pages[row] = pp;
        if (a.marker_count) a.marker_count[row] = carry_m;
        if (a.n_image) a.n_image[row] = carry_i;
      }
    }
  }
  cl.sync();   // every CTA has read the peers' summaries

  // ---- phase 2: per-token pages and block descriptors ----
  const int pp = srow[0], last = srow[1];
  const bool marker_mode = pp > 0;
  const int per_page = a.per_page;
  const int bs = a.block_size;
  const bool blocks = (a.blk_lo || a.blk_hi || a.blk_bits || a.blk_has_image) && a.n_blocks > 0;
  const int words = bs >= 32 ? bs / 32 : 1;
  int nq_cta = 0;
  for (int k = rank; k < n_tiles; k += kIdCluster) {
    const int t0 = k * kIdTile;
    const uint2 fl = load_flags(t0);
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < kIdPer; ++j) {
      const uint32_t f = flag_at(fl, j);
      mine += ((f >> 1) << 16) | (f & 1u);
    }
    uint32_t total;
    const uint32_t ex = block_excl_sum<kIdThreads>(mine, swarp, total);
    int cm = spre_m[k / kIdCluster] + (int)(ex >> 16);
    int ci = spre_i[k / kIdCluster] + (int)(ex & 0xffffu);
    int nq = 0;
#pragma unroll
    for (int j = 0; j < kIdPer; ++j) {
      const uint32_t f = flag_at(fl, j);
      cm += (int)(f >> 1);
      ci += (int)(f & 1u);
      const int t = t0 + tid * kIdPer + j;
      int ip = -1, q = -1;
      if (t < S) {
        const bool img = f & 1u;
        if (a.rule == 0) {
          if (img) ip = marker_mode ? cm - 1 : (ci - 1) / per_page;
          const bool pre = t <= last;
          q = pre ? cm - 1 : cm - 1 - (marker_mode ? pp : 0);
          if (pre && !a.page_scope_prefill) q = -1;
          if (q < 0) q = -1;
        } else if (img) {
          ip = cm > 0 ? cm - 1 : (ci - 1) / per_page;
        }
        nq += q >= 0;
      }
      spage[tid * kIdPer + j] = ip;
      sqp[tid * kIdPer + j] = q;
    }
    nq_cta += nq;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kIdPer; ++j) {
      const int off = j * kIdThreads + tid;
      const int t = t0 + off;
      if (t < S) {
        if (a.image_mask) a.image_mask[(int64_t)row * a.image_mask_stride + t] = sflag[off] & 1u;
        if (a.image_page) store_page(a.image_page, a.page_elem_bytes, (int64_t)row * a.image_page_stride + t, spage[off]);
        if (a.query_page) store_page(a.query_page, a.page_elem_bytes, (int64_t)row * a.query_page_stride + t, sqp[off]);
      }
    }
    if (blocks) {
      const int nb_tile = kIdTile / bs;
      for (int kb = warp; kb < nb_tile; kb += kIdThreads / 32) {
        const int gb = t0 / bs + kb;
        if (gb >= a.n_blocks) break;
        int lo = INT_MAX, hi = -1;
        bool has = false;
        for (int e = lane; e < bs; e += 32) {
          const int p = spage[kb * bs + e];
          if (p >= 0) {
            lo = min(lo, p);
            hi = max(hi, p);
          }
          has |= (sflag[kb * bs + e] & 1u) != 0;
        }
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        has = __any_sync(0xffffffffu, has);
        if (hi < 0) lo = -1;
        const int64_t o = (int64_t)row * a.n_blocks + gb;
        if (a.blk_bits) {
          for (int w = 0; w < words; ++w) {
            uint32_t m = 0;
            for (int e = lane; e < bs; e += 32) {
              const int p = spage[kb * bs + e];
              const int kk = p - lo;
              if (p >= 0 && (kk >> 5) == w) m |= 1u << (kk & 31);
            }
            m = __reduce_or_sync(0xffffffffu, m);
            if (lane == 0) a.blk_bits[o * words + w] = m;
          }
        }
        if (lane == 0) {
          if (a.blk_lo) a.blk_lo[o] = lo;
          if (a.blk_hi) a.blk_hi[o] = hi;
          if (a.blk_has_image) a.blk_has_image[o] = has;
        }
      }
    }
    __syncthreads();
  }
  // blocks past the last tile
  if (blocks && rank == 0) {
    const int first = n_tiles * (kIdTile / bs);
    for (int gb = first + tid; gb < a.n_blocks; gb += kIdThreads) {
      const int64_t o = (int64_t)row * a.n_blocks + gb;
      if (a.blk_lo) a.blk_lo[o] = -1;
      if (a.blk_hi) a.blk_hi[o] = -1;
      if (a.blk_has_image) a.blk_has_image[o] = 0;
      if (a.blk_bits)
        for (int w = 0; w < words; ++w) a.blk_bits[o * words + w] = 0;
    }
  }
  if (a.n_query) {
    nq_cta = __reduce_add_sync(0xffffffffu, nq_cta);
    if (lane == 0 && nq_cta) atomicAdd(a.n_query + row, nq_cta);
  }
}

// ---------------------------------------------------------------------------
// page_state_kernel: one CTA per request, tiles of kStTile tokens scanned in
// order with the running marker count, image run and pp carried across
// tiles.  Restates page_state.py:217-313 and decode_meta_triton.py:38-87, and
// page_state.py:315-328 for the bounds of the blocks it wrote.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t warp_min64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, o));
  return v;
}

__device__ __forceinline__ int64_t warp_max64(int64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, o));
  return v;
}

constexpr int kStThreads = 256;
constexpr int kStPer = 8;
constexpr int kStTile = kStThreads * kStPer;   // 2048 tokens

__device__ __forceinline__ int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

__global__ void __launch_bounds__(kStThreads) page_state_kernel(DashPageStateArgs a) {
  __shared__ __align__(16) uint8_t sflag[kStTile];
  __shared__ uint32_t swarp[32];
  __shared__ int smax[32];
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qs = a.q_start ? a.q_start[r] : (int64_t)r;
  const int64_t qe = a.q_start ? a.q_start[r + 1] : (int64_t)r + 1;
  const int64_t sp = a.start_pos ? a.start_pos[r] : (int64_t)a.seq_lens[r] - 1;
  const int bs = a.block_size;
  const int64_t ns = a.num_slots;
  const int32_t* bt = a.block_table + (int64_t)r * a.bt_stride;

  // carry-in from the slot of position sp - 1
  int prev_m = 0, prev_i = 0, prev_pp = 0;
  if (sp - 1 >= 0) {
    const int64_t p = sp - 1;
    const int64_t blk = min(p / bs, (int64_t)a.bt_width - 1);
    const int64_t slot = clamp64((int64_t)bt[blk] * bs + p % bs, 0, ns - 1);
    prev_m = a.slot_marker_cum[slot];
    prev_i = a.slot_img_run[slot];
    prev_pp = a.slot_prompt_pages[slot];
  }
  const int64_t gen0 = a.gen_start ? a.gen_start[r] : INT64_MAX;

  int cm_carry = prev_m, ci_carry = prev_i, x_carry = 0;
  for (int64_t t0 = qs; t0 < qe; t0 += kStTile) {
#pragma unroll
    for (int j = 0; j < kStPer; ++j) {
      const int off = j * kStThreads + tid;
      const int64_t t = t0 + off;
      uint32_t f = 0;
      if (t < qe)
        f = token_flags(__ldg(a.input_ids + t), a.image_token_id, a.mm_pad_shift, a.has_page_token,
                        a.page_token_id);
      sflag[off] = (uint8_t)f;
    }
    __syncthreads();
    const uint2 fl = *reinterpret_cast<const uint2*>(sflag + tid * kStPer);
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < kStPer; ++j) {
      const uint32_t f = flag_at(fl, j);
      mine += ((f >> 1) << 16) | (f & 1u);
    }
    uint32_t total;
    const uint32_t ex = block_excl_sum<kStThreads>(mine, swarp, total);
    // x = marker count at image tokens (0 elsewhere); pp is its running max
    int cm = cm_carry + (int)(ex >> 16), ci = ci_carry + (int)(ex & 0xffffu);
    int xmax = 0;
    {
      int c = cm;
#pragma unroll
      for (int j = 0; j < kStPer; ++j) {
        const uint32_t f = flag_at(fl, j);
        c += (int)(f >> 1);
        if (f & 1u) xmax = max(xmax, c);
      }
    }
    int xtot;
    const int xex = block_excl_max<kStThreads>(xmax, smax, xtot);
    int run_x = max(x_carry, xex);
#pragma unroll
    for (int j = 0; j < kStPer; ++j) {
      const uint32_t f = flag_at(fl, j);
      const int64_t t = t0 + tid * kStPer + j;
      cm += (int)(f >> 1);
      ci += (int)(f & 1u);
      const bool img = f & 1u;
      if (img) run_x = max(run_x, cm);
      if (t < qe) {
        const int ip = img ? (cm > 0 ? cm - 1 : (ci - 1) / a.per_page) : -1;
        const int pp = max(run_x, prev_pp);
        const bool gen = t < a.num_decode_tokens || sp + (t - qs) >= gen0;
        const int resp = cm - 1 - pp;
        const int text = gen ? (resp >= 0 ? resp : -1) : (cm > pp ? cm - 1 : -1);
        a.q_page[t] = img ? ip : text;
        const int64_t slot = clamp64(a.slot_mapping[t], 0, ns - 1);
        a.slot_img_page[slot] = ip;
        a.slot_marker_cum[slot] = cm;
        a.slot_img_run[slot] = ci;
        a.slot_prompt_pages[slot] = pp;
      }
    }
    cm_carry += (int)(total >> 16);
    ci_carry += (int)(total & 0xffffu);
    x_carry = max(x_carry, xtot);
    __syncthreads();
  }

  // slots past the last token of the request's last block lose their page
  const int64_t end = sp + (qe - qs);
  const int64_t last_blk = clamp64(max(end - 1, (int64_t)0) / bs, 0, (int64_t)a.bt_width - 1);
  const int rem = (int)(end % bs);
  if (rem > 0) {
    const int64_t phys = bt[last_blk];
    for (int o = rem + tid; o < bs; o += kStThreads)
      a.slot_img_page[clamp64(phys * bs + o, 0, ns - 1)] = -1;
  }
  if (!a.blk_lo) return;
  __syncthreads();
  // page bounds of the physical blocks this request wrote
  const int64_t n_blocks = ns / bs;
  const int64_t b_first =
      min(clamp64(max(sp, (int64_t)0) / bs, 0, (int64_t)a.bt_width - 1), last_blk);
  for (int64_t lb = b_first + warp; lb <= last_blk; lb += kStThreads / 32) {
    const int64_t phys = bt[lb];
    if (phys < 0 || phys >= n_blocks) continue;
    int lo = INT_MAX, hi = -1;
    for (int e = lane; e < bs; e += 32) {
      const int p = a.slot_img_page[phys * bs + e];
      hi = max(hi, p);
      if (p >= 0) lo = min(lo, p);
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lane == 0) {
      a.blk_lo[phys] = hi >= 0 ? lo : -1;
      a.blk_hi[phys] = hi;
    }
  }
}

// ---------------------------------------------------------------------------
// page_allow_kernel: one warp per row; a first pass over the blocks finds
// whether the row has a match (fallback), the second writes the row.
// ---------------------------------------------------------------------------
constexpr int kAllowWarps = 8;

__global__ void __launch_bounds__(kAllowWarps * 32) page_allow_kernel(DashPageAllowArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kAllowWarps + warp;
  if (r >= a.rows) return;
  const int64_t s = a.row_seq ? (int64_t)a.row_seq[r] : r / a.rows_per_seq;
  const int64_t qi = a.q_pos ? s * a.q_stride + clamp64(a.q_pos[r], 0, (int64_t)a.q_len - 1) : r;
  const int64_t q64 = load_page(a.q_page, a.q_elem_bytes, qi);
  const int q = q64 < 0 ? -1 : (int)min(q64, (int64_t)INT_MAX);
  const int64_t live = a.seq_lens ? (int64_t)a.seq_lens[s] : INT64_MAX;
  auto same = [&](int b) -> bool {
    if (q < 0 || b >= a.desc_width || (int64_t)b * a.block_size >= live) return false;
    int64_t i;
    if (a.block_table) {
      i = clamp64(a.block_table[s * a.bt_stride + b], 0, a.num_desc - 1);
    } else {
      i = s * a.desc_seq_rows + b;
      if (i >= a.num_desc) return false;
    }
    return page_desc_holds(a.page_lo, a.page_hi, a.page_bits, a.page_bits_words, i, q);
  };
  bool open = false;
  if (a.fallback) {
    bool any = false;
    for (int b0 = 0; b0 < a.width && !any; b0 += 32) {
      const int b = b0 + lane;
      any = __any_sync(0xffffffffu, b < a.width && same(b));
    }
    open = !any;
  }
  uint8_t* out = a.out + r * a.out_stride;
  for (int b = lane; b < a.width; b += 32) out[b] = open ? 1 : (uint8_t)same(b);
}

// one warp per (row, block): lo / hi / page bits of the block's page ids
__global__ void __launch_bounds__(256) page_blocks_kernel(DashPageBlocksArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * 8 + warp;
  if (g >= (int64_t)a.rows * a.n_blocks) return;
  const int64_t s = g / a.n_blocks;
  const int b = (int)(g - s * a.n_blocks);
  const int bs = a.block_size;
  const int64_t t0 = (int64_t)b * bs;
  const int64_t base = s * a.stride;
  int64_t lo = INT64_MAX, hi = -1;
  for (int e = lane; e < bs; e += 32) {
    const int64_t t = t0 + e;
    if (t < a.len) {
      const int64_t p = load_page(a.pages, a.elem_bytes, base + t);
      if (p >= 0) {
        lo = min(lo, p);
        hi = max(hi, p);
      }
    }
  }
  lo = warp_min64(lo);
  hi = warp_max64(hi);
  if (hi < 0) lo = -1;
  if (a.bits) {
    const int words = bs >= 32 ? bs / 32 : 1;
    for (int w = 0; w < words; ++w) {
      uint32_t m = 0;
      for (int e = lane; e < bs; e += 32) {
        const int64_t t = t0 + e;
        if (t < a.len) {
          const int64_t p = load_page(a.pages, a.elem_bytes, base + t);
          const int64_t kk = p - lo;
          if (p >= 0 && (kk >> 5) == w) m |= 1u << (kk & 31);
        }
      }
      m = __reduce_or_sync(0xffffffffu, m);
      if (lane == 0) a.bits[g * words + w] = m;
    }
  }
  if (lane == 0) {
    a.lo[g] = (int32_t)min(lo, (int64_t)INT_MAX);
    a.hi[g] = (int32_t)min(hi, (int64_t)INT_MAX);
  }
}

__global__ void page_decode_kernel(DashPageDecodeArgs a) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= a.n_seq) return;
  int m = a.marker_count[s];
  if (a.has_page_token && a.last_ids[(int64_t)s * a.ids_stride] == a.page_token_id) ++m;
  a.marker_count[s] = m;
  const int q = m - 1 - a.prompt_pages[s];
  a.q_page[s] = q >= 0 ? q : -1;
}

// one warp per (row, block)
__global__ void __launch_bounds__(256) block_any_kernel(DashBlockAnyArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * 8 + warp;
  if (g >= (int64_t)a.rows * a.n_blocks) return;
  const int64_t s = g / a.n_blocks;
  const int b = (int)(g - s * a.n_blocks);
  const uint8_t* m = a.mask + s * a.mask_stride;
  bool any = false;
  const int64_t t0 = (int64_t)b * a.block_size;
  for (int e = lane; e < a.block_size; e += 32) {
    const int64_t t = t0 + e;
    any |= t < a.len && m[t] != 0;
  }
  any = __any_sync(0xffffffffu, any);
  if (lane == 0) a.out[s * a.out_stride + b] = any;
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
int launch_page_ids(const DashPageIdsArgs& a, cudaStream_t st) {
  if (a.n_seq == 0) return DASH_OK;
  const int n_tiles = (a.key_length + kIdTile - 1) / kIdTile;
  if (n_tiles > kIdCluster * kIdMaxTilesPerCta)
    return set_error(DASH_ERR_UNSUPPORTED, "key_length %d > %d", a.key_length,
                     kIdCluster * kIdMaxTilesPerCta * kIdTile);
  page_ids_kernel<<<(unsigned)a.n_seq * kIdCluster, kIdThreads, 0, st>>>(a);
  count_launch();
  return check_launch("page_ids_kernel");
}

int launch_page_state(const DashPageStateArgs& a, cudaStream_t st) {
  if (a.num_reqs == 0) return DASH_OK;
  page_state_kernel<<<(unsigned)a.num_reqs, kStThreads, 0, st>>>(a);
  count_launch();
  return check_launch("page_state_kernel");
}

int launch_page_allow(const DashPageAllowArgs& a, cudaStream_t st) {
  if (a.rows == 0 || a.width == 0) return DASH_OK;
  page_allow_kernel<<<(unsigned)((a.rows + kAllowWarps - 1) / kAllowWarps), kAllowWarps * 32, 0, st>>>(a);
  count_launch();
  return check_launch("page_allow_kernel");
}

int launch_page_blocks(const DashPageBlocksArgs& a, cudaStream_t st) {
  const int64_t n = (int64_t)a.rows * a.n_blocks;
  if (n == 0) return DASH_OK;
  page_blocks_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(a);
  count_launch();
  return check_launch("page_blocks_kernel");
}

int launch_page_decode(const DashPageDecodeArgs& a, cudaStream_t st) {
  if (a.n_seq == 0) return DASH_OK;
  page_decode_kernel<<<(unsigned)((a.n_seq + 127) / 128), 128, 0, st>>>(a);
  count_launch();
  return check_launch("page_decode_kernel");
}

int launch_block_any(const DashBlockAnyArgs& a, cudaStream_t st) {
  const int64_t n = (int64_t)a.rows * a.n_blocks;
  if (n == 0) return DASH_OK;
  block_any_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(a);
  count_launch();
  return check_launch("block_any_kernel");
}

}  // namespace dash
