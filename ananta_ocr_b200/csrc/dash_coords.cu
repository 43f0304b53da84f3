// dash_coords.cu -- Page2D rotary coordinates of a serving step and their
// cos/sin tables.
//
// Every token of an OCR prompt gets a (token, page) coordinate pair: the page
// is the token's prompt page (marker count) or, for text after the prompt
// pages and for generated tokens, its response page; the token coordinate is
// the token's rank inside its (request, page) bucket, counted across steps.
// The running state of a request (marker count, prompt pages, per-page token
// counts) lives in a state row; rows are matched to requests by a key (the
// request's first physical KV block) and reused least-recently-used.
//
//   coord_rows_kernel   one warp: match each request's key to a live row or
//                       take a free / least recently used one (ties: lowest
//                       row), reset rows that are new or restart at position 0
//   page_coord_kernel   one warp per request: 32 tokens at a time in order,
//                       marker count (warp scan), prompt pages (running max),
//                       page, and the rank in the page bucket (peers of equal
//                       page by __match_any_sync; the group leader advances the
//                       row's counter)
//   cos_sin_2d_kernel   one warp per token: angles t * inv_tok[j] / p * inv_page[j]
//                       (p = page mod page_mod), duplicated halves, cos/sin
//
// Semantics: WHL page2d_rope.py:327-620 (PageCoordState: _rows, step),
// decode_meta_triton.py:89-104 (decode branch) and :166-209 / :354-389
// (cos_sin_2d_fused), page2d_rope.py:109-127 (PageRope2D.cos_sin).  Not
// reproduced: the speculative-decoding rewind (_rewind_rejected/_snapshot),
// which only acts when a step re-submits positions a previous step already
// committed.
#include <cuda_bf16.h>
#include <climits>
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32) coord_rows_kernel(DashPageCoordArgs a) {
  const int lane = threadIdx.x;
  const int M = a.max_rows;
  // this step's stamp
  int64_t step = 0;
  if (lane == 0) step = ++a.step[0];
  step = __shfl_sync(0xffffffffu, (long long)step, 0);
  // pass 1: requests whose key is live keep their row (stamped now); the
  // first request of a repeated key decides for the later ones
  for (int r = 0; r < a.num_reqs; ++r) {
    const int64_t key = a.row_key[r];
    int found = INT_MAX;
    for (int m0 = 0; m0 < M; m0 += 32) {
      const int m = m0 + lane;
      const bool hit = m < M && a.state_key[m] == key;
      const uint32_t b = __ballot_sync(0xffffffffu, hit);
      if (b) { found = m0 + __ffs(b) - 1; break; }
    }
    if (lane == 0) a.rows[r] = found == INT_MAX ? -1 : found;
    if (lane == 0 && found != INT_MAX) a.state_stamp[found] = step;
    __syncwarp();
  }
  // pass 2: the other requests take free rows first, then the least recently
  // stamped (ties to the lowest row), in request order
  for (int r = 0; r < a.num_reqs; ++r) {
    const int64_t key = a.row_key[r];
    int row = a.rows[r];
    bool reset = row >= 0 && a.start_pos[r] <= 0;
    if (row < 0) {
      // a repeated key of an earlier request of this step shares its row
      int dup = -1;
      for (int q0 = 0; q0 < r; q0 += 32) {
        const int q = q0 + lane;
        const bool same = q < r && a.row_key[q] == key;
        const uint32_t b = __ballot_sync(0xffffffffu, same);
        if (b) { dup = q0 + __ffs(b) - 1; break; }
      }
      if (dup >= 0) {
        row = a.rows[dup];
      } else {
        // priority: free rows (-1), else the stamp; the lowest row on ties
        long long best = LLONG_MAX;
        int best_row = INT_MAX;
        for (int m = lane; m < M; m += 32) {
          const long long pr = a.state_key[m] >= 0 ? (long long)a.state_stamp[m] : -1LL;
          if (pr < best || (pr == best && m < best_row)) { best = pr; best_row = m; }
        }
        for (int o = 16; o > 0; o >>= 1) {
          const long long ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int orw = __shfl_xor_sync(0xffffffffu, best_row, o);
          if (ob < best || (ob == best && orw < best_row)) { best = ob; best_row = orw; }
        }
        row = best_row;
        reset = true;
        if (lane == 0) { a.state_key[row] = key; a.state_stamp[row] = step; }
      }
    }
    if (reset) {
      if (lane == 0) { a.c_marker[row] = 0; a.c_pp[row] = 0; }
      for (int c = lane; c < a.max_pages; c += 32) a.cnt[(int64_t)row * a.max_pages + c] = 0;
    }
    if (lane == 0) a.rows[r] = row;
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32) page_coord_kernel(DashPageCoordArgs a) {
  const int r = blockIdx.x, lane = threadIdx.x;
  const int row = a.rows[r];
  const int64_t qs = a.q_start ? a.q_start[r] : (int64_t)r;
  const int64_t qe = a.q_start ? a.q_start[r + 1] : (int64_t)r + 1;
  const int64_t sp = a.start_pos[r];
  const int64_t g0 = a.gen_start ? a.gen_start[r] : INT64_MAX;
  int32_t* cnt = a.cnt + (int64_t)row * a.max_pages;
  int cm = a.c_marker[row], pp = a.c_pp[row];
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t t0 = qs; t0 < qe; t0 += 32) {
    const int64_t t = t0 + lane;
    const bool valid = t < qe;
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
    int64_t id = valid ? a.input_ids[t] : -1;
    const bool img = valid && (id == a.image_token_id || (a.mm_pad_shift > 0 && id >= a.mm_pad_shift));
    const bool mark = valid && a.has_page_token && id == a.page_token_id;
    // marker count: carry + inclusive count of markers up to this token
    const int mc = cm + __popc(__ballot_sync(0xffffffffu, mark) & (lt | (1u << lane)));
    // prompt pages: running max of the marker count at image tokens
    int x = img ? mc : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = max(x, y);
    }
    const int ppt = max(pp, x);
    const bool gen = t < a.num_decode_tokens || sp + (t - qs) >= g0;
    const bool in_prefill = !gen && (img || mc > ppt);
    const int resp = min(max(mc - ppt, 0), ppt);
    const int page = min(max(in_prefill ? mc : resp, 0), a.max_pages - 1);
    // rank inside the page bucket: earlier peers of this chunk + the counter
    const uint32_t peers = __match_any_sync(0xffffffffu, valid ? page : -1) & vmask;
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (valid && lane == leader) {
      base = cnt[page];
      cnt[page] = base + __popc(peers);
    }
    base = __shfl_sync(0xffffffffu, base, valid ? leader : lane);
    if (valid) {
      a.tok_pos[t] = (int64_t)base + __popc(peers & lt);
      a.page_pos[t] = page;
    }
    __syncwarp();
    const int last = 31 - __clz(vmask);
    cm = __shfl_sync(0xffffffffu, mc, last);
    pp = __shfl_sync(0xffffffffu, ppt, last);
  }
  if (lane == 0) { a.c_marker[row] = cm; a.c_pp[row] = pp; }
}

// ---------------------------------------------------------------------------
template <bool BF16>
__global__ void __launch_bounds__(128) cos_sin_2d_kernel(DashCosSin2DArgs a) {
  const int64_t t = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= a.num_tokens) return;
  const int lane = threadIdx.x & 31;
  const int half = a.dim / 2;
  const float tf = (float)a.tok_pos[t];
  int64_t p = a.page_pos[t];
  if (a.page_mod > 0) {
    p %= a.page_mod;
    if (p < 0) p += a.page_mod;
  }
  const float pf = (float)p;
  for (int off = lane; off < a.dim; off += 32) {
    const int j = off < half ? off : off - half;
    const float ang = j < a.n_tok ? tf * a.inv_tok[j] : pf * a.inv_page[j - a.n_tok];
    float s, c;
    sincosf(ang, &s, &c);
    if (BF16) {
      reinterpret_cast<__nv_bfloat16*>(a.cos)[t * a.stride + off] = __float2bfloat16_rn(c);
      reinterpret_cast<__nv_bfloat16*>(a.sin)[t * a.stride + off] = __float2bfloat16_rn(s);
    } else {
      reinterpret_cast<float*>(a.cos)[t * a.stride + off] = c;
      reinterpret_cast<float*>(a.sin)[t * a.stride + off] = s;
    }
  }
}

int launch_page_coords(const DashPageCoordArgs& a, cudaStream_t st) {
  coord_rows_kernel<<<1, 32, 0, st>>>(a);
  count_launch();
  int rc = check_launch("coord_rows_kernel");
  if (rc) return rc;
  page_coord_kernel<<<a.num_reqs, 32, 0, st>>>(a);
  count_launch();
  return check_launch("page_coord_kernel");
}

int launch_cos_sin_2d(const DashCosSin2DArgs& a, cudaStream_t st) {
  if (a.num_tokens == 0) return DASH_OK;
  const unsigned grid = (unsigned)((a.num_tokens + 3) / 4);
  if (a.out_bf16) cos_sin_2d_kernel<true><<<grid, 128, 0, st>>>(a);
  else cos_sin_2d_kernel<false><<<grid, 128, 0, st>>>(a);
  count_launch();
  return check_launch("cos_sin_2d_kernel");
}

}  // namespace dash
