/*
 * dash_b200.h -- C ABI of the B200 (sm_100a) DASH block-sparse attention library
 * (libdash_b200.so).
 *
 * DASH is ANANTA_OCR's SR-SWA attention: every query token attends to a
 * sliding window of `local_window` tokens plus up to K remote key blocks picked
 * by a single-head 1.5-entmax router, each remote block carrying an additive
 * log-prior bias.  The library implements the forward path:
 *
 *   dash_kbar_pool      stage-0 head_cls pooling of index keys into one
 *                       summary key per block (k-bar)
 *   dash_route          block scores + 1.5-entmax + top-K selection + bias,
 *                       emitting compact ascending int32 block lists
 *   dash_block_max      indexer-mode stage-0 scores (block max of token scores)
 *   dash_prefill_attn   gather attention for many query tokens (tcgen05/TMEM)
 *   dash_decode_attn    gather attention for decode tokens over a block-paged
 *                       KV cache (split-KV with fused combine)
 *
 * Conventions
 *  - All pointers are DEVICE pointers unless stated; strides are in ELEMENTS.
 *  - Every entry point returns a DASH_* status; on failure dash_last_error()
 *    holds a message.  Kernels never trap: a bounds check that fails on the
 *    device records a DASH_DEV_* code in the optional DashDeviceError word
 *    (device memory, zero-initialised by the caller) and skips the access.
 *  - Work is enqueued on `stream` (a cudaStream_t); nothing synchronises.
 *  - The routing of a query token is shared by all attention heads (the
 *    reference router has one index head); `n_index_heads` > 1 selects the
 *    multi-index-head layout of sparse_gather_triton.py.
 */
#ifndef DASH_B200_H
#define DASH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DASH_OK 0
#define DASH_ERR_INVALID 1     /* malformed argument (shape, null pointer, alignment)  */
#define DASH_ERR_UNSUPPORTED 2 /* well formed but outside what the kernels implement   */
#define DASH_ERR_CUDA 3        /* a CUDA runtime or driver call failed                  */
#define DASH_ERR_WORKSPACE 4   /* workspace pointer missing or too small                */

#define DASH_DEV_TIMEOUT 1     /* a bounded wait inside a kernel ran out               */
#define DASH_DEV_BAD_BLOCK 2   /* routed block id outside [0, blocks of the sequence)   */
#define DASH_DEV_BAD_PAGE 3    /* block-table page id outside [0, num_pages)            */

#define DASH_DTYPE_F32 0
#define DASH_DTYPE_BF16 1
#define DASH_DTYPE_F16 2

typedef void* dash_stream_t; /* cudaStream_t */

/* Device-side error word (allocate 16 bytes of device memory, zero it). */
typedef struct {
  int32_t code;  /* first DASH_DEV_* code, 0 = none */
  int32_t where; /* kernel site id */
  int64_t info;  /* offending value */
} DashDeviceError;

/* Sequences of a batch.  Query row i of sequence s sits at position
 * pos0[s] + i and attends keys [0, pos]; the sequence holds kv_len[s] tokens.
 *   q_start  [n_seq+1] first query row of each sequence in a packed (varlen)
 *            row layout (cu_seqlens_q); NULL: sequence s owns rows
 *            [s*q_len_fixed, (s+1)*q_len_fixed) and strides use stride_seq.
 *   pos0     [n_seq] position of the first query row; NULL: kv_len - q_len
 *            (the queries are the last tokens: prefill without prefix, decode).
 *   kv_len   [n_seq] live tokens (seq_lens); NULL: kv_len_fixed for all.
 *   q_len_fixed  rows per sequence when q_start == NULL; the TOTAL number of
 *            query rows (q_start[n_seq]) when q_start != NULL.
 *   max_q_len    upper bound of any sequence's query rows.
 *   kv_len_fixed also gives the allocated token extent of contiguous K/V.   */
typedef struct {
  int32_t n_seq;
  int32_t q_len_fixed;
  int32_t kv_len_fixed;
  int32_t max_q_len;
  const int32_t* q_start;
  const int32_t* pos0;
  const int32_t* kv_len;
} DashSeqs;

/* Key/value storage.
 *  contiguous (block_table == NULL): element (seq s, token t, head h, dim c) at
 *      base + s*stride_seq + t*stride_tok + h*stride_head + c
 *  block-paged (block_table != NULL): token t of sequence s lives in page
 *      p = block_table[s*bt_stride + t/page_size] at offset t%page_size:
 *      base + p*stride_seq + (t%page_size)*stride_tok + h*stride_head + c
 *  (page_size == block_size: one sparse block per page.)                     */
typedef struct {
  const void* k;
  const void* v;
  int32_t dtype; /* DASH_DTYPE_BF16 or DASH_DTYPE_F16 */
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t pad0;
  int64_t stride_seq, stride_tok, stride_head;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t num_pages;
} DashKV;

/* Routed blocks per query row: idx[row*row_stride + ih*ihead_stride + j],
 * j < K, -1 = unused slot; bias likewise (NULL = no bias).  Query head hq
 * reads index head  hq / (n_heads / n_index_heads).  Lists need not be sorted
 * or duplicate-free; ids outside the sequence's causal range are ignored.   */
typedef struct {
  const int32_t* idx;
  const float* bias;
  int64_t row_stride;
  int64_t ihead_stride;
  int32_t K;
  int32_t n_index_heads;
} DashRoutes;

/* Queries and outputs: element (seq s, query row i, head h, dim c) at
 *   q + (q_start ? (q_start[s]+i)*stride_tok : s*stride_seq + i*stride_tok)
 *     + h*stride_head + c                                                    */
typedef struct {
  const void* q;
  void* out;
  int64_t q_stride_seq, q_stride_tok, q_stride_head;
  int64_t o_stride_seq, o_stride_tok, o_stride_head;
  int32_t n_heads;
  int32_t pad0;
  float* lse;                 /* optional natural-log LSE, same (s, i, h) addressing */
  int64_t lse_stride_seq, lse_stride_tok, lse_stride_head;
} DashQO;

/* ---------------------------------------------------------------------- */
/* Stage-0 head_cls pooling (k-bar).
 * Replaces: dash_attention.py:863-888 (_block_scores_headcls pooling),
 *           modeling_deepseekv2.py:362-379 (_block_scores_infer),
 *           WHL sglang/srt/layers/attention/unlimited_dash_ops/route_triton.py:36-72
 *           (_kbar_page_kernel) and :707-726 (kbar_refresh_tail_triton).
 * contiguous (pages == NULL): summary of block b of sequence s (tokens
 *   [b*block_size, min(seq_len, (b+1)*block_size))) -> kbar row s*kbar_seq_rows+b.
 * paged: for each plan entry i with ntok[i] > 0, the first ntok[i] tokens of
 *   page pages[i] -> kbar row pages[i].                                    */
typedef struct {
  const void* keys;
  int32_t dtype;       /* DASH_DTYPE_F32 or DASH_DTYPE_BF16 */
  int32_t d;           /* index dim, <= 256 */
  int32_t block_size;  /* <= 256 */
  int32_t n_seq;
  int32_t seq_len;
  int32_t n_plan;
  int64_t tok_stride;  /* elements between consecutive tokens */
  int64_t seq_stride;  /* contiguous: elements between sequences */
  int64_t page_stride; /* paged: elements between pages */
  int64_t kbar_seq_rows;
  const float* head_cls; /* [d] or NULL (= zeros: block mean) */
  const int64_t* pages;
  const int32_t* ntok;
  float* kbar;
  int64_t kbar_row_stride;
} DashKbarArgs;
int dash_kbar_pool(const DashKbarArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Routing: scores, candidates, 1.5-entmax prior, top-K selection, bias.
 * Replaces: modeling_deepseekv2.py:351-388 (_block_scores_infer scoring) +
 *           modeling_deepseekv2.py:309-333 (_infer_route_select),
 *           WHL dash_router.py:131-174 (DashRouterMath.route_and_select),
 *           WHL route_triton.py:624-678 (route_prefill_triton) and
 *           :730-847 (route_decode_triton).
 * Row r is query row r of `seqs` (same packing as the attention).  Block b
 * of row r is a candidate iff b <= pos/block_size - local_blocks and
 * b*block_size < kv_len (and cand[...] != 0 when a mask is given, with the
 * per-row fallback to all remote blocks when the mask leaves none).
 * Output: out_idx[r*out_stride + j], j < out_width: selected ids ascending,
 * -1 tail; out_bias alongside (0 on unused slots).  Selection = top-K by
 * score among candidates, ties to the lowest block id; the entmax prior is
 * evaluated over the top-`topm` entries (topm <= 0: all blocks).            */
typedef struct {
  DashSeqs seqs;
  const float* idx_q;     /* [rows, d] router queries */
  int64_t q_row_stride;
  const float* kbar;      /* k-bar rows */
  int64_t kbar_row_stride;
  const int32_t* block_table; /* paged k-bar cache: row = block_table[s*bt_stride+b] */
  int64_t bt_stride;
  int64_t kbar_seq_rows;  /* contiguous k-bar: row = s*kbar_seq_rows + b */
  int64_t num_kbar_rows;  /* bounds check of k-bar rows */
  int32_t width;          /* blocks scored per row (max_block) */
  int32_t d;              /* == 128 */
  const float* scores_in; /* optional [rows, width] precomputed scores (skips scoring) */
  int64_t scores_in_stride;
  float* scores_out;      /* optional [rows, width] */
  int64_t scores_out_stride;
  const uint8_t* cand;    /* optional candidate mask, [rows or n_seq, width] */
  int64_t cand_row_stride;
  int32_t cand_per_seq;   /* 1: one mask row per sequence */
  int32_t block_size;
  int32_t local_blocks;
  int32_t topm;
  int32_t K;
  int32_t out_width;      /* >= K */
  float idx_scale;        /* scaling_factor / sqrt(index_dim) */
  float prior_floor;
  float inv_sigma;
  int32_t pad0;
  int32_t* out_idx;
  float* out_bias;
  int64_t out_stride;
  int32_t* out_count;     /* optional valid slots per row */
  DashDeviceError* device_error;
  /* Page-aware candidates (optional; when page_q is set, cand is ignored).
   * Block b of row r is a candidate iff it is remote and the image-page set
   * of its descriptor i holds q = page_q[r]: q >= 0, page_lo[i] >= 0,
   * page_lo[i] <= q <= page_hi[i] and, when page_bits is given, bit
   * (q - page_lo[i]) of page_bits[i*page_bits_words ...] is set.
   * i = block_table[s*bt_stride + b] when block_table is set (descriptors of
   * physical blocks), else s*page_seq_rows + b.  Rows left without a
   * candidate fall back to all remote blocks.  Replaces the `image_allow`
   * input of WHL route_triton.py:159-167 built by page_state.py:330-371 /
   * decode_meta_triton.py:107-163, and the `block_cand` of
   * modeling_deepseekv2.py:310-319 built by _sparse_base_impl.py:2383-2484. */
  const int32_t* page_q;
  const int32_t* page_lo;
  const int32_t* page_hi;
  const uint32_t* page_bits;
  int64_t page_seq_rows;
  int64_t num_page_desc;   /* descriptors addressable (bounds check) */
  int32_t page_bits_words;
  int32_t pad1;
} DashRouteArgs;
int dash_route(const DashRouteArgs* args, dash_stream_t stream);

/* Decode routing with the k-bar tail refresh of the same step in one launch.
 * Replaces the pair WHL route_triton.py:707-726 (kbar_refresh_tail_triton)
 * then :730-847 (route_decode_triton), as called per decode step by
 * WHL unlimited_ocr_v2_backend.py.  `refresh` is a paged DashKbarArgs plan
 * (pages/ntok) writing the k-bar rows that `args` reads (NULL: dash_route).
 * The rows it refreshes must not be rows this launch scores: the tail pages
 * of a decode step lie in every row's local window when tail_pages <=
 * local_blocks.  Few-row decode launches with d == 128 and 16-byte aligned
 * keys run the refresh on the routing cluster's idle CTAs; any other form
 * runs the refresh, then the routing, as two launches.                    */
int dash_route_refresh(const DashRouteArgs* args, const DashKbarArgs* refresh, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Page-aware candidate domain (image pages of an OCR document).
 *
 * Token ids mark image placeholders (image_token_id, or any id >=
 * mm_pad_shift when mm_pad_shift > 0) and page starts (page_token_id when
 * has_page_token).  Per row, cum(t) = page markers at positions <= t and
 * run(t) = image tokens at positions <= t.
 *
 * dash_page_ids -- one pass over contiguous rows of token ids.
 * Replaces: _sparse_base_impl.py:2189-2260 (_build_page_aware_ids, rule 0),
 *           :2363-2381 (_build_flat_image_token_mask), :2177-2187
 *           (_build_image_block_allow_mask) and the prefill branch of
 *           modeling_anantaocr.py:468-481 (_uocr_dash_decode_allow, rule 1).
 *   rule 0: pp = cum at the row's last image token (0 without one); the row
 *           is in marker mode iff pp > 0; image page = marker mode ? cum - 1
 *           : (run - 1) / per_page; query page = cum - 1 at positions <= the
 *           last image token (-1 unless page_scope_prefill), cum - 1 - pp
 *           after it in marker mode, cum - 1 otherwise; negative -> -1.
 *   rule 1: image page = cum > 0 ? cum - 1 : (run - 1) / per_page (per
 *           token); query pages are not produced.
 * Image pages are -1 at non-image tokens.  Tokens at t >= ids_len read as id
 * -1.  Block outputs cover n_blocks blocks of block_size tokens per row
 * (tokens past key_length count as non-image): lo/hi = min/max image page >=
 * 0 in the block (-1 when none), bits = set of pages present (bit k: page
 * lo + k; exact for rule 0, where a block spans fewer than block_size
 * pages), has_image = any image token.  block_size: power of two in
 * [16, 256] (block outputs only).  Per-row outputs: prompt_pages = pp,
 * marker_count = cum at key_length - 1, n_image / n_query = image tokens /
 * tokens with a query page >= 0.  Every output pointer is optional.       */
typedef struct {
  const int64_t* token_ids;   /* [n_seq, ids_stride] */
  int64_t ids_stride;
  int32_t n_seq;
  int32_t ids_len;            /* columns present in token_ids */
  int32_t key_length;         /* tokens per row processed */
  int32_t per_page;           /* >= 1 */
  int64_t image_token_id;
  int64_t page_token_id;
  int64_t mm_pad_shift;       /* 0: off */
  int32_t has_page_token;
  int32_t rule;               /* 0 or 1 */
  int32_t page_scope_prefill;
  int32_t block_size;
  int32_t n_blocks;           /* blocks per row of the block outputs */
  int32_t page_elem_bytes;    /* 4 (int32) or 8 (int64) for image_page / query_page */
  uint8_t* image_mask;  int64_t image_mask_stride;   /* [n_seq, key_length] */
  void* image_page;     int64_t image_page_stride;   /* [n_seq, key_length] */
  void* query_page;     int64_t query_page_stride;   /* [n_seq, key_length] */
  int32_t* blk_lo;                                   /* [n_seq, n_blocks] */
  int32_t* blk_hi;
  uint32_t* blk_bits;                                /* [n_seq, n_blocks, max(1, block_size/32)] */
  uint8_t* blk_has_image;
  int32_t* prompt_pages;                             /* [n_seq] */
  int32_t* marker_count;
  int32_t* n_image;
  int32_t* n_query;
  DashDeviceError* device_error;
} DashPageIdsArgs;
int dash_page_ids(const DashPageIdsArgs* args, dash_stream_t stream);

/* dash_page_state_step -- per-slot page bookkeeping of a block-paged KV
 * cache for one serving step (a mixed batch of requests, tokens packed).
 * Replaces: page_state.py:217-313 (PageIsolationState.step) and the page
 * part of decode_meta_triton.py:18-87 (_decode_meta_kernel).
 * Request r owns tokens [q_start[r], q_start[r+1]) at positions
 * start_pos[r] + i (q_start NULL: request r owns token r; start_pos NULL:
 * start_pos[r] = seq_lens[r] - 1).  Carry-in (marker count, image run,
 * prompt pages) is read from the slot of position start_pos - 1.  Per token:
 * marker_cum, img_run, image page (rule 1 of dash_page_ids), pp = max(carry,
 * marker_cum at the latest image token of this step), query page = image
 * page at image tokens, else (generated token ? marker_cum - 1 - pp (-1 if
 * negative) : (marker_cum > pp ? marker_cum - 1 : -1)).  A token is
 * generated iff its index < num_decode_tokens, or its position >=
 * gen_start[r] (gen_start optional).  The four slot arrays are written at
 * slot_mapping (clamped to [0, num_slots)); then slots past the last token
 * in each request's last block get image page -1.  When blk_lo/blk_hi are
 * given, the image-page bounds of every physical block written in this step
 * are recomputed from the slot array (page_state.py:315-328).            */
typedef struct {
  const int64_t* input_ids;   /* [num_tokens] */
  const int64_t* q_start;     /* [num_reqs+1] or NULL */
  const int64_t* start_pos;   /* [num_reqs] or NULL */
  const int32_t* seq_lens;    /* [num_reqs], used when start_pos is NULL */
  const int64_t* gen_start;   /* [num_reqs] or NULL */
  const int32_t* block_table; int64_t bt_stride;
  const int64_t* slot_mapping;/* [num_tokens] */
  int64_t num_slots;
  int64_t image_token_id;
  int64_t page_token_id;
  int64_t mm_pad_shift;
  int32_t num_tokens;
  int32_t num_reqs;
  int32_t num_decode_tokens;
  int32_t bt_width;
  int32_t block_size;
  int32_t per_page;
  int32_t has_page_token;
  int32_t pad0;
  int32_t* slot_img_page;     /* [num_slots] state, in/out */
  int32_t* slot_marker_cum;
  int32_t* slot_img_run;
  int32_t* slot_prompt_pages;
  int32_t* q_page;            /* [num_tokens] out */
  int32_t* blk_lo;            /* [num_slots / block_size] or NULL */
  int32_t* blk_hi;
  DashDeviceError* device_error;
} DashPageStateArgs;
int dash_page_state_step(const DashPageStateArgs* args, dash_stream_t stream);

/* dash_page_allow -- dense per-row candidate mask out[r, b] (uint8), b <
 * width, from a query page per row and block page descriptors.
 * Replaces: page_state.py:330-371 (build_query_allow), decode_meta_triton.py
 * :107-163 (_decode_allow_kernel), _sparse_base_impl.py:2383-2402 +
 * :2457-2484 (_build_page_aware_image_block_mask + _build_kl_candidate_mask
 * fallback) and the decode branch of modeling_anantaocr.py:482-496.
 * Row r belongs to sequence s = row_seq ? row_seq[r] : r / rows_per_seq.
 * Block b < desc_width has descriptor i = block_table[s*bt_stride + b]
 * (clamped to [0, num_desc)) or s*desc_seq_rows + b; blocks >= desc_width
 * and (seq_lens given) blocks with b*block_size >= seq_lens[s] never match.
 * same = match as in dash_route's page mode; out = same, or 1 everywhere
 * when fallback != 0 and the row has no match.                             */
typedef struct {
  int32_t rows;
  int32_t width;
  uint8_t* out; int64_t out_stride;
  const void* q_page;         /* [rows], or [n_seq, q_stride] when q_pos is set */
  int32_t q_elem_bytes;       /* 4 (int32) or 8 (int64) */
  int32_t q_len;              /* q_pos set: query page of row r = q_page[s*q_stride +
                                 clamp(q_pos[r], 0, q_len - 1)] */
  const int64_t* q_pos;       /* [rows] or NULL */
  int64_t q_stride;
  const int32_t* row_seq;     /* [rows] or NULL */
  int32_t rows_per_seq;
  int32_t desc_width;
  const int32_t* page_lo;
  const int32_t* page_hi;
  const uint32_t* page_bits;  /* or NULL: range test only */
  int32_t page_bits_words;
  int32_t block_size;
  int64_t num_desc;
  const int32_t* block_table; int64_t bt_stride;
  int64_t desc_seq_rows;
  const int32_t* seq_lens;    /* or NULL */
  int32_t fallback;
  int32_t pad0;
} DashPageAllowArgs;
int dash_page_allow(const DashPageAllowArgs* args, dash_stream_t stream);

/* dash_page_blocks -- block page descriptors from image page ids (-1 = no
 * image page): for block b < n_blocks of row s, over tokens t < min(len,
 * (b+1)*block_size): lo/hi = min/max page >= 0 (-1 when none), bits = pages
 * present relative to lo (words = max(1, block_size/32); a page beyond
 * 32*words of lo sets no bit).
 * Replaces the per-block test of _sparse_base_impl.py:2390-2401 and
 * page_state.py:315-328 (block_page_bounds, via a [num_blocks, block_size]
 * view of the slot pages).                                                 */
typedef struct {
  const void* pages; int64_t stride;   /* [rows, stride] */
  int32_t elem_bytes;                  /* 4 or 8 */
  int32_t rows;
  int32_t len;
  int32_t block_size;
  int32_t n_blocks;
  int32_t pad0;
  int32_t* lo;                         /* [rows, n_blocks] */
  int32_t* hi;
  uint32_t* bits;                      /* [rows, n_blocks, words] or NULL */
} DashPageBlocksArgs;
int dash_page_blocks(const DashPageBlocksArgs* args, dash_stream_t stream);

/* dash_page_decode_query -- decode-step query page of the contiguous decoder.
 * Replaces: modeling_anantaocr.py:482-486 (_uocr_dash_decode_allow decode
 * branch): marker_count[s] += (last_ids[s*ids_stride] == page_token_id);
 * q_page[s] = marker_count[s] - 1 - prompt_pages[s], -1 when negative.     */
typedef struct {
  const int64_t* last_ids; int64_t ids_stride;
  int32_t n_seq;
  int32_t has_page_token;
  int64_t page_token_id;
  int32_t* marker_count;      /* in/out */
  const int32_t* prompt_pages;
  int32_t* q_page;            /* out */
} DashPageDecodeArgs;
int dash_page_decode_query(const DashPageDecodeArgs* args, dash_stream_t stream);

/* dash_block_any -- out[s, b] = any(mask[s, t]) over the tokens t <
 * min(len, (b+1)*block_size) of block b, b < n_blocks.
 * Replaces: _sparse_base_impl.py:2177-2187 (_build_image_block_allow_mask). */
typedef struct {
  const uint8_t* mask; int64_t mask_stride;
  int32_t rows;
  int32_t len;
  int32_t block_size;
  int32_t n_blocks;
  uint8_t* out; int64_t out_stride;
} DashBlockAnyArgs;
int dash_block_any(const DashBlockAnyArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Indexer stage-0 block scores (block max over remote keys).
 * Replaces: sparse_gather_triton.py:431-467 (triton_block_max_score, clamp=0,
 *           empty=-inf), modeling_deepseekv2.py:389-400 and
 *           dash_attention.py:801-835 (clamp=1, empty=-1e9).
 * out[b, c, blk] = max over keys j of block blk with seg[b,c] <= j <=
 * pos[b,c] - local_window and j < Sk of <q[b,c], k[b,j]> (clamped to +-1e4
 * when clamp != 0); `empty` when the block has no such key.                 */
typedef struct {
  const float* q; int64_t q_stride_b, q_stride_c;
  const float* k; int64_t k_stride_b, k_stride_j;
  const int32_t* pos; int64_t pos_stride_b, pos_stride_c;
  const int32_t* seg; int64_t seg_stride_b, seg_stride_c; /* NULL = 0 */
  int32_t B, C, Sk, d, block_size, nblk, local_window, clamp;
  float empty;
  int32_t pad0;
  float* out; int64_t out_stride_b, out_stride_c;
} DashBlockMaxArgs;
int dash_block_max(const DashBlockMaxArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Prefill gather attention (tcgen05 / TMEM / TMA).
 * Replaces: sparse_gather_e2e_triton.py:342-391 (triton_gather_attention_e2e,
 *           forward), sparse_gather_triton.py:343-392 (triton_gather_attention,
 *           forward; bias = NULL), WHL attend_triton.py:523-596
 *           (dash_sparse_attn).
 * Query token at position p, head h: logits over keys j <= p, j >= seg,
 *   local  (j > p - local_window): scale*<q,k_j>
 *   remote (block j/block_size routed for the token, j <= p - local_window):
 *          scale*<q,k_j> + bias of that slot
 * out = softmax(logits) @ V.  head_dim 128,
 * n_heads / n_kv_heads in {1,2,4,8,16}; block_size 32 (two blocks per 64-key
 * tile; paged: 32-token pages) or a multiple of 64 up to 256.  Workspace:
 * dash_prefill_workspace_size. */
typedef struct {
  DashSeqs seqs;
  DashKV kv;
  DashRoutes routes;
  DashQO qo;
  const int32_t* seg_start; /* optional per query row first attendable key (packing) */
  float scale;
  int32_t block_size;
  int32_t local_window;
  /* 0: automatic; 1: tile-major (each 128-row tile walks the union of its
   * rows' blocks); 2: routed part gathered by key block (block sizes 32, 64,
   * 128; 1, 2 or 4 query heads per kv head), merged with the window part.
   * Automatic is tile-major. */
  int32_t mode;
  void* workspace;
  size_t workspace_bytes;
  DashDeviceError* device_error;
  /* fused output gather (optional): n_peers device pointers (a device array)
   * to other ranks' copies of `out` (same strides, e.g. from dash_peer_import);
   * every output row is also stored there (posted stores, complete when the
   * grid completes).  The caller orders a cross-rank completion step after
   * the call on the same stream. */
  void* const* out_peers;
  int32_t n_peers;
  /* mode 2: scratch for the routed partials in MiB (0: 2048); the work runs
   * in chunks of sequences x query tiles x kv heads whose partials fit it */
  int32_t part_budget_mib;
} DashPrefillArgs;
size_t dash_prefill_workspace_size(const DashPrefillArgs* args);
int dash_prefill_attn(const DashPrefillArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Peer device memory for the fused output gather (no reference counterpart:
 * the reference runs on one GPU; BASELINE's multi-GPU split gathers the output
 * shards over NVLink).  A rank exports a device buffer as a CUDA IPC handle of
 * the allocation holding it plus the buffer's offset; another rank of the same
 * node imports it (the allocation is opened once per process) and gets a
 * device pointer it may pass as a DashPrefillArgs.out_peers entry.  Handles are
 * plain bytes and travel between processes through the host.  close releases
 * one import; the mapping goes when its last import is closed.              */
typedef struct {
  char handle[64];       /* cudaIpcMemHandle_t of the allocation */
  int64_t offset;        /* buffer start inside the allocation */
  int64_t alloc_bytes;   /* allocation size (bounds check on import) */
} DashPeerHandle;
int dash_peer_export(const void* ptr, DashPeerHandle* out);
int dash_peer_import(const DashPeerHandle* handle, void** ptr);
int dash_peer_close(void* ptr);

/* ---------------------------------------------------------------------- */
/* Serving-step plans, computed on the device in one launch (no host sync).
 * Replaces: WHL route_triton.py:576-601 (kbar_all_plan), :605-620
 *           (prefill_row2req), :682-703 (kbar_tail_plan).
 * pages/ntok (optional, [n_req * width]): request r owns entries
 *   [r*width, (r+1)*width); entry j names block
 *     mode 0 (blocks a prefill chunk wrote): b = context_lens[r]/block_size + j
 *     mode 1 (mutable tail, newest first):   b = max(last_r - j, 0),
 *            last_r = max(ceil(seq_lens[r]/block_size) - 1, 0)
 *   pages[e] = block_table[r, min(b, bt_width - 1)],
 *   ntok[e]  = clamp(seq_lens[r] - b*block_size, 0, block_size)
 *   (an entry with ntok 0 is skipped by dash_kbar_pool).
 * row2req (optional, [cu_seqlens_q[n_req]]): rows [cu[r], cu[r+1]) get r.   */
typedef struct {
  const int32_t* block_table; int64_t bt_stride;
  const int32_t* seq_lens;      /* [n_req] */
  const int32_t* context_lens;  /* [n_req], mode 0 */
  const int32_t* cu_seqlens_q;  /* [n_req + 1], for row2req */
  int32_t n_req, block_size, width, mode, bt_width, pad0;
  int64_t* pages;
  int32_t* ntok;
  int32_t* row2req;
} DashServingPlanArgs;
int dash_serving_plan(const DashServingPlanArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Page2D rotary coordinates of a serving step (two launches).
 * Replaces: WHL page2d_rope.py:327-620 (PageCoordState._rows / step) and the
 *           coordinate part of decode_meta_triton.py:89-104 (decode_meta_fused).
 * Request r owns tokens [q_start[r], q_start[r+1]) (q_start NULL: token r),
 * the first at position start_pos[r].  Its state row is the live row whose
 * state_key equals row_key[r], else a free row (state_key -1) or the least
 * recently stamped one (ties: lowest row), which is reset; a matched row is
 * reset too when start_pos[r] <= 0.  Per token, in order: marker count
 * mc = carry + markers so far; prompt pages pp = max(carry, mc at image tokens
 * so far); generated iff flat index < num_decode_tokens or position >=
 * gen_start[r]; page = clamp(!generated && (image || mc > pp) ? mc :
 * min(max(mc - pp, 0), pp), 0, max_pages - 1); tok = the row's count of that
 * page, then the count grows by one.  The row keeps mc, pp and the counts.
 * State arrays are device memory the caller keeps across steps (state_key
 * initialised to -1, step to 0); rows is scratch [num_reqs].
 * No speculative-decoding rewind.                                          */
typedef struct {
  const int64_t* input_ids;    /* [num_tokens] */
  const int64_t* q_start;      /* [num_reqs + 1] or NULL */
  const int64_t* start_pos;    /* [num_reqs] */
  const int64_t* gen_start;    /* [num_reqs] or NULL */
  const int64_t* row_key;      /* [num_reqs], e.g. the first physical block */
  int64_t image_token_id, page_token_id, mm_pad_shift;
  int32_t num_tokens, num_reqs, num_decode_tokens, has_page_token, max_rows, max_pages;
  int64_t* state_key;          /* [max_rows] */
  int64_t* state_stamp;        /* [max_rows] */
  int64_t* step;               /* [1] */
  int32_t* c_marker;           /* [max_rows] */
  int32_t* c_pp;               /* [max_rows] */
  int32_t* cnt;                /* [max_rows, max_pages] */
  int32_t* rows;               /* [num_reqs] scratch */
  int64_t* tok_pos;            /* [num_tokens] out */
  int64_t* page_pos;           /* [num_tokens] out */
} DashPageCoordArgs;
int dash_page_coords(const DashPageCoordArgs* args, dash_stream_t stream);

/* Page2D cos/sin table: row t, column c (j = c mod dim/2):
 *   angle = j < n_tok ? tok_pos[t] * inv_tok[j] : (page_pos[t] mod page_mod) * inv_page[j - n_tok]
 * (fp32; page_mod 0 = no fold), cos/sin stored as fp32 or bf16 (round to
 * nearest) with row stride `stride` elements.
 * Replaces: WHL decode_meta_triton.py:166-209, :354-389 (cos_sin_2d_fused) and
 *           page2d_rope.py:109-127 (PageRope2D.cos_sin).                    */
typedef struct {
  const int64_t* tok_pos;
  const int64_t* page_pos;
  const float* inv_tok;   /* [n_tok] */
  const float* inv_page;  /* [dim/2 - n_tok] */
  void* cos;
  void* sin;
  int64_t stride;
  int64_t page_mod;
  int32_t num_tokens, dim, n_tok, out_bf16;
} DashCosSin2DArgs;
int dash_cos_sin_2d(const DashCosSin2DArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Decode gather attention over a block-paged (or contiguous) KV cache.
 * Replaces: WHL attend_triton.py:600-715 (dash_sparse_attn_decode) with the
 *           split-K merge of WHL common.py:40-89, and the decode attend of
 *           modeling_deepseekv2.py:424-451 (_decode_attend).
 * Same logit rule as prefill.  The selected blocks plus the local window are
 * split across `num_splits` CTAs per (row, kv head) (0 = automatic); partial
 * results go to the workspace and the last CTA of each (row, kv head) merges
 * them (no CTA ever waits for another).  Workspace: dash_decode_workspace_size. */
typedef struct {
  DashSeqs seqs;
  DashKV kv;
  DashRoutes routes;
  DashQO qo;
  float scale;
  int32_t block_size;
  int32_t local_window;
  int32_t num_splits;
  void* workspace;
  size_t workspace_bytes;
  DashDeviceError* device_error;
} DashDecodeArgs;
/* Bytes of split scratch dash_decode_attn needs for these arguments; 0 when it
 * needs none (one split) or when the arguments are malformed (dash_decode_attn
 * then returns the status and dash_last_error says why). */
size_t dash_decode_workspace_size(const DashDecodeArgs* args);
int dash_decode_attn(const DashDecodeArgs* args, dash_stream_t stream);

/* Allocation-free decode (no counterpart in the reference; the reference
 * allocates its split scratch through PyTorch).  For callers that cannot call
 * cudaMalloc or hand the library a workspace -- e.g. a host program whose
 * device memory is owned by its own pool, or a bare FFI consumer without an
 * allocator.  Same arguments and result as dash_decode_attn; `workspace` is
 * ignored.  The split scratch is a fixed array of
 * DASH_NOALLOC_SCRATCH_BYTES inside this library's device memory (each GPU
 * that loads the library holds it until process exit); calls whose split
 * scratch would exceed it return DASH_ERR_WORKSPACE with a message.  The
 * first call on each device looks up the array's device address (with that
 * device current), so make a first call on a device before any stream
 * capture.  All calls share the one array, which keeps the last call's
 * contents; every call first clears the arrival counters in it (an
 * asynchronous memset on `stream`).  Calls that overlap on the GPU (other
 * streams, other host threads) race on the array and must be serialised by
 * the caller.  No cudaMalloc, cudaFree or allocating library routine is
 * called. */
#define DASH_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int dash_decode_attn_noalloc(const DashDecodeArgs* args, dash_stream_t stream);
size_t dash_noalloc_scratch_bytes(void);

/* ---------------------------------------------------------------------- */
/* Router front end: index projections + RMSNorm + RoPE (+ index-K write).
 * Replaces: modeling_deepseekv2.py:336-348 (_router_qk) with the _RMSNorm of
 *           dash_attention.py:680-700 (norm_clamp = 1), and WHL
 *           unlimited_ocr_v2.py:145-162 (index_q/k_proj + GemmaRMSNorm +
 *           apply_page2d_rope_pair of WHL page2d_rope.py:130-141 / :233-257,
 *           norm_clamp = 0) with the index-K store of WHL
 *           memory_pool.py:5573-5591 (set_index_k_buffer).
 * Per token t (row of hidden [T, hidden_dim] bf16):
 *   xq = bf16(hidden[t] . w_q^T), xk likewise (bf16 GEMM, fp32 accumulate);
 *   y = bf16((x * rsqrt(mean(x^2) + eps)) * (1 + norm_w))      (norm_clamp = 0)
 *       with x non-finite -> 0 and clamps to +-1e4 after each product when
 *       norm_clamp = 1;
 *   RoPE (cos/sin [T, d] bf16, optional), rotate-half pairs (j, j + d/2),
 *   each product and the sum rounded to bf16 (the reference's bf16 ops):
 *       o_j = bf16(bf16(y_j cos_j) + bf16(rot_j sin_j)), rot = (-y_hi, y_lo);
 *   idx_q[t] = o_q (fp32); idx_k row (slot_mapping ? slot_mapping[t] : t) = o_k
 *   (fp32 or bf16).  d = 128, hidden_dim a multiple of 64 (>= 64).           */
typedef struct {
  const void* hidden; int64_t hidden_stride;   /* bf16, elements */
  const void* w_q; const void* w_k;            /* bf16 [d, hidden_dim] (nn.Linear weights) */
  int64_t w_stride;
  const float* norm_q; const float* norm_k;    /* [d] */
  const void* cos; const void* sin;            /* bf16 [T, cs_stride] or NULL (no RoPE) */
  int64_t cs_stride;
  float eps;
  int32_t norm_clamp;
  int32_t T;
  int32_t hidden_dim;
  int32_t d;
  int32_t k_dtype;                             /* DASH_DTYPE_F32 or DASH_DTYPE_BF16 */
  float* idx_q; int64_t q_stride;              /* [T, d] fp32 */
  void* idx_k; int64_t k_stride;               /* rows of d */
  const int64_t* slot_mapping;                 /* optional [T] */
  int64_t k_rows;                              /* rows addressable through slot_mapping */
  DashDeviceError* device_error;
  /* Fused k-bar refresh (optional; replaces the separate dash_kbar_pool launch
   * of WHL route_triton.py:707-726 on decode steps): after the idx_k write,
   * the k-bar row kbar_page[t] (>= 0) is recomputed from the first
   * kbar_ntok[t] cache rows of that page (rows kbar_page[t] * kbar_block_size
   * + j), with dash_kbar_pool's arithmetic (bitwise the same result).  Needs
   * slot_mapping; a page named by token t may receive no other token of this
   * call (one token per request, as in a decode step). */
  const int64_t* kbar_page;                    /* [T] or NULL */
  const int32_t* kbar_ntok;                    /* [T] */
  const float* kbar_head_cls;                  /* [d] or NULL (block mean) */
  float* kbar; int64_t kbar_row_stride;
  int32_t kbar_block_size;
  int32_t pad1;
} DashIndexProjArgs;
int dash_index_proj(const DashIndexProjArgs* args, dash_stream_t stream);

/* dash_rope_kv_write -- main-branch RoPE + paged K/V store for one step.
 * Replaces: WHL page2d_rope.py:301-323 (apply_page2d_rope_pair on q and k:
 *           rotate-half RoPE, each product and the sum rounded to bf16) and
 *           WHL memory_pool.py:5524-5545 (set_kv_buffer).
 * Token t: q[t] (n_q_heads x head_dim bf16) is rotated into q_out[t] (may be
 * q itself); k[t] rotated and v[t] copied into k_cache / v_cache rows
 * slot_mapping[t] (n_kv_heads x head_dim each, cache row stride in elements).
 * cos/sin [T, head_dim] bf16 (NULL: no rotation).  v NULL: k is only rotated
 * (into k_cache rows; slot_mapping NULL: row t), which is
 * apply_page2d_rope_pair itself.  head_dim = 128.                           */
typedef struct {
  const void* q; int64_t q_stride;          /* [T, n_q_heads * head_dim] bf16 */
  void* q_out; int64_t q_out_stride;
  const void* k; int64_t k_stride;          /* [T, n_kv_heads * head_dim] */
  const void* v; int64_t v_stride;
  const void* cos; const void* sin; int64_t cs_stride;
  void* k_cache; void* v_cache;             /* rows of n_kv_heads * head_dim */
  int64_t cache_row_stride;
  const int64_t* slot_mapping;              /* [T] */
  int64_t num_slots;
  int32_t T;
  int32_t n_q_heads;
  int32_t n_kv_heads;
  int32_t head_dim;
  DashDeviceError* device_error;
} DashRopeKVArgs;
int dash_rope_kv_write(const DashRopeKVArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* dash_attn_bwd -- training backward of the contiguous gather attention.
 * Replaces: sparse_gather_e2e_triton.py:118-189 (_e2e_attn_bwd_dq_kernel,
 *           with the d_bias atomics), :192-262 (_e2e_attn_bwd_dkv_kernel)
 *           and :319-337 (_E2EGatherAttnFn.backward: delta, block mask).
 * q, o, dout, dq: [n_seq, seq_len, n_heads, head_dim]; k, v, dk, dv:
 * [n_seq, seq_len, n_kv_heads, head_dim]; all contiguous, one dtype, 16-byte
 * aligned.  lse [n_seq, seq_len, n_heads] (natural log, as the forward
 * writes it).  idx / bias [n_seq, seq_len, K]: one routed list per token
 * shared by all heads (-1 unused; later duplicates and ids outside the
 * sequence's blocks are ignored; bias NULL = 0).  d_bias (optional)
 * [n_seq, seq_len, K]: gradient of each slot's bias (0 on ignored slots),
 * summed over all heads.  Scratch: delta [n_seq, seq_len, n_heads] fp32,
 * flags (dash_attn_bwd_flag_words() uint32 words) and, for bf16 / fp16,
 * dq_acc [n_seq, seq_len, n_heads, head_dim] fp32 (16-byte aligned).
 * bf16 / fp16 run on the tensor cores, fp32 on the CUDA cores.  head_dim
 * 128, block_size a multiple of 32, n_heads / n_kv_heads in {1, 2, 4, 8},
 * K <= 256.                                                                 */
typedef struct {
  const void* q; const void* k; const void* v; const void* o; const void* dout;
  void* dq; void* dk; void* dv;
  const float* lse;
  const int32_t* idx;
  const float* bias;
  float* d_bias;
  float* delta;
  uint32_t* flags;
  float* dq_acc;
  int32_t n_seq, seq_len, n_heads, n_kv_heads;
  int32_t head_dim, dtype, block_size, local_window;
  int32_t K, pad0;
  float scale, pad1;
  DashDeviceError* device_error;
  /* Several index heads and packed sequences (bf16 / fp16 only):
   * n_index_heads HI > 1 gives routes idx / bias / d_bias as
   * [n_seq, HI, seq_len, K], kv head h reading index head h * HI / n_kv_heads
   * (HI divides n_kv_heads); seg_start [n_seq, seq_len] int32 (or NULL = 0)
   * limits row t to keys in [seg_start, t].
   * Replaces: sparse_gather_triton.py:107-316 (_gather_attn_bwd_dq/dkv,
   *           HI index heads and segment starts).                          */
  const int32_t* seg_start;
  int32_t n_index_heads;
  int32_t pad2;
} DashAttnBwdArgs;
int dash_attn_bwd(const DashAttnBwdArgs* args, dash_stream_t stream);
int64_t dash_attn_bwd_flag_words(const DashAttnBwdArgs* args);

/* dash_entmax15_fwd / dash_entmax15_bwd -- dense 1.5-entmax over rows of n
 * and its Jacobian-vector product (training prior).
 * Replaces: dash_attention.py:623-658 (_entmax_threshold_and_support,
 *           _Entmax15.forward / backward).
 * fwd: x -> y = relu((x - max x)/2 - tau)^2 with sum y... = 1 at tau.
 * bwd: y, dy -> dx = dy*g - g * sum(dy*g) / max(sum g, 1e-12), g = sqrt(y).
 * All fp32 with a common row stride (elements).                             */
typedef struct {
  const float* x;
  float* y;
  const float* dy;
  float* dx;
  int64_t rows;
  int64_t stride;
  int32_t n;
  int32_t pad0;
} DashEntmaxArgs;
int dash_entmax15_fwd(const DashEntmaxArgs* args, dash_stream_t stream);
int dash_entmax15_bwd(const DashEntmaxArgs* args, dash_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Diagnostics */
int dash_last_error(char* buf, int len);     /* copies the last host-side error message */
int dash_library_version(void);              /* (major << 16) | minor */
int dash_count_launches(int reset);          /* kernels launched by this library so far */
/* sizeof() of the argument structs, in this order: DashSeqs, DashKV, DashRoutes,
 * DashQO, DashKbarArgs, DashRouteArgs, DashBlockMaxArgs, DashPrefillArgs,
 * DashDecodeArgs, DashDeviceError, DashPageIdsArgs, DashPageStateArgs,
 * DashPageAllowArgs, DashPageDecodeArgs, DashBlockAnyArgs, DashPageBlocksArgs,
 * DashIndexProjArgs, DashRopeKVArgs, DashAttnBwdArgs, DashEntmaxArgs,
 * DashServingPlanArgs, DashPeerHandle, DashPageCoordArgs, DashCosSin2DArgs.
 * Lets a binding
 * verify its struct layouts; returns the number of sizes available. */
int dash_abi_sizes(int64_t* out, int n);
/* Self-test of the bounded waits every kernel uses (no reference counterpart):
 * one thread waits on an mbarrier that nothing arrives on, with a limit of
 * `limit_ns` (1 ms .. 1 s); the wait gives up, records DASH_DEV_TIMEOUT in
 * `err` and the kernel returns.  Lets a host check the failure path without
 * hanging or faulting a GPU. */
int dash_selftest_bounded_wait(uint64_t limit_ns, DashDeviceError* err, dash_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* DASH_B200_H */
