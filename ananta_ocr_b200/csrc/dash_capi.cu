// dash_capi.cu -- the extern "C" boundary of libdash_b200.so: argument
// validation (every malformed call returns a status and a message instead of
// reaching a kernel), workspace sizing and kernel launches.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <atomic>

#include "dash_internal.h"

namespace dash {

static thread_local char g_err[512] = {0};
static std::atomic<int> g_launches{0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* kernel) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(DASH_ERR_CUDA, "%s launch failed: %s", kernel, cudaGetErrorString(e));
  return DASH_OK;
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int64_t seq_rows(const DashSeqs& q) {
  // number of query rows; for the packed layout the host passes max_q_len and
  // the row count through q_len_fixed = total rows (see DashSeqs contract)
  return q.q_start ? (int64_t)q.q_len_fixed : (int64_t)q.n_seq * q.q_len_fixed;
}

static int check_seqs(const DashSeqs& q) {
  if (q.n_seq < 0) return set_error(DASH_ERR_INVALID, "n_seq < 0");
  if (q.q_len_fixed < 0) return set_error(DASH_ERR_INVALID, "q_len_fixed < 0");
  if (q.q_start == nullptr && q.max_q_len < q.q_len_fixed)
    return set_error(DASH_ERR_INVALID, "max_q_len < q_len_fixed");
  if (q.kv_len == nullptr && q.kv_len_fixed < 0) return set_error(DASH_ERR_INVALID, "kv_len_fixed < 0");
  return DASH_OK;
}

static int check_kv(const DashKV& kv, int n_heads, int block_size, bool allow_f32 = false) {
  if (!kv.k || !kv.v) return set_error(DASH_ERR_INVALID, "null K/V pointer");
  if (kv.dtype != DASH_DTYPE_BF16 && kv.dtype != DASH_DTYPE_F16 &&
      !(allow_f32 && kv.dtype == DASH_DTYPE_F32 && !kv.block_table))
    return set_error(DASH_ERR_UNSUPPORTED, allow_f32 ? "K/V dtype must be bf16 or fp16 (fp32: contiguous only)"
                                                     : "K/V dtype must be bf16 or fp16");
  if (kv.head_dim != 128) return set_error(DASH_ERR_UNSUPPORTED, "head_dim %d != 128", kv.head_dim);
  if (kv.n_kv_heads <= 0 || n_heads % kv.n_kv_heads != 0)
    return set_error(DASH_ERR_INVALID, "n_heads %d not a multiple of n_kv_heads %d", n_heads, kv.n_kv_heads);
  if (!aligned16(kv.k) || !aligned16(kv.v)) return set_error(DASH_ERR_INVALID, "K/V must be 16-byte aligned");
  if (kv.stride_tok % 8 || kv.stride_head % 8 || kv.stride_seq % 8)
    return set_error(DASH_ERR_INVALID, "K/V strides must be multiples of 8 elements");
  if (kv.block_table && kv.num_pages <= 0) return set_error(DASH_ERR_INVALID, "num_pages must be > 0");
  if (block_size <= 0) return set_error(DASH_ERR_INVALID, "block_size must be > 0");
  return DASH_OK;
}

static int check_routes(const DashRoutes& r, int n_heads, int n_kv_heads) {
  if (r.K < 0) return set_error(DASH_ERR_INVALID, "K < 0");
  if (r.K > 0 && !r.idx) return set_error(DASH_ERR_INVALID, "null route idx");
  if (r.K > 256) return set_error(DASH_ERR_UNSUPPORTED, "K %d > 256", r.K);
  int nih = r.n_index_heads > 0 ? r.n_index_heads : 1;
  if (n_heads % nih != 0 || n_kv_heads % nih != 0)
    return set_error(DASH_ERR_INVALID, "n_index_heads %d must divide heads (%d) and kv heads (%d)", nih,
                     n_heads, n_kv_heads);
  return DASH_OK;
}

static int check_qo(const DashQO& qo) {
  if (!qo.q || !qo.out) return set_error(DASH_ERR_INVALID, "null q/out");
  if (!aligned16(qo.q) || !aligned16(qo.out)) return set_error(DASH_ERR_INVALID, "q/out must be 16-byte aligned");
  if (qo.q_stride_tok % 8 || qo.q_stride_head % 8 || qo.q_stride_seq % 8 || qo.o_stride_tok % 8 ||
      qo.o_stride_head % 8 || qo.o_stride_seq % 8)
    return set_error(DASH_ERR_INVALID, "q/out strides must be multiples of 8 elements");
  return DASH_OK;
}

}  // namespace dash

namespace dash {

// Every check of a decode call that does not depend on the workspace, and the
// split count it will run with.  Shared by dash_decode_attn, the workspace
// query and the allocation-free entry point, so a malformed call is rejected
// before anything is sized (no division by a zero block size, no size from a
// negative row count).
int validate_decode(const DashDecodeArgs* a, int* splits) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  int rc = check_seqs(a->seqs);
  if (!rc) rc = check_kv(a->kv, a->qo.n_heads, a->block_size);
  if (!rc) rc = check_routes(a->routes, a->qo.n_heads, a->kv.n_kv_heads);
  if (!rc) rc = check_qo(a->qo);
  if (rc) return rc;
  if (a->local_window < 0) return set_error(DASH_ERR_INVALID, "local_window must be >= 0");
  if (a->routes.K + a->local_window / a->block_size + 2 > 480)
    return set_error(DASH_ERR_UNSUPPORTED, "too many blocks per decode row");
  if (a->num_splits < 0) return set_error(DASH_ERR_INVALID, "num_splits must be >= 0");
  const int sp = a->num_splits > 0 ? a->num_splits : decode_auto_splits(*a, seq_rows(a->seqs));
  if (sp > 64) return set_error(DASH_ERR_UNSUPPORTED, "num_splits %d > 64", sp);
  *splits = sp;
  return DASH_OK;
}

}  // namespace dash

using namespace dash;

extern "C" {

int dash_last_error(char* buf, int len) {
  if (buf && len > 0) {
    strncpy(buf, g_err, (size_t)len - 1);
    buf[len - 1] = 0;
  }
  return (int)strlen(g_err);
}

int dash_library_version(void) { return (0 << 16) | 1; }

int dash_count_launches(int reset) {
  int v = g_launches.load();
  if (reset) g_launches.store(0);
  return v;
}

int dash_abi_sizes(int64_t* out, int n) {
  const int64_t s[24] = {(int64_t)sizeof(DashSeqs),           (int64_t)sizeof(DashKV),
                         (int64_t)sizeof(DashRoutes),         (int64_t)sizeof(DashQO),
                         (int64_t)sizeof(DashKbarArgs),       (int64_t)sizeof(DashRouteArgs),
                         (int64_t)sizeof(DashBlockMaxArgs),   (int64_t)sizeof(DashPrefillArgs),
                         (int64_t)sizeof(DashDecodeArgs),     (int64_t)sizeof(DashDeviceError),
                         (int64_t)sizeof(DashPageIdsArgs),    (int64_t)sizeof(DashPageStateArgs),
                         (int64_t)sizeof(DashPageAllowArgs),  (int64_t)sizeof(DashPageDecodeArgs),
                         (int64_t)sizeof(DashBlockAnyArgs),   (int64_t)sizeof(DashPageBlocksArgs),
                         (int64_t)sizeof(DashIndexProjArgs),  (int64_t)sizeof(DashRopeKVArgs),
                         (int64_t)sizeof(DashAttnBwdArgs),    (int64_t)sizeof(DashEntmaxArgs),
                         (int64_t)sizeof(DashServingPlanArgs), (int64_t)sizeof(DashPeerHandle),
                         (int64_t)sizeof(DashPageCoordArgs),   (int64_t)sizeof(DashCosSin2DArgs)};
  for (int i = 0; i < n && i < 24; ++i) out[i] = s[i];
  return 24;
}

static int validate_kbar(const DashKbarArgs* a) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (!a->keys || !a->kbar) return set_error(DASH_ERR_INVALID, "null keys/kbar");
  if (a->dtype != DASH_DTYPE_F32 && a->dtype != DASH_DTYPE_BF16)
    return set_error(DASH_ERR_UNSUPPORTED, "k-bar keys must be fp32 or bf16");
  if (a->d <= 0 || a->d > 256) return set_error(DASH_ERR_UNSUPPORTED, "index dim %d not in (0, 256]", a->d);
  if (a->block_size <= 0 || a->block_size > 256)
    return set_error(DASH_ERR_UNSUPPORTED, "block_size %d not in (0, 256]", a->block_size);
  if (a->pages && !a->ntok) return set_error(DASH_ERR_INVALID, "paged plan needs ntok");
  if (!a->pages && (a->n_seq < 0 || a->seq_len < 0)) return set_error(DASH_ERR_INVALID, "bad n_seq/seq_len");
  return DASH_OK;
}

int dash_kbar_pool(const DashKbarArgs* a, dash_stream_t stream) {
  const int rc = validate_kbar(a);
  return rc != DASH_OK ? rc : launch_kbar(*a, (cudaStream_t)stream);
}

static int validate_route(const DashRouteArgs* a) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  int rc = check_seqs(a->seqs);
  if (rc) return rc;
  if (!a->out_idx || !a->out_bias) return set_error(DASH_ERR_INVALID, "null outputs");
  if (a->width <= 0) return set_error(DASH_ERR_INVALID, "width must be > 0");
  if (a->width > 8192) return set_error(DASH_ERR_UNSUPPORTED, "width %d > 8192", a->width);
  if (a->K <= 0 || a->out_width < a->K) return set_error(DASH_ERR_INVALID, "need 0 < K <= out_width");
  int M = a->topm > 0 ? (a->topm < a->width ? a->topm : a->width) : a->width;
  if (M > 256) return set_error(DASH_ERR_UNSUPPORTED, "entmax window %d > 256 (set topm)", M);
  if (!a->scores_in) {
    if (!a->idx_q || !a->kbar) return set_error(DASH_ERR_INVALID, "null idx_q/kbar");
    if (a->d != 128) return set_error(DASH_ERR_UNSUPPORTED, "index dim %d != 128", a->d);
    if (!aligned16(a->kbar) || a->kbar_row_stride % 4) return set_error(DASH_ERR_INVALID, "k-bar must be 16-byte aligned rows");
    if (a->num_kbar_rows <= 0) return set_error(DASH_ERR_INVALID, "num_kbar_rows must be > 0");
    if (a->block_size <= 0) return set_error(DASH_ERR_INVALID, "block_size must be > 0");
  }
  if (a->page_q) {
    if (!a->page_lo || !a->page_hi) return set_error(DASH_ERR_INVALID, "page mode needs page_lo/page_hi");
    if (a->page_bits && (a->page_bits_words <= 0 || a->page_bits_words > 8))
      return set_error(DASH_ERR_INVALID, "page_bits_words %d not in [1, 8]", a->page_bits_words);
    if (a->num_page_desc <= 0) return set_error(DASH_ERR_INVALID, "num_page_desc must be > 0");
    if (!a->block_table && a->page_seq_rows < a->width)
      return set_error(DASH_ERR_INVALID, "page_seq_rows %lld < width %d", (long long)a->page_seq_rows,
                       a->width);
  }
  return DASH_OK;
}

int dash_route(const DashRouteArgs* a, dash_stream_t stream) {
  const int rc = validate_route(a);
  return rc != DASH_OK ? rc : launch_route(*a, seq_rows(a->seqs), (cudaStream_t)stream);
}

int dash_route_refresh(const DashRouteArgs* a, const DashKbarArgs* refresh, dash_stream_t stream) {
  int rc = validate_route(a);
  if (rc != DASH_OK) return rc;
  if (!refresh) return launch_route(*a, seq_rows(a->seqs), (cudaStream_t)stream);
  rc = validate_kbar(refresh);
  if (rc != DASH_OK) return rc;
  if (!refresh->pages) return set_error(DASH_ERR_INVALID, "the folded refresh takes a paged plan");
  if (refresh->kbar != a->kbar && a->kbar)
    return set_error(DASH_ERR_INVALID, "the refresh must write the k-bar rows the routing reads");
  return launch_route_refresh(*a, seq_rows(a->seqs), *refresh, (cudaStream_t)stream);
}

int dash_block_max(const DashBlockMaxArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (!a->q || !a->k || !a->pos || !a->out) return set_error(DASH_ERR_INVALID, "null pointer");
  if (a->d <= 0 || a->d > 256) return set_error(DASH_ERR_UNSUPPORTED, "dim %d not in (0, 256]", a->d);
  if (a->block_size <= 0 || a->block_size > 128)
    return set_error(DASH_ERR_UNSUPPORTED, "block_size %d not in (0, 128]", a->block_size);
  if (a->B < 0 || a->C < 0 || a->Sk < 0 || a->nblk < 0) return set_error(DASH_ERR_INVALID, "negative size");
  return launch_block_max(*a, (cudaStream_t)stream);
}

size_t dash_prefill_workspace_size(const DashPrefillArgs* a) {
  if (!a) return 0;
  return prefill_workspace(*a, seq_rows(a->seqs));
}

int dash_prefill_attn(const DashPrefillArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  int rc = check_seqs(a->seqs);
  if (!rc) rc = check_kv(a->kv, a->qo.n_heads, a->block_size, true);
  if (!rc) rc = check_routes(a->routes, a->qo.n_heads, a->kv.n_kv_heads);
  if (!rc) rc = check_qo(a->qo);
  if (rc) return rc;
  const int G = a->qo.n_heads / a->kv.n_kv_heads;
  if (a->kv.dtype != DASH_DTYPE_F32) {
    // tensor-core kernel: 128-row tiles of 128/G tokens, 64-key tiles
    if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16)
      return set_error(DASH_ERR_UNSUPPORTED, "query heads per kv head %d not in {1,2,4,8,16}", G);
    if (a->block_size != 32 && (a->block_size % 64 != 0 || a->block_size > 256))
      return set_error(DASH_ERR_UNSUPPORTED, "prefill block_size %d not in {32,64,128,192,256}", a->block_size);
  } else if (G > 128) {
    return set_error(DASH_ERR_UNSUPPORTED, "query heads per kv head %d > 128", G);
  }
  if (a->local_window < 0) return set_error(DASH_ERR_INVALID, "local_window must be >= 0");
  if (a->kv.block_table == nullptr && a->seqs.kv_len_fixed <= 0)
    return set_error(DASH_ERR_INVALID, "contiguous K/V needs kv_len_fixed (allocated length)");
  if (a->n_peers < 0 || a->n_peers > 64 || (a->n_peers > 0 && !a->out_peers))
    return set_error(DASH_ERR_INVALID, "n_peers must be in [0, 64] with an out_peers array");
  if (a->mode < 0 || a->mode > 2) return set_error(DASH_ERR_INVALID, "mode %d not in {0,1,2}", a->mode);
  if (a->part_budget_mib < 0) return set_error(DASH_ERR_INVALID, "part_budget_mib must be >= 0");
  if (a->mode == 2 && !prefill_gathered_supported(*a))
    return set_error(DASH_ERR_UNSUPPORTED, "gathered prefill needs bf16/fp16, block_size 32/64/128, "
                     "1/2/4 query heads per kv head and 0 < K <= 256 (block_size %d, K %d)",
                     a->block_size, a->routes.K);
  int64_t rows = seq_rows(a->seqs);
  size_t need = prefill_workspace(*a, rows);
  if (need && (!a->workspace || a->workspace_bytes < need))
    return set_error(DASH_ERR_WORKSPACE, "prefill workspace %zu bytes needed, %zu given", need,
                     a->workspace_bytes);
  return launch_prefill(*a, rows, (cudaStream_t)stream);
}

size_t dash_decode_workspace_size(const DashDecodeArgs* a) {
  int sp = 0;
  if (validate_decode(a, &sp)) return 0;
  return decode_workspace(*a, seq_rows(a->seqs), sp);
}

int dash_decode_attn(const DashDecodeArgs* a, dash_stream_t stream) {
  int sp = 0;
  int rc = validate_decode(a, &sp);
  if (rc) return rc;
  int64_t rows = seq_rows(a->seqs);
  size_t need = decode_workspace(*a, rows, sp);
  if (need && (!a->workspace || a->workspace_bytes < need))
    return set_error(DASH_ERR_WORKSPACE, "decode workspace %zu bytes needed, %zu given", need,
                     a->workspace_bytes);
  return launch_decode(*a, rows, sp, (cudaStream_t)stream);
}

static bool pow2_block(int bs) { return bs >= 16 && bs <= 256 && (bs & (bs - 1)) == 0; }

int dash_page_ids(const DashPageIdsArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->n_seq < 0 || a->key_length < 0 || a->ids_len < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->n_seq > 0 && a->key_length > 0 && a->ids_len > 0 && !a->token_ids)
    return set_error(DASH_ERR_INVALID, "null token_ids");
  if (a->per_page < 1) return set_error(DASH_ERR_INVALID, "per_page must be >= 1");
  if (a->rule != 0 && a->rule != 1) return set_error(DASH_ERR_INVALID, "rule must be 0 or 1");
  if (a->rule == 1 && a->query_page) return set_error(DASH_ERR_INVALID, "rule 1 produces no query pages");
  if ((a->image_page || a->query_page) && a->page_elem_bytes != 4 && a->page_elem_bytes != 8)
    return set_error(DASH_ERR_INVALID, "page_elem_bytes must be 4 or 8");
  const bool blocks = a->blk_lo || a->blk_hi || a->blk_bits || a->blk_has_image;
  if (blocks) {
    if (!pow2_block(a->block_size))
      return set_error(DASH_ERR_UNSUPPORTED, "block_size %d: block outputs need a power of two in [16, 256]",
                       a->block_size);
    if (a->n_blocks < 0) return set_error(DASH_ERR_INVALID, "n_blocks < 0");
  }
  return launch_page_ids(*a, (cudaStream_t)stream);
}

int dash_page_state_step(const DashPageStateArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->num_reqs < 0 || a->num_tokens < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->num_reqs == 0) return DASH_OK;
  if (!a->input_ids || !a->block_table || !a->slot_mapping || !a->q_page)
    return set_error(DASH_ERR_INVALID, "null ids/block_table/slot_mapping/q_page");
  if (!a->slot_img_page || !a->slot_marker_cum || !a->slot_img_run || !a->slot_prompt_pages)
    return set_error(DASH_ERR_INVALID, "null slot state");
  if (!a->q_start && a->num_tokens != a->num_reqs)
    return set_error(DASH_ERR_INVALID, "without q_start every request owns one token");
  if (!a->start_pos && !a->seq_lens) return set_error(DASH_ERR_INVALID, "need start_pos or seq_lens");
  if (a->num_slots <= 0 || a->block_size <= 0 || a->bt_width <= 0 || a->per_page < 1)
    return set_error(DASH_ERR_INVALID, "num_slots, block_size, bt_width and per_page must be > 0");
  if (!a->blk_lo != !a->blk_hi) return set_error(DASH_ERR_INVALID, "blk_lo and blk_hi go together");
  return launch_page_state(*a, (cudaStream_t)stream);
}

int dash_page_allow(const DashPageAllowArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->rows < 0 || a->width < 0 || a->desc_width < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->rows == 0 || a->width == 0) return DASH_OK;
  if (!a->out || !a->q_page || !a->page_lo || !a->page_hi)
    return set_error(DASH_ERR_INVALID, "null out/q_page/page_lo/page_hi");
  if (!a->row_seq && a->rows_per_seq <= 0) return set_error(DASH_ERR_INVALID, "rows_per_seq must be > 0");
  if (a->q_elem_bytes != 4 && a->q_elem_bytes != 8) return set_error(DASH_ERR_INVALID, "q_elem_bytes must be 4 or 8");
  if (a->q_pos && a->q_len <= 0) return set_error(DASH_ERR_INVALID, "q_len must be > 0 with q_pos");
  if (a->page_bits && (a->page_bits_words <= 0 || a->page_bits_words > 8))
    return set_error(DASH_ERR_INVALID, "page_bits_words %d not in [1, 8]", a->page_bits_words);
  if (a->num_desc <= 0) return set_error(DASH_ERR_INVALID, "num_desc must be > 0");
  if (a->seq_lens && a->block_size <= 0) return set_error(DASH_ERR_INVALID, "block_size must be > 0");
  return launch_page_allow(*a, (cudaStream_t)stream);
}

int dash_page_blocks(const DashPageBlocksArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->rows < 0 || a->len < 0 || a->n_blocks < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->block_size <= 0 || a->block_size > 256)
    return set_error(DASH_ERR_UNSUPPORTED, "block_size %d not in (0, 256]", a->block_size);
  if (a->elem_bytes != 4 && a->elem_bytes != 8) return set_error(DASH_ERR_INVALID, "elem_bytes must be 4 or 8");
  if (a->rows > 0 && a->n_blocks > 0 && (!a->lo || !a->hi || (a->len > 0 && !a->pages)))
    return set_error(DASH_ERR_INVALID, "null pages/lo/hi");
  return launch_page_blocks(*a, (cudaStream_t)stream);
}

int dash_index_proj(const DashIndexProjArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->T < 0) return set_error(DASH_ERR_INVALID, "T < 0");
  if (a->T == 0) return DASH_OK;
  if (a->d != 128) return set_error(DASH_ERR_UNSUPPORTED, "index dim %d != 128", a->d);
  if (a->hidden_dim <= 0 || a->hidden_dim % 64)
    return set_error(DASH_ERR_UNSUPPORTED, "hidden_dim %d must be a positive multiple of 64", a->hidden_dim);
  if (!a->hidden || !a->w_q || !a->w_k || !a->norm_q || !a->norm_k || !a->idx_q || !a->idx_k)
    return set_error(DASH_ERR_INVALID, "null pointer");
  if (!aligned16(a->hidden) || !aligned16(a->w_q) || !aligned16(a->w_k))
    return set_error(DASH_ERR_INVALID, "hidden and weights must be 16-byte aligned");
  if (a->hidden_stride < a->hidden_dim || a->hidden_stride % 8 || a->w_stride < a->hidden_dim || a->w_stride % 8)
    return set_error(DASH_ERR_INVALID, "hidden / weight row strides must cover hidden_dim and be multiples of 8");
  if (!a->cos != !a->sin) return set_error(DASH_ERR_INVALID, "cos and sin go together");
  if (a->cos && (!aligned16(a->cos) || !aligned16(a->sin) || a->cs_stride % 8 || a->cs_stride < a->d))
    return set_error(DASH_ERR_INVALID, "cos/sin must be 16-byte aligned with a row stride multiple of 8 >= d");
  if (a->k_dtype != DASH_DTYPE_F32 && a->k_dtype != DASH_DTYPE_BF16)
    return set_error(DASH_ERR_UNSUPPORTED, "idx_k dtype must be fp32 or bf16");
  if (a->slot_mapping && a->k_rows <= 0) return set_error(DASH_ERR_INVALID, "k_rows must be > 0 with slot_mapping");
  if (a->kbar_page) {
    if (!a->slot_mapping || !a->kbar_ntok || !a->kbar)
      return set_error(DASH_ERR_INVALID, "the fused k-bar refresh needs slot_mapping, kbar_ntok and kbar");
    if (a->kbar_block_size <= 0 || a->kbar_block_size > 256)
      return set_error(DASH_ERR_UNSUPPORTED, "kbar_block_size %d not in (0, 256]", a->kbar_block_size);
    if (a->kbar_row_stride < a->d) return set_error(DASH_ERR_INVALID, "kbar_row_stride < d");
  }
  if (!aligned16(a->idx_q) || a->q_stride % 4 || a->q_stride < a->d)
    return set_error(DASH_ERR_INVALID, "idx_q must be 16-byte aligned with a row stride multiple of 4 >= d");
  if ((reinterpret_cast<uintptr_t>(a->idx_k) & (a->k_dtype == DASH_DTYPE_BF16 ? 7 : 15)) || a->k_stride % 4 ||
      a->k_stride < a->d)
    return set_error(DASH_ERR_INVALID, "idx_k rows must be aligned for vector stores (row stride multiple of 4 >= d)");
  return launch_index_proj(*a, (cudaStream_t)stream);
}

int dash_rope_kv_write(const DashRopeKVArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->T < 0 || a->n_q_heads < 0 || a->n_kv_heads < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->T == 0) return DASH_OK;
  if (a->head_dim != 128) return set_error(DASH_ERR_UNSUPPORTED, "head_dim %d != 128", a->head_dim);
  if ((a->n_q_heads && (!a->q || !a->q_out)) || (a->n_kv_heads && (!a->k || !a->k_cache)) ||
      (a->v && !a->v_cache))
    return set_error(DASH_ERR_INVALID, "null pointer");
  if (!a->cos != !a->sin) return set_error(DASH_ERR_INVALID, "cos and sin go together");
  const void* ptrs[7] = {a->q, a->q_out, a->k, a->v, a->k_cache, a->v_cache, a->cos};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return set_error(DASH_ERR_INVALID, "tensors must be 16-byte aligned");
  if (a->sin && !aligned16(a->sin)) return set_error(DASH_ERR_INVALID, "tensors must be 16-byte aligned");
  if (a->q_stride % 8 || a->q_out_stride % 8 || a->k_stride % 8 || a->v_stride % 8 || a->cache_row_stride % 8 ||
      (a->cos && a->cs_stride % 8))
    return set_error(DASH_ERR_INVALID, "row strides must be multiples of 8 elements");
  if (a->cache_row_stride < (int64_t)a->n_kv_heads * a->head_dim)
    return set_error(DASH_ERR_INVALID, "cache rows shorter than n_kv_heads * head_dim");
  if (a->n_kv_heads && a->num_slots <= 0) return set_error(DASH_ERR_INVALID, "num_slots must be > 0");
  return launch_rope_kv(*a, (cudaStream_t)stream);
}

int dash_page_decode_query(const DashPageDecodeArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->n_seq < 0) return set_error(DASH_ERR_INVALID, "n_seq < 0");
  if (a->n_seq > 0 && (!a->last_ids || !a->marker_count || !a->prompt_pages || !a->q_page))
    return set_error(DASH_ERR_INVALID, "null pointer");
  return launch_page_decode(*a, (cudaStream_t)stream);
}

int dash_block_any(const DashBlockAnyArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->rows < 0 || a->len < 0 || a->n_blocks < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->block_size <= 0) return set_error(DASH_ERR_INVALID, "block_size must be > 0");
  if (a->rows > 0 && a->n_blocks > 0 && (!a->out || (a->len > 0 && !a->mask)))
    return set_error(DASH_ERR_INVALID, "null mask/out");
  return launch_block_any(*a, (cudaStream_t)stream);
}

static int check_attn_bwd(const DashAttnBwdArgs* a) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->n_seq < 0 || a->seq_len < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->head_dim != 128) return set_error(DASH_ERR_UNSUPPORTED, "head_dim %d != 128", a->head_dim);
  if (a->block_size <= 0 || a->block_size % 32)
    return set_error(DASH_ERR_UNSUPPORTED, "block_size %d must be a positive multiple of 32", a->block_size);
  if (a->local_window <= 0) return set_error(DASH_ERR_INVALID, "local_window must be > 0");
  if (a->K < 0 || a->K > 256) return set_error(DASH_ERR_UNSUPPORTED, "K %d not in [0, 256]", a->K);
  if (a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads)
    return set_error(DASH_ERR_INVALID, "n_heads must be a multiple of n_kv_heads");
  const int G = a->n_heads / a->n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(DASH_ERR_UNSUPPORTED, "query heads per kv head %d not in {1,2,4,8}", G);
  if (a->dtype != DASH_DTYPE_BF16 && a->dtype != DASH_DTYPE_F16 && a->dtype != DASH_DTYPE_F32)
    return set_error(DASH_ERR_UNSUPPORTED, "dtype must be bf16, fp16 or fp32");
  const int HI = a->n_index_heads > 1 ? a->n_index_heads : 1;
  if (a->n_kv_heads % HI)
    return set_error(DASH_ERR_INVALID, "n_index_heads %d must divide n_kv_heads %d", HI, a->n_kv_heads);
  if ((HI > 1 || a->seg_start) && a->dtype == DASH_DTYPE_F32)
    return set_error(DASH_ERR_UNSUPPORTED, "several index heads / segment starts need bf16 or fp16");
  return DASH_OK;
}

int64_t dash_attn_bwd_flag_words(const DashAttnBwdArgs* a) {
  if (check_attn_bwd(a)) return -1;
  return (int64_t)attn_bwd_flag_words(*a);
}

int dash_attn_bwd(const DashAttnBwdArgs* a, dash_stream_t stream) {
  int rc = check_attn_bwd(a);
  if (rc) return rc;
  if ((int64_t)a->n_seq * a->seq_len == 0) return DASH_OK;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->dq || !a->dk || !a->dv || !a->lse ||
      !a->delta || !a->flags || (a->K > 0 && !a->idx))
    return set_error(DASH_ERR_INVALID, "null pointer");
  const void* vec[] = {a->q, a->k, a->v, a->o, a->dout, a->dq, a->dk, a->dv};
  for (const void* p : vec)
    if (!aligned16(p)) return set_error(DASH_ERR_INVALID, "q/k/v/o/dout/dq/dk/dv must be 16-byte aligned");
  if (a->scale <= 0.f) return set_error(DASH_ERR_INVALID, "scale must be > 0");
  if ((a->dtype == DASH_DTYPE_BF16 || a->dtype == DASH_DTYPE_F16) && (!a->dq_acc || !aligned16(a->dq_acc)))
    return set_error(DASH_ERR_INVALID, "bf16/fp16 need a 16-byte aligned dq_acc scratch");
  return launch_attn_bwd(*a, (cudaStream_t)stream);
}

static int check_entmax(const DashEntmaxArgs* a, bool bwd) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->rows < 0 || a->n < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->rows > 0 && a->stride < a->n) return set_error(DASH_ERR_INVALID, "row stride < n");
  if (a->rows > 0 && a->n > 0 && (bwd ? (!a->y || !a->dy || !a->dx) : (!a->x || !a->y)))
    return set_error(DASH_ERR_INVALID, "null pointer");
  return DASH_OK;
}

int dash_serving_plan(const DashServingPlanArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->n_req < 0) return set_error(DASH_ERR_INVALID, "n_req < 0");
  if (a->n_req == 0) return DASH_OK;
  if (!a->seq_lens) return set_error(DASH_ERR_INVALID, "null seq_lens");
  if (a->pages || a->ntok) {
    if (!a->pages || !a->ntok || !a->block_table)
      return set_error(DASH_ERR_INVALID, "a page plan needs pages, ntok and block_table");
    if (a->block_size <= 0 || a->width < 0 || a->bt_width <= 0 || a->bt_stride < a->bt_width)
      return set_error(DASH_ERR_INVALID, "block_size and bt_width must be > 0, width >= 0, "
                       "bt_stride >= bt_width");
    if (a->mode != 0 && a->mode != 1) return set_error(DASH_ERR_INVALID, "mode must be 0 or 1");
    if (a->mode == 0 && !a->context_lens) return set_error(DASH_ERR_INVALID, "mode 0 needs context_lens");
  }
  if (a->row2req && !a->cu_seqlens_q) return set_error(DASH_ERR_INVALID, "row2req needs cu_seqlens_q");
  return launch_serving_plan(*a, (cudaStream_t)stream);
}

int dash_page_coords(const DashPageCoordArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->num_reqs < 0 || a->num_tokens < 0) return set_error(DASH_ERR_INVALID, "negative size");
  if (a->num_reqs == 0) return DASH_OK;
  if (!a->q_start && a->num_tokens != a->num_reqs)
    return set_error(DASH_ERR_INVALID, "without q_start every request owns one token");
  if (!a->input_ids || !a->start_pos || !a->row_key || !a->state_key || !a->state_stamp || !a->step ||
      !a->c_marker || !a->c_pp || !a->cnt || !a->rows || !a->tok_pos || !a->page_pos)
    return set_error(DASH_ERR_INVALID, "null pointer");
  if (a->max_rows < a->num_reqs || a->max_pages < 1)
    return set_error(DASH_ERR_INVALID, "need max_rows >= num_reqs and max_pages >= 1");
  return launch_page_coords(*a, (cudaStream_t)stream);
}

int dash_cos_sin_2d(const DashCosSin2DArgs* a, dash_stream_t stream) {
  if (!a) return set_error(DASH_ERR_INVALID, "null args");
  if (a->num_tokens < 0) return set_error(DASH_ERR_INVALID, "num_tokens < 0");
  if (a->num_tokens == 0) return DASH_OK;
  if (a->dim <= 0 || a->dim % 2 || a->n_tok <= 0 || a->n_tok >= a->dim / 2)
    return set_error(DASH_ERR_INVALID, "need an even dim and 0 < n_tok < dim / 2");
  if (a->stride < a->dim || a->page_mod < 0) return set_error(DASH_ERR_INVALID, "bad stride / page_mod");
  if (!a->tok_pos || !a->page_pos || !a->inv_tok || !a->inv_page || !a->cos || !a->sin)
    return set_error(DASH_ERR_INVALID, "null pointer");
  return launch_cos_sin_2d(*a, (cudaStream_t)stream);
}

int dash_entmax15_fwd(const DashEntmaxArgs* a, dash_stream_t stream) {
  int rc = check_entmax(a, false);
  return rc ? rc : launch_entmax15(*a, false, (cudaStream_t)stream);
}

int dash_entmax15_bwd(const DashEntmaxArgs* a, dash_stream_t stream) {
  int rc = check_entmax(a, true);
  return rc ? rc : launch_entmax15(*a, true, (cudaStream_t)stream);
}

}  // extern "C"
