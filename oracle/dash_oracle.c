/*
 * dash_oracle.c -- CPU restatement of ANANTA_OCR's DASH block-sparse attention
 * forward (router + gather attention), used ONLY as test infrastructure: the
 * parity checker of tests/, the smoke check of __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py.  The product path (ananta_ocr_b200) never calls
 * into this file; it fails loudly when its CUDA library is missing.
 *
 * Parity pin: every function below is checked against golden vectors produced
 * by running the reference's own PyTorch functions in the build container
 * (tests/golden/make_golden.py -> tests/golden/*.npz, tests/test_oracle_golden.py).
 *
 * Floating-point operation order.  The router half of this file (k-bar pooling,
 * block scores, selection) fixes ONE explicit fp32 operation sequence: every dot
 * product is a sequential fmaf chain over the feature index, every sum a
 * sequential fp32 add in index order, exp() is det_expf() below (a Cody-Waite
 * range reduction plus a degree-7 Taylor polynomial, written from the maths).
 * The CUDA router kernels evaluate the same sequence with __fmaf_rn/__fmul_rn,
 * so block scores -- and therefore the selected block indices -- are
 * bit-identical between this oracle and the GPU.  The reference (torch/BLAS)
 * sums in another order, so against the reference the scores agree to fp32
 * rounding and the indices agree except at near-ties; the golden test checks
 * exactly that.
 *
 * The attention half accumulates in double precision (it is the fp32/fp64
 * reference the bf16 kernels are compared to with a tolerance).
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -ffp-contract=off -shared -fPIC).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#define ORC_SCORE_NEG (-1.0e9f)   /* dash_attention.py:602 _SCORE_NEG          */
#define ORC_ENTMAX_NEG (-1.0e4f)  /* modeling_deepseekv2.py:55 _ENTMAX_NEG     */
#define ORC_ACT_CLAMP (1.0e4f)    /* dash_attention.py:604 _ACT_CLAMP           */

static inline float f_as(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_as(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* clamp that keeps NaN as NaN, like torch.clamp (dash_attention.py:887). */
static inline float clamp_act(float z) {
  if (z < -ORC_ACT_CLAMP) return -ORC_ACT_CLAMP;
  if (z > ORC_ACT_CLAMP) return ORC_ACT_CLAMP;
  return z;
}

/* exp(x) for x <= 0 with a fixed operation sequence (Cody-Waite reduction by
 * ln2 split in a 16-bit head and a tail, Horner Taylor polynomial of degree 7,
 * exact scaling by 2^n).  Inputs below -87 return 0 (the pooling weights it
 * feeds are then far below the fp32 resolution of the 1.0 weight of the row
 * maximum). */
float det_expf(float x) {
  if (x != x) return x;
  if (x < -87.0f) return 0.0f;
  if (x > 0.0f) x = 0.0f;
  const float log2e = f_as(0x3FB8AA3Bu);       /* 1.44269504 */
  const float ln2_hi = f_as(0x3F317200u);      /* 0.693145751953125 */
  const float ln2_lo = f_as(0x35BFBE8Eu);      /* 1.42860677e-06 */
  float n = rintf(x * log2e);
  float r = fmaf(n, -ln2_hi, x);
  r = fmaf(n, -ln2_lo, r);
  float p = f_as(0x39500D01u);                 /* 1/5040 */
  p = fmaf(p, r, f_as(0x3AB60B61u));           /* 1/720  */
  p = fmaf(p, r, f_as(0x3C088889u));           /* 1/120  */
  p = fmaf(p, r, f_as(0x3D2AAAABu));           /* 1/24   */
  p = fmaf(p, r, f_as(0x3E2AAAABu));           /* 1/6    */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;                             /* in [-126, 0] */
  float s = f_as((uint32_t)(ni + 127) << 23);
  return p * s;
}

/* ------------------------------------------------------------------------ */
/* Stage-0 head_cls pooling of one key block.                                */
/* Restates dash_attention.py:863-888 (_block_scores_headcls),               */
/* modeling_deepseekv2.py:362-379 (_block_scores_infer, head_cls branch),    */
/* WHL sglang/.../unlimited_dash_ops/dash_stage0.py:25-41 (_summary_keys)    */
/* and route_triton.py:36-72 (_kbar_page_kernel).                            */
/*   aw_j = clamp(<k_j, hc> / sqrt(d)); w = masked softmax over the n valid  */
/*   tokens (denominator >= 1e-6); kbar = sum_j w_j k_j; non-finite -> 0.    */
/* head_cls == 0 reduces to the block mean.                                  */
/* ------------------------------------------------------------------------ */
void orc_kbar_block(const float* keys, int64_t key_stride, int n_valid, int d,
                    const float* hc, float inv_sqrt_d, float* out) {
  float aw[1024];
  float e[1024];
  if (n_valid > 1024) n_valid = 1024;
  if (n_valid <= 0) {
    for (int c = 0; c < d; ++c) out[c] = 0.0f;
    return;
  }
  float rmax = -INFINITY;
  for (int j = 0; j < n_valid; ++j) {
    const float* kj = keys + (int64_t)j * key_stride;
    float acc = 0.0f;
    for (int c = 0; c < d; ++c) acc = fmaf(kj[c], hc[c], acc);
    float a = clamp_act(acc * inv_sqrt_d);
    aw[j] = a;
    if (a > rmax) rmax = a;
  }
  float sum = 0.0f;
  for (int j = 0; j < n_valid; ++j) {
    e[j] = det_expf(aw[j] - rmax);
    sum = sum + e[j];
  }
  float den = sum > 1e-6f ? sum : 1e-6f;
  for (int j = 0; j < n_valid; ++j) e[j] = e[j] / den;
  for (int c = 0; c < d; ++c) {
    float acc = 0.0f;
    for (int j = 0; j < n_valid; ++j) acc = fmaf(e[j], keys[(int64_t)j * key_stride + c], acc);
    if (!(acc == acc) || acc == INFINITY || acc == -INFINITY) acc = 0.0f;
    out[c] = acc;
  }
}

/* Contiguous k-bar for keys [B, S, d] (row stride d): out [B, nblk, d]. */
void orc_kbar_contig(const float* idx_k, int B, int S, int d, int bs,
                     const float* hc, float* out) {
  int nblk = (S + bs - 1) / bs;
  float inv_sqrt_d = (float)(1.0 / sqrt((double)d));
#pragma omp parallel for collapse(2) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int k = 0; k < nblk; ++k) {
      int n = S - k * bs;
      if (n > bs) n = bs;
      orc_kbar_block(idx_k + ((int64_t)b * S + (int64_t)k * bs) * d, d, n, d, hc,
                     inv_sqrt_d, out + ((int64_t)b * nblk + k) * d);
    }
}

/* Paged k-bar for an index-key cache [num_pages, bs, d] (row stride d):
 * out[page] for each (page, ntok) pair of the plan; ntok == 0 entries are
 * skipped (route_triton.py:69-72). */
void orc_kbar_paged(const float* cache, int bs, int d, const int64_t* pages,
                    const int32_t* ntok, int n_plan, const float* hc, float* kbar_out) {
  float inv_sqrt_d = (float)(1.0 / sqrt((double)d));
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n_plan; ++i) {
    if (ntok[i] <= 0) continue;
    orc_kbar_block(cache + pages[i] * (int64_t)bs * d, d, ntok[i], d, hc, inv_sqrt_d,
                   kbar_out + pages[i] * (int64_t)d);
  }
}

/* ------------------------------------------------------------------------ */
/* Block scores.  modeling_deepseekv2.py:380-388, dash_stage0.py:44-59,      */
/* route_triton.py:529-572 / 75-126:                                         */
/*   z = clamp(<q, kbar_b> / sqrt(d)); kept iff b <= qblk - local_blocks and */
/*   the block holds a live token (b*bs < kv_len); else SCORE_NEG.           */
/* kbar rows are addressed through an optional block table (paged cache).    */
/* ------------------------------------------------------------------------ */
void orc_scores(const float* q, int64_t q_stride, int n_rows, const int64_t* q_pos,
                const int64_t* row_kv_len, const float* kbar, int64_t kbar_row_stride,
                const int64_t* row_kbar_base, const int32_t* block_table,
                const int64_t* row_bt_base, int d, int nblk, int bs, int local_blocks,
                float* out, int64_t out_stride) {
  float inv_sqrt_d = (float)(1.0 / sqrt((double)d));
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n_rows; ++r) {
    const float* qr = q + (int64_t)r * q_stride;
    int64_t qblk = q_pos[r] / bs;
    int64_t kvl = row_kv_len[r];
    for (int b = 0; b < nblk; ++b) {
      float z = ORC_SCORE_NEG;
      if ((int64_t)b <= qblk - local_blocks && (int64_t)b * bs < kvl) {
        int64_t kr = block_table ? (int64_t)block_table[row_bt_base[r] + b]
                                 : row_kbar_base[r] + b;
        const float* kb = kbar + kr * kbar_row_stride;
        float acc = 0.0f;
        for (int c = 0; c < d; ++c) acc = fmaf(qr[c], kb[c], acc);
        z = clamp_act(acc * inv_sqrt_d);
      }
      out[(int64_t)r * out_stride + b] = z;
    }
  }
}

/* Indexer stage-0 block-max scores (dash_attention.py:801-835,              */
/* modeling_deepseekv2.py:389-400, sparse_gather_triton.py:395-467):         */
/*   s_j = clamp(<q, k_j>); keys kept iff seg <= j <= pos - LW;  block score  */
/*   = max over kept keys of the block, `empty` when none is kept.           */
void orc_block_max(const float* q, int64_t q_stride, int n_rows, const int64_t* q_pos,
                   const int64_t* q_seg, const float* k, int64_t k_stride, int Sk, int d,
                   int bs, int nblk, int local_window, int clamp_dots, float empty,
                   float* out, int64_t out_stride) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < n_rows; ++r) {
    const float* qr = q + (int64_t)r * q_stride;
    int64_t hi = q_pos[r] - local_window;   /* last remote key */
    int64_t lo = q_seg ? q_seg[r] : 0;
    for (int b = 0; b < nblk; ++b) {
      float m = empty;
      int any = 0;
      for (int t = 0; t < bs; ++t) {
        int64_t j = (int64_t)b * bs + t;
        if (j >= Sk || j > hi || j < lo) continue;
        const float* kj = k + j * k_stride;
        float acc = 0.0f;
        for (int c = 0; c < d; ++c) acc = fmaf(qr[c], kj[c], acc);
        if (clamp_dots) acc = clamp_act(acc);
        if (!any || acc > m || (acc != acc)) { m = acc; any = 1; }
      }
      out[(int64_t)r * out_stride + b] = m;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* 1.5-entmax (dash_attention.py:623-648, dash_router.py:25-52): sort-based  */
/* exact threshold over a row that is ALREADY sorted descending.             */
/* ------------------------------------------------------------------------ */
static void entmax15_sorted(const float* xs, int M, float* p) {
  float z[4096];
  float xmax = xs[0];
  for (int i = 0; i < M; ++i) z[i] = (xs[i] - xmax) / 2.0f;
  float cs = 0.0f, cs2 = 0.0f;
  int support = 0;
  float tau_at[4096];
  for (int k = 0; k < M; ++k) {
    float rho = (float)(k + 1);
    cs = cs + z[k];
    cs2 = cs2 + z[k] * z[k];
    float mean = cs / rho;
    float mean_sq = cs2 / rho;
    float ss = rho * (mean_sq - mean * mean);
    float delta = (1.0f - ss) / rho;
    float dnz = delta > 0.0f ? delta : 0.0f;
    float tau = mean - sqrtf(dnz);
    tau_at[k] = tau;
    if (tau <= z[k]) support++;
  }
  if (support < 1) support = 1;
  float tau_star = tau_at[support - 1];
  for (int i = 0; i < M; ++i) {
    float t = z[i] - tau_star;
    t = t > 0.0f ? t : 0.0f;
    p[i] = t * t;
  }
}

/* ------------------------------------------------------------------------ */
/* Canonical routing selection: modeling_deepseekv2.py:309-333               */
/* (_infer_route_select) == dash_router.py:131-174 (route_and_select).       */
/*   cand = remote & cmask, per-row fallback to remote when empty;           */
/*   x = cand ? s*idx_scale : ENTMAX_NEG;  top-M of x (M = topm, or nblk     */
/*   when topm <= 0), ties -> lowest block id;  prior = entmax15(top-M);     */
/*   keep the first K; valid = cand; logp = log(max(prior, floor));          */
/*   bias = valid ? (logp - mean_valid(logp)) / sigma : 0.                    */
/* Output is canonical: valid block ids ascending, -1 tail, bias permuted    */
/* alongside; n_valid per row is returned in out_cnt (may be NULL).          */
/* ------------------------------------------------------------------------ */
void orc_select(const float* scores, int64_t s_stride, const uint8_t* cmask,
                int64_t c_stride, int n_rows, int nblk, float idx_scale, int topm,
                int K, float prior_floor, float inv_sigma, int32_t* out_idx,
                float* out_bias, int64_t o_stride, int32_t* out_cnt) {
#pragma omp parallel for schedule(dynamic, 16)
  for (int r = 0; r < n_rows; ++r) {
    const float* s = scores + (int64_t)r * s_stride;
    const uint8_t* cm = cmask ? cmask + (int64_t)r * c_stride : NULL;
    uint8_t* cand = (uint8_t*)malloc((size_t)nblk);
    float* x = (float*)malloc(sizeof(float) * (size_t)nblk);
    int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)nblk);
    int any = 0;
    for (int b = 0; b < nblk; ++b) {
      int remote = s[b] > ORC_SCORE_NEG * 0.5f;
      cand[b] = (uint8_t)(remote && (!cm || cm[b]));
      any |= cand[b];
    }
    if (!any)
      for (int b = 0; b < nblk; ++b) cand[b] = (uint8_t)(s[b] > ORC_SCORE_NEG * 0.5f);
    float fs = idx_scale;
    for (int b = 0; b < nblk; ++b) {
      float v = cand[b] ? s[b] * fs : ORC_ENTMAX_NEG;
      if (!(v == v) || v == INFINITY || v == -INFINITY) v = ORC_ENTMAX_NEG;
      x[b] = v;
    }
    int M = topm > 0 ? (topm < nblk ? topm : nblk) : nblk;
    if (M < 1) M = 1;
    /* stable selection of the top-M: (x desc, id asc) */
    for (int b = 0; b < nblk; ++b) order[b] = b;
    for (int i = 0; i < M; ++i) {
      int best = i;
      for (int j = i + 1; j < nblk; ++j) {
        int oj = order[j], ob = order[best];
        if (x[oj] > x[ob] || (x[oj] == x[ob] && oj < ob)) best = j;
      }
      int t = order[i]; order[i] = order[best]; order[best] = t;
    }
    float xs[4096], prior[4096];
    for (int i = 0; i < M; ++i) xs[i] = x[order[i]];
    entmax15_sorted(xs, M, prior);
    int Kc = K < M ? K : M;
    if (Kc < 1) Kc = 1;
    float logp[4096];
    int cnt = 0;
    float lsum = 0.0f;
    for (int i = 0; i < Kc; ++i) {
      float pr = prior[i] > prior_floor ? prior[i] : prior_floor;
      logp[i] = logf(pr);
      if (cand[order[i]]) { cnt++; lsum = lsum + logp[i]; }
    }
    float mu = lsum / (float)(cnt > 0 ? cnt : 1);
    /* canonical ascending output */
    int32_t sel_id[4096];
    float sel_b[4096];
    int nv = 0;
    for (int i = 0; i < Kc; ++i) {
      if (!cand[order[i]]) continue;
      float bb = (logp[i] - mu) * inv_sigma;
      int j = nv++;
      while (j > 0 && sel_id[j - 1] > order[i]) { sel_id[j] = sel_id[j - 1]; sel_b[j] = sel_b[j - 1]; --j; }
      sel_id[j] = order[i];
      sel_b[j] = bb;
    }
    int32_t* oi = out_idx + (int64_t)r * o_stride;
    float* ob = out_bias + (int64_t)r * o_stride;
    for (int i = 0; i < K; ++i) {
      oi[i] = i < nv ? sel_id[i] : -1;
      ob[i] = i < nv ? sel_b[i] : 0.0f;
    }
    if (out_cnt) out_cnt[r] = nv;
    free(cand); free(x); free(order);
  }
}

/* ------------------------------------------------------------------------ */
/* Gather attention for a set of (row, head) pairs, double accumulation.     */
/* Restates dash_attention.py:980-1006 (_forward_dense),                     */
/* modeling_deepseekv2.py:424-451 (_decode_attend) and the kernels           */
/* sparse_gather_e2e_triton.py:34-115, sparse_gather_triton.py:29-104,       */
/* WHL attend_triton.py:88-292 / 307-518:                                     */
/*   key j (0 <= j <= pos, j >= seg) is LOCAL when j > pos - LW (bias 0);    */
/*   otherwise it is read iff its block j/bs is in the row's routed list,    */
/*   with that slot's bias (first occurrence of a duplicated id wins).       */
/*   logit = scale * <q, k_j> + bias; out = softmax(logit) @ V.              */
/* Keys are addressed as  base + page(j/bs)*page_stride + (j%bs)*tok_stride  */
/* + head*head_stride, page(b) = block_table ? block_table[bt_base + b] : b, */
/* which covers both contiguous [.., S, ..] and block-paged caches.          */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* q;  int64_t q_row_stride;      /* q row of pair i at q + i*q_row_stride */
  const float* k;  const float* v;            /* key / value bases                    */
  int64_t page_stride, tok_stride, head_stride;
  const int32_t* block_table;                 /* NULL for contiguous                  */
  const int64_t* pair_kv_base;                /* per pair: offset added to k/v (elements) */
  const int64_t* pair_bt_base;                /* per pair: row offset into block_table */
  const int64_t* pair_pos;                    /* query position                        */
  const int64_t* pair_seg;                    /* first attendable key (NULL = 0)       */
  const int64_t* pair_head;                   /* kv head                                */
  const int32_t* idx; const float* bias;      /* routed list of pair i at idx + i*K (bias may be NULL) */
  int64_t idx_row_stride;
  int K, bs, local_window, d;
  float scale;
  int use_bias;
} OrcAttnArgs;

void orc_attend_pairs(const OrcAttnArgs* a, int n_pairs, float* out, float* lse_out) {
#pragma omp parallel for schedule(dynamic, 4)
  for (int i = 0; i < n_pairs; ++i) {
    const float* q = a->q + (int64_t)i * a->q_row_stride;
    int64_t pos = a->pair_pos[i];
    int64_t seg = a->pair_seg ? a->pair_seg[i] : 0;
    int64_t h = a->pair_head[i];
    int64_t kvb = a->pair_kv_base ? a->pair_kv_base[i] : 0;
    int64_t btb = a->pair_bt_base ? a->pair_bt_base[i] : 0;
    const int32_t* il = a->idx + (int64_t)i * a->idx_row_stride;
    const float* bl = a->bias ? a->bias + (int64_t)i * a->idx_row_stride : NULL;
    int64_t nkeys = pos + 1;
    double* logit = (double*)malloc(sizeof(double) * (size_t)(nkeys > 0 ? nkeys : 1));
    unsigned char* keep = (unsigned char*)malloc((size_t)(nkeys > 0 ? nkeys : 1));
    double mx = -INFINITY;
    for (int64_t j = 0; j < nkeys; ++j) {
      keep[j] = 0;
      if (j < seg) continue;
      int local = j > pos - a->local_window;
      double bb = 0.0;
      if (!local) {
        int64_t blk = j / a->bs;
        int found = 0;
        for (int s = 0; s < a->K; ++s)
          if (il[s] >= 0 && il[s] == blk) {
            found = 1;
            bb = (a->use_bias && bl) ? (double)bl[s] : 0.0;
            break;
          }
        if (!found) continue;
      }
      int64_t blk = j / a->bs;
      int64_t page = a->block_table ? (int64_t)a->block_table[btb + blk] : blk;
      const float* kj = a->k + kvb + page * a->page_stride + (j % a->bs) * a->tok_stride +
                        h * a->head_stride;
      double acc = 0.0;
      for (int c = 0; c < a->d; ++c) acc += (double)q[c] * (double)kj[c];
      double lg = (double)a->scale * acc + bb;
      logit[j] = lg;
      keep[j] = 1;
      if (lg > mx) mx = lg;
    }
    double den = 0.0;
    double* o = (double*)calloc((size_t)a->d, sizeof(double));
    for (int64_t j = 0; j < nkeys; ++j) {
      if (!keep[j]) continue;
      double p = exp(logit[j] - mx);
      den += p;
      int64_t blk = j / a->bs;
      int64_t page = a->block_table ? (int64_t)a->block_table[btb + blk] : blk;
      const float* vj = a->v + kvb + page * a->page_stride + (j % a->bs) * a->tok_stride +
                        h * a->head_stride;
      for (int c = 0; c < a->d; ++c) o[c] += p * (double)vj[c];
    }
    for (int c = 0; c < a->d; ++c)
      out[(int64_t)i * a->d + c] = den > 0.0 ? (float)(o[c] / den) : 0.0f;
    if (lse_out) lse_out[i] = den > 0.0 ? (float)(mx + log(den)) : -INFINITY;
    free(o); free(logit); free(keep);
  }
}
