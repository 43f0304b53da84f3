"""numpy restatement of the page-aware candidate domain of the DASH router.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``, never by the product package.

An OCR document is a token sequence in which image placeholders
(``image_token_id``) carry the visual tokens of each page and ``page_token_id``
markers open the pages.  The router's remote candidates are restricted to the
blocks holding image tokens of the query token's own page.  Each function below
restates one reference function (cited) over int64 numpy arrays, with the
reference's own padding, clamping and fallback rules.  ``make_document_ids``
builds the seeded synthetic documents the tests and the bench use.
"""
from __future__ import annotations

import numpy as np

IMAGE_TOKEN_ID = 128815      # config.json:156
PAGE_TOKEN_ID = 128827       # config.json:160
PER_PAGE_IMAGE_TOKENS = 273  # config.json:161
MM_PAD_SHIFT = 1_000_000     # WHL page_state.py:19


def _cumsum(x):
    return np.cumsum(x.astype(np.int64), axis=-1)


# ---------------------------------------------------------------------------
# contiguous (HF) path
# ---------------------------------------------------------------------------
def pad_ids(token_ids, key_length):
    """token_ids[..., :key_length] padded with -1 (_sparse_base_impl.py:2197-2199)."""
    t = np.asarray(token_ids, dtype=np.int64)[..., :key_length]
    if t.shape[-1] < key_length:
        t = np.concatenate([t, np.full(t.shape[:-1] + (key_length - t.shape[-1],), -1, np.int64)], -1)
    return t


def page_aware_ids(token_ids, image_token_id, page_token_id, per_page, key_length,
                   page_scope_prefill=False):
    """_sparse_base_impl.py:2189-2223 (DeepseekV2Indexer._build_page_aware_ids),
    without the batch-level ``None`` return of :2258-2260 (see ``page_aware_ids_or_none``).

    Returns (image_token_mask bool, image_token_page_ids int64,
    query_token_page_ids int64, prompt_pages int64 [B], marker_count int64 [B])."""
    ids = pad_ids(token_ids, key_length)
    img = ids == image_token_id
    starts = ids == page_token_id
    cum = _cumsum(starts)
    S = ids.shape[-1]
    ar = np.arange(S)
    last_img = (img.astype(np.int64) * (ar + 1)).max(axis=-1, initial=0) - 1
    pp = np.take_along_axis(cum, np.clip(last_img, 0, None)[:, None], 1)[:, 0] if S else \
        np.zeros(ids.shape[0], np.int64)
    pp = pp * (last_img >= 0)
    marker_mode = pp > 0
    per = max(1, int(per_page))
    run = _cumsum(img) - 1
    ipi = np.where(marker_mode[:, None], cum - 1, np.floor_divide(run, per))
    ipi = np.where(img, ipi, -1)
    raw = cum - 1
    resp = raw - np.where(marker_mode, pp, 0)[:, None]
    in_prefill = ar[None, :] <= last_img[:, None]
    qpi = np.where(in_prefill, raw, resp)
    if not page_scope_prefill:
        qpi = np.where(in_prefill, -1, qpi)
    qpi = np.where(qpi < 0, -1, qpi)
    mcum = cum[:, -1] if S else np.zeros(ids.shape[0], np.int64)
    return img, ipi, qpi, pp, mcum


def page_aware_ids_or_none(*args, **kw):
    """The reference's return contract (_sparse_base_impl.py:2258-2260)."""
    img, ipi, qpi, _, _ = page_aware_ids(*args, **kw)
    if img.sum() == 0 or (qpi >= 0).sum() == 0:
        return None, None, None
    return img, ipi, qpi


def flat_image_token_mask(token_ids, image_token_id, key_length):
    """_sparse_base_impl.py:2363-2381; None when the batch has no image token."""
    m = pad_ids(token_ids, key_length) == image_token_id
    return None if m.sum() == 0 else m


def image_block_allow_mask(image_token_mask, num_key_blocks, block_size):
    """_sparse_base_impl.py:2177-2187: [B, nblk] any image token in the block."""
    m = np.asarray(image_token_mask, dtype=bool)
    B, Sk = m.shape
    n = num_key_blocks * block_size
    m = m[:, :n] if Sk >= n else np.concatenate([m, np.zeros((B, n - Sk), bool)], 1)
    return m.reshape(B, num_key_blocks, block_size).any(-1)


def page_blocks(image_token_page_ids, num_key_blocks, block_size):
    """[B, nblk, bs] image page ids padded with -1 / truncated
    (_sparse_base_impl.py:2390-2397)."""
    p = np.asarray(image_token_page_ids, dtype=np.int64)
    B, k_len = p.shape
    n = num_key_blocks * block_size
    p = p[:, :n] if k_len >= n else np.concatenate([p, np.full((B, n - k_len), -1, np.int64)], 1)
    return p.reshape(B, num_key_blocks, block_size)


def page_aware_image_block_mask(image_token_page_ids, query_token_page_ids, pos_chunk,
                                num_key_blocks, block_size):
    """_sparse_base_impl.py:2383-2402: [B, C, nblk] block holds an image token of
    the query's page (query page gathered at the clamped position)."""
    qp_all = np.asarray(query_token_page_ids, dtype=np.int64)
    pos = np.clip(np.asarray(pos_chunk, dtype=np.int64), 0, qp_all.shape[-1] - 1)
    qp = np.take_along_axis(qp_all, pos, 1)
    kp = page_blocks(image_token_page_ids, num_key_blocks, block_size)
    out = np.zeros(qp.shape + (num_key_blocks,), bool)
    step = 256                                   # query chunks, as the reference's q_chunk
    for c0 in range(0, qp.shape[1], step):
        q = qp[:, c0:c0 + step]
        out[:, c0:c0 + step] = ((kp[:, None] == q[:, :, None, None]).any(-1)
                                & (q >= 0)[:, :, None])
    return out


def kl_candidate_mask(pos_chunk, num_key_blocks, image_token_mask, block_size,
                      image_bucket_constraint, image_token_page_ids=None,
                      query_token_page_ids=None):
    """_sparse_base_impl.py:2457-2484 (_build_kl_candidate_mask) as [B, C, nblk]
    (the reference's singleton head axis dropped)."""
    pos = np.asarray(pos_chunk, dtype=np.int64)
    B, C = pos.shape
    if image_bucket_constraint and image_token_page_ids is not None \
            and query_token_page_ids is not None:
        cand = page_aware_image_block_mask(image_token_page_ids, query_token_page_ids, pos,
                                           num_key_blocks, block_size)
    elif image_token_mask is not None:
        blk = image_block_allow_mask(image_token_mask, num_key_blocks, block_size)
        cand = np.broadcast_to(blk[:, None, :], (B, C, num_key_blocks)).copy()
    else:
        cand = np.ones((B, C, num_key_blocks), bool)
    has = cand.any(-1, keepdims=True)
    return np.where(has, cand, True)


def dash_block_cand(token_ids, image_token_id, page_token_id, per_page, key_length, pos_ids,
                    num_key_blocks, block_size, image_bucket_constraint,
                    page_scope_prefill=False):
    """modeling_deepseekv2.py:87-114 (_dash_page_ids + _dash_block_cand):
    [B, S, nblk] bool, or None when the document has no usable image ids."""
    if image_bucket_constraint:
        itm, ipi, qpi = page_aware_ids_or_none(token_ids, image_token_id, page_token_id,
                                               per_page, key_length, page_scope_prefill)
    else:
        itm = flat_image_token_mask(token_ids, image_token_id, key_length)
        ipi = qpi = None
    if itm is None and (ipi is None or qpi is None):
        return None
    return kl_candidate_mask(pos_ids, num_key_blocks, itm, block_size, image_bucket_constraint,
                             ipi, qpi)


def page_descriptors(image_token_page_ids, num_key_blocks, block_size):
    """Compact form of the per-block page sets: lo/hi (min/max page >= 0, -1 when
    the block has none) and bit k set iff page lo + k is present."""
    kp = page_blocks(image_token_page_ids, num_key_blocks, block_size)
    valid = kp >= 0
    hi = np.where(valid, kp, -1).max(-1)
    lo = np.where(valid, kp, np.iinfo(np.int64).max).min(-1)
    lo = np.where(hi >= 0, lo, -1)
    words = max(1, block_size // 32)
    bits = np.zeros(kp.shape[:2] + (words,), np.uint32)
    B, nb, _ = kp.shape
    for b in range(B):
        for j in range(nb):
            for p in set(kp[b, j][kp[b, j] >= 0].tolist()):
                k = p - lo[b, j]
                if k < 32 * words:
                    bits[b, j, k >> 5] |= np.uint32(1 << (k & 31))
    return lo, hi, bits


def decode_allow_prefill(ids, image_token_id, page_token_id, per_page, block_size):
    """modeling_anantaocr.py:468-481 (_uocr_dash_decode_allow, q_len > 1): per
    block [min, max] image page (per-token marker rule), pp, marker count."""
    ids = np.asarray(ids, dtype=np.int64)
    B, L = ids.shape
    img = ids == image_token_id
    cum = _cumsum(ids == page_token_id)
    run = _cumsum(img)
    per = max(1, int(per_page))
    page = np.where(cum > 0, cum - 1, np.floor_divide(run - 1, per))
    page = np.where(img, page, -1)
    pp = np.maximum.accumulate(np.where(img, cum, 0), axis=-1)[:, -1]
    nblk = -(-L // block_size)
    pg = np.concatenate([page, np.full((B, nblk * block_size - L), -1, np.int64)], 1)
    pg = pg.reshape(B, nblk, block_size)
    bmax = pg.max(-1)
    bmin = np.where(pg >= 0, pg, 1 << 30).min(-1)
    bmin = np.where(bmax >= 0, bmin, -1)
    return {"bmin": bmin, "bmax": bmax, "pp": pp, "mcum": cum[:, -1].copy()}


def decode_allow_step(state, last_ids, total, page_token_id, block_size):
    """modeling_anantaocr.py:482-496 (q_len == 1): updates state['mcum'] and
    returns allow [B, nblk] (same page, or every block when the row has none)."""
    st = state
    st["mcum"] = st["mcum"] + (np.asarray(last_ids) == page_token_id).astype(np.int64)
    qp = st["mcum"] - 1 - st["pp"]
    qp = np.where(qp >= 0, qp, -1)[:, None]
    nblk = -(-int(total) // block_size)
    bmin, bmax = st["bmin"], st["bmax"]
    same = (bmin >= 0) & (bmin <= qp) & (bmax >= qp) & (qp >= 0)
    open_row = (qp[:, 0] < 0) | ~same.any(-1)
    allow = np.zeros((bmin.shape[0], nblk), bool)
    n0 = min(nblk, same.shape[-1])
    allow[:, :n0] = same[:, :n0]
    return allow | open_row[:, None]


# ---------------------------------------------------------------------------
# block-paged serving path (sglang wheel)
# ---------------------------------------------------------------------------
def is_image(ids, image_token_id):
    """WHL page_state.py:22-24."""
    ids = np.asarray(ids, dtype=np.int64)
    return (ids >= MM_PAD_SHIFT) | (ids == image_token_id)


def new_slot_state(num_slots):
    """WHL page_state.py:185-198."""
    return {"img_page": np.full(num_slots, -1, np.int64), "marker_cum": np.zeros(num_slots, np.int64),
            "img_run": np.zeros(num_slots, np.int64), "prompt_pages": np.zeros(num_slots, np.int64)}


def page_state_step(state, ids, q_start, start_pos, block_table, slot_mapping, num_slots,
                    block_size, per_page, image_token_id, page_token_id,
                    num_decode_tokens=0, gen_start=None):
    """WHL page_state.py:200-313 (PageIsolationState._carry + step): updates the
    slot state in place, returns q_page [T] int64."""
    ids = np.asarray(ids, dtype=np.int64)
    q_start = np.asarray(q_start, dtype=np.int64)
    start_pos = np.asarray(start_pos, dtype=np.int64)
    bt = np.asarray(block_table, dtype=np.int64)
    T = int(q_start[-1])
    R = start_pos.shape[0]
    bs = block_size
    q_page = np.zeros(T, np.int64)
    for r in range(R):
        prev_m = prev_i = prev_pp = 0
        if start_pos[r] - 1 >= 0:
            p = start_pos[r] - 1
            blk = min(p // bs, bt.shape[1] - 1)
            slot = int(np.clip(bt[r, blk] * bs + p % bs, 0, num_slots - 1))
            prev_m = state["marker_cum"][slot]
            prev_i = state["img_run"][slot]
            prev_pp = state["prompt_pages"][slot]
        m, i, x = prev_m, prev_i, 0
        for t in range(q_start[r], q_start[r + 1]):
            img = ids[t] >= MM_PAD_SHIFT or ids[t] == image_token_id
            mk = page_token_id is not None and ids[t] == page_token_id
            m += int(mk)
            i += int(img)
            ip = (m - 1 if m > 0 else (i - 1) // per_page) if img else -1
            if img:
                x = max(x, m)
            pp = max(x, prev_pp)
            gen = t < num_decode_tokens or (gen_start is not None
                                            and start_pos[r] + (t - q_start[r]) >= gen_start[r])
            resp = m - 1 - pp
            text = (resp if resp >= 0 else -1) if gen else (m - 1 if m > pp else -1)
            q_page[t] = ip if img else text
            sl = int(np.clip(slot_mapping[t], 0, num_slots - 1))
            state["img_page"][sl] = ip
            state["marker_cum"][sl] = m
            state["img_run"][sl] = i
            state["prompt_pages"][sl] = pp
    for r in range(R):
        end = start_pos[r] + (q_start[r + 1] - q_start[r])
        last_blk = int(np.clip(max(end - 1, 0) // bs, 0, bt.shape[1] - 1))
        phys = bt[r, last_blk]
        rem = end % bs
        if rem > 0:
            for o in range(rem, bs):
                state["img_page"][int(np.clip(phys * bs + o, 0, num_slots - 1))] = -1
    return q_page


def block_page_bounds(slot_img_page, num_blocks, block_size):
    """WHL page_state.py:315-328 (int16 casts aside: page ids stay small)."""
    pages = np.asarray(slot_img_page, dtype=np.int64)[:num_blocks * block_size]
    pages = pages.reshape(num_blocks, block_size)
    bmax = pages.max(1)
    bmin = np.where(pages >= 0, pages, 32767).min(1)
    bmin = np.where(bmax >= 0, bmin, -1)
    return bmin, bmax


def build_query_allow(slot_img_page, block_table, q_start, q_page, max_block, num_blocks,
                      block_size):
    """WHL page_state.py:330-371: [T, max_block] same page | open row."""
    bmin, bmax = block_page_bounds(slot_img_page, num_blocks, block_size)
    bt = np.asarray(block_table, dtype=np.int64)
    q_start = np.asarray(q_start, dtype=np.int64)
    w = min(max_block, bt.shape[1])
    R = bt.shape[0]
    bmin_r = np.full((R, max_block), -1, np.int64)
    bmax_r = np.full((R, max_block), -1, np.int64)
    idx = np.clip(bt[:, :w], 0, num_blocks - 1)
    bmin_r[:, :w] = bmin[idx]
    bmax_r[:, :w] = bmax[idx]
    T = int(q_start[-1])
    req = np.searchsorted(q_start[1:], np.arange(T), side="right").clip(max=R - 1)
    qp = np.asarray(q_page, dtype=np.int64)[:, None]
    bmin_q, bmax_q = bmin_r[req], bmax_r[req]
    same = (bmin_q >= 0) & (bmin_q <= qp) & (qp <= bmax_q) & (qp >= 0)
    open_row = (qp < 0) | ~same.any(-1, keepdims=True)
    return same | open_row


def decode_allow(slot_img_page, block_table, q_page, seq_lens, max_block, num_blocks,
                 block_size):
    """WHL decode_meta_triton.py:107-163 (_decode_allow_kernel): [R, max_block]."""
    bt = np.asarray(block_table, dtype=np.int64)
    R = len(q_page)
    W = min(max_block, bt.shape[1])
    pages = np.asarray(slot_img_page, dtype=np.int64)
    out = np.zeros((R, max_block), bool)
    for r in range(R):
        qp, seq = int(q_page[r]), int(seq_lens[r])
        same = np.zeros(max_block, bool)
        for w in range(W):
            if w * block_size >= seq:
                continue
            ph = int(np.clip(bt[r, w], 0, num_blocks - 1))
            ip = pages[ph * block_size:(ph + 1) * block_size]
            bmax = ip.max()
            bmin = ip[ip >= 0].min() if bmax >= 0 else -1
            same[w] = bmin >= 0 and bmin <= qp <= bmax and qp >= 0
        open_row = qp < 0 or not same.any()
        out[r] = same | open_row
    return out


def local_union(allow, seq_lens, max_block, block_size, local_blocks):
    """WHL decode_meta_triton.py:212-243 (_local_union_kernel)."""
    allow = np.asarray(allow, dtype=bool)
    out = np.zeros((allow.shape[0], max_block), bool)
    for r in range(allow.shape[0]):
        q_blk = (int(seq_lens[r]) - 1) // block_size
        hi = min(max(q_blk, 0), max_block - 1)
        lo = min(max(q_blk - (local_blocks - 1), 0), max_block - 1)
        w = np.arange(max_block)
        a = np.zeros(max_block, bool)
        n = min(max_block, allow.shape[1])
        a[:n] = allow[r, :n]
        out[r] = a | ((w >= lo) & (w <= hi))
    return out


# ---------------------------------------------------------------------------
# serving-step plans (which k-bar pages to refresh; row -> request)
# ---------------------------------------------------------------------------
def _plan_entry(bt_row, seq_len, blk, block_size, bt_width):
    page = int(bt_row[min(blk, bt_width - 1)])
    live = min(max(int(seq_len) - blk * block_size, 0), block_size)
    return page, live


def plan_prefill_pages(block_table, seq_lens, context_lens, block_size, max_block, max_query_len):
    """WHL route_triton.py:576-601 (kbar_all_plan): per request, ``width``
    consecutive blocks from the one holding its first new token; a block past
    the usable table width names the last column (with 0 live tokens)."""
    R = len(seq_lens)
    bt_width = min(int(max_block), block_table.shape[1])
    width = min(bt_width, -(-int(max_query_len) // block_size) + 1)
    pages = np.zeros(R * width, np.int64)
    ntok = np.zeros(R * width, np.int32)
    for r in range(R):
        first = int(context_lens[r]) // block_size
        for j in range(width):
            pages[r * width + j], ntok[r * width + j] = _plan_entry(
                block_table[r], seq_lens[r], first + j, block_size, bt_width)
    return pages, ntok


def plan_tail_pages(block_table, seq_lens, block_size, tail_pages):
    """WHL route_triton.py:682-703 (kbar_tail_plan): the ``tail_pages`` newest
    blocks of every request, newest first, clamped at block 0."""
    R = len(seq_lens)
    pages = np.zeros(R * tail_pages, np.int64)
    ntok = np.zeros(R * tail_pages, np.int32)
    for r in range(R):
        n_blocks = -(-int(seq_lens[r]) // block_size)
        last = max(n_blocks - 1, 0)
        for j in range(tail_pages):
            pages[r * tail_pages + j], ntok[r * tail_pages + j] = _plan_entry(
                block_table[r], seq_lens[r], max(last - j, 0), block_size, block_table.shape[1])
    return pages, ntok


def rows_to_requests(cu_seqlens_q):
    """WHL route_triton.py:605-620 (prefill_row2req): request of every query row."""
    out = []
    for r in range(len(cu_seqlens_q) - 1):
        out += [r] * int(cu_seqlens_q[r + 1] - cu_seqlens_q[r])
    return np.asarray(out, np.int32)


# ---------------------------------------------------------------------------
# synthetic documents
# ---------------------------------------------------------------------------
def make_document_ids(rng, length, *, n_pages, page_tokens=PER_PAGE_IMAGE_TOKENS,
                      markers=True, text_in_page=0, empty_pages=0, lead_images=0,
                      response_pages=1, vocab=100_000):
    """One seeded OCR-like document of exactly ``length`` ids: optional lead image
    tokens before any marker, ``n_pages`` pages of [<PAGE>] + image tokens (with
    ``text_in_page`` text ids scattered inside), ``empty_pages`` markers without
    images, then a text tail carrying ``response_pages`` more markers."""
    out = []
    out += [IMAGE_TOKEN_ID] * lead_images
    kinds = ["img"] * n_pages + ["empty"] * empty_pages
    rng.shuffle(kinds)
    for k in kinds:
        if markers:
            out.append(PAGE_TOKEN_ID)
        if k == "img":
            page = [IMAGE_TOKEN_ID] * page_tokens
            for _ in range(text_in_page):
                page.insert(int(rng.integers(1, len(page))), int(rng.integers(0, vocab)))
            out += page
    tail = max(0, length - len(out))
    text = rng.integers(0, vocab, size=tail).tolist()
    if markers and tail > 0:
        for _ in range(response_pages):
            text[int(rng.integers(0, tail))] = PAGE_TOKEN_ID
    out += text
    return np.asarray(out[:length], dtype=np.int64)
