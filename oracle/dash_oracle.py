"""numpy front-end of the CPU oracle (``oracle/dash_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``, never by the product package.

Each function restates one reference function (cited per function) over numpy
arrays.  Router functions (k-bar pooling, block scores, selection) run the
fixed fp32 operation order of the C file, which the CUDA router reproduces bit
for bit; attention functions accumulate in double precision.
"""
from __future__ import annotations

import ctypes as C
import math
import os

import numpy as np

from . import build as _build

SCORE_NEG = -1.0e9
ENTMAX_NEG = -1.0e4

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = C.CDLL(path)
        _declare(_lib)
    return _lib


_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_i64p = C.POINTER(C.c_int64)
_u8p = C.POINTER(C.c_uint8)


class OrcAttnArgs(C.Structure):
    _fields_ = [
        ("q", _f32p), ("q_row_stride", C.c_int64),
        ("k", _f32p), ("v", _f32p),
        ("page_stride", C.c_int64), ("tok_stride", C.c_int64), ("head_stride", C.c_int64),
        ("block_table", _i32p),
        ("pair_kv_base", _i64p), ("pair_bt_base", _i64p), ("pair_pos", _i64p),
        ("pair_seg", _i64p), ("pair_head", _i64p),
        ("idx", _i32p), ("bias", _f32p), ("idx_row_stride", C.c_int64),
        ("K", C.c_int), ("bs", C.c_int), ("local_window", C.c_int), ("d", C.c_int),
        ("scale", C.c_float), ("use_bias", C.c_int),
    ]


def _declare(L):
    L.det_expf.argtypes = [C.c_float]
    L.det_expf.restype = C.c_float
    L.orc_kbar_contig.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p]
    L.orc_kbar_paged.argtypes = [_f32p, C.c_int, C.c_int, _i64p, _i32p, C.c_int, _f32p, _f32p]
    L.orc_scores.argtypes = [_f32p, C.c_int64, C.c_int, _i64p, _i64p, _f32p, C.c_int64,
                             _i64p, _i32p, _i64p, C.c_int, C.c_int, C.c_int, C.c_int,
                             _f32p, C.c_int64]
    L.orc_block_max.argtypes = [_f32p, C.c_int64, C.c_int, _i64p, _i64p, _f32p, C.c_int64,
                                C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                C.c_float, _f32p, C.c_int64]
    L.orc_select.argtypes = [_f32p, C.c_int64, _u8p, C.c_int64, C.c_int, C.c_int, C.c_float,
                             C.c_int, C.c_int, C.c_float, C.c_float, _i32p, _f32p,
                             C.c_int64, _i32p]
    L.orc_attend_pairs.argtypes = [C.POINTER(OrcAttnArgs), C.c_int, _f32p, _f32p]


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int) -> None:
    """Set the OpenMP thread count used by the oracle library."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    try:
        gomp = C.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(int(n))
    except OSError:
        pass


def det_expf(x: float) -> float:
    return float(lib().det_expf(C.c_float(x)))


# --------------------------------------------------------------------------
# Stage-0 pooling and block scores
# --------------------------------------------------------------------------
def kbar_contig(idx_k, head_cls, block_size):
    """[B,S,d] index keys -> [B,nblk,d] head_cls summaries.

    Restates modeling_deepseekv2.py:362-379 / dash_attention.py:863-888."""
    k = _c(idx_k, np.float32)
    B, S, d = k.shape
    nblk = (S + block_size - 1) // block_size
    hc = _c(head_cls, np.float32).reshape(d)
    out = np.empty((B, nblk, d), np.float32)
    lib().orc_kbar_contig(_p(k, _f32p), B, S, d, block_size, _p(hc, _f32p), _p(out, _f32p))
    return out


def kbar_paged(index_cache, pages, ntok, head_cls, kbar_out):
    """Refresh ``kbar_out[page]`` for each planned (page, ntok).

    Restates WHL route_triton.py:36-72 / dash_stage0.py:25-41, 106-149."""
    cache = _c(index_cache, np.float32)
    P, bs, d = cache.shape
    pages = _c(pages, np.int64).reshape(-1)
    ntok = _c(ntok, np.int32).reshape(-1)
    hc = _c(head_cls, np.float32).reshape(d)
    assert kbar_out.dtype == np.float32 and kbar_out.flags.c_contiguous
    lib().orc_kbar_paged(_p(cache, _f32p), bs, d, _p(pages, _i64p), _p(ntok, _i32p),
                         len(pages), _p(hc, _f32p), _p(kbar_out, _f32p))
    return kbar_out


def block_scores_headcls(idx_q, idx_k, q_pos, block_size, local_blocks, head_cls, nblk=None):
    """``_block_scores_infer`` head_cls branch (modeling_deepseekv2.py:351-388).

    idx_q [B,Lq,d], idx_k [B,S,d] (all keys so far), q_pos [B,Lq] -> [B,Lq,nblk]."""
    q = _c(idx_q, np.float32)
    B, Lq, d = q.shape
    S = idx_k.shape[1]
    if nblk is None:
        nblk = (S + block_size - 1) // block_size
    kb = kbar_contig(idx_k, head_cls, block_size)
    nb_k = kb.shape[1]
    if nb_k < nblk:
        kb = np.concatenate([kb, np.zeros((B, nblk - nb_k, d), np.float32)], 1)
    kb = _c(kb, np.float32)
    out = np.empty((B, Lq, nblk), np.float32)
    pos = _c(np.broadcast_to(q_pos, (B, Lq)), np.int64).reshape(-1)
    kvl = np.full(B * Lq, S, np.int64)
    base = np.repeat(np.arange(B, dtype=np.int64) * kb.shape[1], Lq)
    lib().orc_scores(_p(q, _f32p), d, B * Lq, _p(pos, _i64p), _p(kvl, _i64p), _p(kb, _f32p),
                     d, _p(base, _i64p), None, None, d, nblk, block_size, local_blocks,
                     _p(out, _f32p), nblk)
    return out


def scores_paged(idx_q, q_pos, row_req, seq_lens, k_bar, block_table, block_size,
                 local_blocks, width):
    """Paged block scores off a k-bar page cache.

    Restates WHL route_triton.py:529-572 (_score_prefill_kernel) and
    dash_stage0.py:152-186 (headcls_scores_decode): row r scores blocks
    0..width-1 of request row_req[r]."""
    q = _c(idx_q, np.float32)
    n, d = q.shape
    pos = _c(q_pos, np.int64)
    req = _c(row_req, np.int64)
    kvl = _c(np.asarray(seq_lens, np.int64)[req], np.int64)
    bt = _c(block_table, np.int32)
    btb = _c(req * bt.shape[1], np.int64)
    kb = _c(k_bar, np.float32)
    out = np.empty((n, width), np.float32)
    lib().orc_scores(_p(q, _f32p), d, n, _p(pos, _i64p), _p(kvl, _i64p), _p(kb, _f32p), d,
                     None, _p(bt, _i32p), _p(btb, _i64p), d, width, block_size,
                     local_blocks, _p(out, _f32p), width)
    return out


def block_scores_indexer(idx_q, idx_k, q_pos, block_size, local_window, nblk=None,
                         q_seg=None, clamp=True, empty=SCORE_NEG):
    """Indexer stage-0: block max of token scores over remote keys.

    clamp=True/empty=SCORE_NEG restates modeling_deepseekv2.py:389-400 and
    dash_attention.py:801-835; clamp=False/empty=-inf restates
    sparse_gather_triton.py:395-467 (triton_block_max_score)."""
    q = _c(idx_q, np.float32)
    k = _c(idx_k, np.float32)
    B, Lq, d = q.shape
    Sk = k.shape[1]
    if nblk is None:
        nblk = (Sk + block_size - 1) // block_size
    out = np.empty((B, Lq, nblk), np.float32)
    pos = _c(np.broadcast_to(q_pos, (B, Lq)), np.int64)
    seg = None if q_seg is None else _c(np.broadcast_to(q_seg, (B, Lq)), np.int64)
    for b in range(B):
        lib().orc_block_max(_p(q[b], _f32p), d, Lq, _p(pos[b], _i64p),
                            None if seg is None else _p(_c(seg[b], np.int64), _i64p),
                            _p(_c(k[b], np.float32), _f32p), d, Sk, d, block_size, nblk,
                            local_window, int(bool(clamp)), float(empty),
                            _p(out[b], _f32p), nblk)
    return out


# --------------------------------------------------------------------------
# Selection
# --------------------------------------------------------------------------
def route_select(scores, cand=None, idx_scale=1.0, topm=16, K=16, prior_floor=1e-2,
                 sigma=1.0):
    """Canonical selection (modeling_deepseekv2.py:309-333, dash_router.py:131-174).

    scores [..., nblk] fp32; cand optional bool [..., nblk].
    Returns (idx int32 [..., K] ascending with -1 tail, bias fp32 [..., K], count)."""
    s = _c(scores, np.float32)
    lead = s.shape[:-1]
    nblk = s.shape[-1]
    s2 = s.reshape(-1, nblk)
    n = s2.shape[0]
    cm = None
    if cand is not None:
        cm = _c(np.broadcast_to(cand, s.shape).reshape(-1, nblk), np.uint8)
    idx = np.empty((n, K), np.int32)
    bias = np.empty((n, K), np.float32)
    cnt = np.empty(n, np.int32)
    lib().orc_select(_p(s2, _f32p), nblk, _p(cm, _u8p), nblk, n, nblk,
                     float(np.float32(idx_scale)), int(topm), int(K), float(prior_floor),
                     float(np.float32(1.0 / sigma)), _p(idx, _i32p), _p(bias, _f32p), K,
                     _p(cnt, _i32p))
    return idx.reshape(*lead, K), bias.reshape(*lead, K), cnt.reshape(lead)


# --------------------------------------------------------------------------
# Attention
# --------------------------------------------------------------------------
def _attend(q_rows, k, v, page_stride, tok_stride, head_stride, block_table, kv_base,
            bt_base, pos, seg, head, idx, bias, bs, local_window, scale):
    q_rows = _c(q_rows, np.float32)
    n, d = q_rows.shape
    idx = _c(idx, np.int32)
    K = idx.shape[-1]
    use_bias = bias is not None
    bias_a = _c(bias, np.float32) if use_bias else None
    keep = [q_rows, k, v, idx, bias_a]
    kv_base = _c(kv_base, np.int64)
    bt_base = None if bt_base is None else _c(bt_base, np.int64)
    pos = _c(pos, np.int64)
    seg = None if seg is None else _c(seg, np.int64)
    head = _c(head, np.int64)
    bt = None if block_table is None else _c(block_table, np.int32)
    keep += [kv_base, bt_base, pos, seg, head, bt]
    args = OrcAttnArgs(
        _p(q_rows, _f32p), d, _p(k, _f32p), _p(v, _f32p), page_stride, tok_stride, head_stride,
        _p(bt, _i32p), _p(kv_base, _i64p), _p(bt_base, _i64p), _p(pos, _i64p),
        _p(seg, _i64p), _p(head, _i64p), _p(idx, _i32p), _p(bias_a, _f32p), K, K, bs,
        local_window, d, float(scale), int(use_bias))
    out = np.empty((n, d), np.float32)
    lse = np.empty(n, np.float32)
    lib().orc_attend_pairs(C.byref(args), n, _p(out, _f32p), _p(lse, _f32p))
    del keep
    return out, lse


def attend_contig(q, k, v, idx, bias, block_size, local_window, scale, rows=None,
                  seg=None, return_lse=False):
    """Contiguous DASH attend (dash_attention.py:980-1006 _forward_dense;
    sparse_gather_e2e_triton.py:34-115).

    q [B,H,T,D], k/v [B,Hkv,T,D], idx [B,T,K] (routes shared by all heads, -1 pad),
    bias [B,T,K] or None.  ``rows`` is an optional int array of token positions to
    evaluate (all when None).  Returns [B,H,len(rows),D] fp32."""
    q = np.asarray(q, np.float32)
    k = _c(k, np.float32)
    v = _c(v, np.float32)
    B, H, T, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    rows = np.arange(T) if rows is None else np.asarray(rows, np.int64)
    nr = len(rows)
    bb, hh, rr = np.meshgrid(np.arange(B), np.arange(H), np.arange(nr), indexing="ij")
    bb, hh, rr = bb.reshape(-1), hh.reshape(-1), rr.reshape(-1)
    t = rows[rr]
    q_rows = q[bb, hh, t]
    kv_head = hh // G
    kv_base = (bb * Hkv * T * D).astype(np.int64)
    idx_r = np.asarray(idx)[bb, t]
    bias_r = None if bias is None else np.asarray(bias)[bb, t]
    seg_r = None if seg is None else np.asarray(seg)[bb, t]
    out, lse = _attend(q_rows, k, v, block_size * D, D, T * D, None, kv_base, None, t,
                       seg_r, kv_head, idx_r, bias_r, block_size, local_window, scale)
    o = out.reshape(B, H, nr, D)
    if return_lse:
        return o, lse.reshape(B, H, nr)
    return o


def attend_paged(q, k_cache, v_cache, idx, bias, block_table, row_req, row_pos,
                 block_size, local_window, scale, return_lse=False):
    """Paged DASH attend (WHL attend_triton.py:88-292 prefill, 307-518 decode;
    modeling_deepseekv2.py:424-451 for the decode semantics).

    q [N,H,D]; caches [P,bs,Hkv,D]; idx/bias [N,K] (shared by all kv heads);
    block_table [R,W]; row_req/row_pos [N].  Returns [N,H,D] fp32."""
    q = np.asarray(q, np.float32)
    kc = _c(k_cache, np.float32)
    vc = _c(v_cache, np.float32)
    N, H, D = q.shape
    P, bs, Hkv, _ = kc.shape
    assert bs == block_size
    G = H // Hkv
    nn, hh = np.meshgrid(np.arange(N), np.arange(H), indexing="ij")
    nn, hh = nn.reshape(-1), hh.reshape(-1)
    q_rows = q[nn, hh]
    bt = _c(block_table, np.int32)
    row_req = np.asarray(row_req, np.int64)
    row_pos = np.asarray(row_pos, np.int64)
    bt_base = row_req[nn] * bt.shape[1]
    idx_r = np.asarray(idx)[nn]
    bias_r = None if bias is None else np.asarray(bias)[nn]
    out, lse = _attend(q_rows, kc, vc, bs * Hkv * D, Hkv * D, D, bt,
                       np.zeros(len(nn), np.int64), bt_base, row_pos[nn], None, hh // G,
                       idx_r, bias_r, block_size, local_window, scale)
    if return_lse:
        return out.reshape(N, H, D), lse.reshape(N, H)
    return out.reshape(N, H, D)


# --------------------------------------------------------------------------
# Synthetic inputs (seeded; shapes and distributions of the BASELINE configs)
# --------------------------------------------------------------------------
def page_offsets(rng, S, n_heads, d, n_pages, page_tokens, std):
    """Per-page mean offsets: one N(0, std) vector per page per head, text tail 0."""
    off = np.zeros((n_heads, S, d), np.float32)
    for p in range(n_pages):
        a, b = p * page_tokens, min(S, (p + 1) * page_tokens)
        if a >= S:
            break
        off[:, a:b] = (rng.standard_normal((n_heads, 1, d)) * std).astype(np.float32)
    return off


def make_router_inputs(seed, B, S, n_pages, page_tokens, offset_std, d_idx=128, scale=0.5):
    """Router idx_q/idx_k [B,S,d_idx] fp32 only (drawn like q/k, with page offsets)."""
    rng = np.random.default_rng(seed)
    iq = np.empty((B, S, d_idx), np.float32)
    ik = np.empty((B, S, d_idx), np.float32)
    for b in range(B):
        ioff = (page_offsets(rng, S, 1, d_idx, n_pages, page_tokens, offset_std)[0]
                if offset_std else 0.0)
        iq[b] = rng.standard_normal((S, d_idx), dtype=np.float32) * scale + ioff
        ik[b] = rng.standard_normal((S, d_idx), dtype=np.float32) * scale + ioff
    return iq, ik


def make_prefill_inputs(seed, B, H, S, D, n_pages, page_tokens, offset_std, d_idx=128,
                        scale=0.5):
    """q,k,v [B,H,S,D] and router idx_q/idx_k [B,S,d_idx] (fp32 numpy)."""
    rng = np.random.default_rng(seed)
    q = np.empty((B, H, S, D), np.float32)
    k = np.empty((B, H, S, D), np.float32)
    v = np.empty((B, H, S, D), np.float32)
    iq = np.empty((B, S, d_idx), np.float32)
    ik = np.empty((B, S, d_idx), np.float32)
    for b in range(B):
        off = page_offsets(rng, S, H, D, n_pages, page_tokens, offset_std) if offset_std else 0.0
        q[b] = rng.standard_normal((H, S, D), dtype=np.float32) * scale + off
        k[b] = rng.standard_normal((H, S, D), dtype=np.float32) * scale + off
        v[b] = rng.standard_normal((H, S, D), dtype=np.float32) * scale
        ioff = (page_offsets(rng, S, 1, d_idx, n_pages, page_tokens, offset_std)[0]
                if offset_std else 0.0)
        iq[b] = rng.standard_normal((S, d_idx), dtype=np.float32) * scale + ioff
        ik[b] = rng.standard_normal((S, d_idx), dtype=np.float32) * scale + ioff
    return q, k, v, iq, ik
