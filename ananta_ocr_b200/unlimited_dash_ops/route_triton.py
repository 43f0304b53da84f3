"""Drop-in for the serving path's ``unlimited_dash_ops/route_triton.py``
(WHL sglang/srt/layers/attention/unlimited_dash_ops/route_triton.py).

Same entry points, keyword arguments and caller-owned output buffers; the
routing runs on libdash_b200.so.  Selection semantics follow the torch router
of the same package (dash_router.py:131-174, DashRouterMath.route_and_select):
top-``budget`` blocks by score (ties to the lowest id), entmax prior over the
top-``topm`` candidates, centred log-prior bias; ids packed ascending with -1 /
0.0 in unused slots.  The planning helpers (``kbar_tail_plan``,
``kbar_all_plan``, ``prefill_row2req``) are the same small torch index
computations as route_triton.py:576-620, 682-703.
"""
from __future__ import annotations

import torch

from .. import ops

SCORE_NEG = -1.0e9
ENTMAX_NEG = -1.0e4
ACT_CLAMP = 1.0e4
SCAN_TILE = 128


@torch.no_grad()
def kbar_all_plan(*, block_table, seq_lens, context_lens, block_size: int, max_block: int,
                  max_query_len: int, device, out=None):
    """Pages changed by a prefill step: the boundary page plus the pages of the
    query span (route_triton.py:576-601)."""
    sl = seq_lens.to(device=device, dtype=torch.int64)
    ctx = context_lens.to(device=device, dtype=torch.int64)
    W = min(int(max_block), int(block_table.shape[1]))
    width = min(W, -(-int(max_query_len) // int(block_size)) + 1)
    p0 = ctx // block_size
    blk = p0[:, None] + torch.arange(width, device=device)[None, :]
    pages = block_table[:, :W].to(torch.int64).gather(1, blk.clamp(max=W - 1))
    tok = (sl[:, None] - blk * block_size).clamp(0, block_size)
    n = sl.shape[0] * width
    if out is not None:
        pages_buf, tok_buf = out
        pages_buf[:n].copy_(pages.reshape(-1))
        tok_buf[:n].copy_(tok.reshape(-1).to(torch.int32))
        return pages_buf[:n], tok_buf[:n]
    return pages.reshape(-1).contiguous(), tok.reshape(-1).to(torch.int32).contiguous()


@torch.no_grad()
def prefill_row2req(*, cu_seqlens_q, device, out=None, total_q=None):
    """Query row -> request index (route_triton.py:605-620)."""
    cu = cu_seqlens_q.to(device=device, dtype=torch.int64)
    q_lens = cu[1:] - cu[:-1]
    r = torch.arange(q_lens.numel(), device=device)
    row2req = torch.repeat_interleave(r, q_lens).to(torch.int32)
    if out is not None:
        out[:row2req.shape[0]].copy_(row2req)
        return out[:row2req.shape[0]]
    return row2req.contiguous()


@torch.no_grad()
def kbar_tail_plan(*, block_table, seq_lens, block_size: int, tail_pages: int, device, out=None):
    """Mutable tail pages of every request and their live token counts
    (route_triton.py:682-703)."""
    sl = seq_lens.to(device=device, dtype=torch.int64)
    nb = (sl + block_size - 1) // block_size
    last = (nb - 1).clamp(min=0)
    offs = torch.arange(tail_pages, device=device)
    blk = (last[:, None] - offs[None, :]).clamp(min=0)
    w = int(block_table.shape[1])
    pages = block_table[:, :w].to(torch.int64).gather(1, blk.clamp(max=w - 1))
    tok = (sl[:, None] - blk * block_size).clamp(0, block_size)
    n = pages.numel()
    if out is None or out[0].shape[0] < n:
        return pages.reshape(-1).contiguous(), tok.reshape(-1).to(torch.int32).contiguous()
    p_buf, t_buf = out[0][:n], out[1][:n]
    p_buf.copy_(pages.reshape(-1))
    t_buf.copy_(tok.reshape(-1))
    return p_buf, t_buf


@torch.no_grad()
def kbar_refresh_tail_triton(*, kv_cache, k_bar, block_table, seq_lens, head_cls,
                             block_size: int, tail_pages: int = 1, plan=None):
    """Refresh the k-bar summaries of the planned pages (route_triton.py:707-726).
    ``kv_cache`` is the index-key cache [num_pages, block_size, d]."""
    if plan is None:
        plan = kbar_tail_plan(block_table=block_table, seq_lens=seq_lens, block_size=block_size,
                              tail_pages=tail_pages, device=k_bar.device)
    pages, tok = plan
    cache = kv_cache.view(kv_cache.shape[0], block_size, -1)
    ops.kbar_pool_paged(cache, pages, tok, head_cls, k_bar)


def _out_slots(out_idx, topm, out_slots):
    M = min(int(out_slots or topm), int(out_idx.shape[-1]))
    assert M & (M - 1) == 0, f"out_slots must be a power of two, got {M}"
    return M


@torch.no_grad()
def route_prefill_triton(*, idx_q, k_bar, block_table, seq_lens, cu_seqlens_q, context_lens,
                         row2req, image_allow, out_idx, out_bias, max_block: int,
                         block_size: int, local_blocks: int, idx_scale: float,
                         prior_floor: float, sigma: float, topm: int, budget=None,
                         q_chunk: int = 2048, out_slots=None, score_buf=None, page_domain=None):
    """Prefill routing into caller-owned ``out_idx``/``out_bias`` [total_q, slots].
    ``page_domain`` (extension: a ``pages.PageDomain`` of the page state's
    bounds, e.g. ``PageIsolationState.candidate_domain``) replaces the dense
    ``image_allow``.  Returns (M, None, 0): the slot width, no diagnostic score
    chunk."""
    total_q = int(idx_q.shape[0])
    W = min(int(max_block), int(block_table.shape[1]))
    M = _out_slots(out_idx, topm, out_slots)
    K = max(1, min(int(budget or M), M))
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    seqs = ops.Seqs(n_seq=int(seq_lens.shape[0]), q_start=cu_seqlens_q.to(torch.int32),
                    pos0=context_lens.to(torch.int32), kv_len_t=seq_lens.to(torch.int32),
                    total_rows=total_q, max_q_len=total_q)
    cand = None if image_allow is None else image_allow[:total_q]
    ops.route(seqs, width=W, block_size=block_size, local_blocks=local_blocks,
              idx_scale=idx_scale, prior_floor=prior_floor, sigma=sigma, topm=int(topm), K=K,
              idx_q=idx_q, kbar=k_bar, block_table=bt, cand=cand,
              out_idx=out_idx[:total_q], out_bias=out_bias[:total_q], out_width=M,
              page=page_domain)
    return M, None, 0


@torch.no_grad()
def route_decode_triton(*, idx_q, k_bar, block_table, seq_lens, image_allow, out_idx, out_bias,
                        max_block: int, block_size: int, local_blocks: int,
                        decode_query_len: int, idx_scale: float, prior_floor: float,
                        sigma: float, topm: int, score_buf=None, budget=None, out_slots=None,
                        entmax_base=None, entmax_fit=None, entmax_width: int = 0,
                        score_buf_win=None, bounds=None, page_domain=None):
    """Decode routing for ``nd = R * decode_query_len`` rows (the last
    ``decode_query_len`` tokens of each request).  The window-narrowing
    arguments of the reference are accepted; the fused kernel scans all
    ``max_block`` columns of a row in one pass.  ``page_domain`` as in
    ``route_prefill_triton``.  Returns the slot width M."""
    nd = int(idx_q.shape[0])
    dql = max(1, int(decode_query_len))
    W = min(int(max_block), int(block_table.shape[1]))
    M = _out_slots(out_idx, topm, out_slots)
    K = max(1, min(int(budget or M), M))
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    R = nd // dql
    seqs = ops.Seqs(n_seq=R, q_len=dql, kv_len=0, kv_len_t=seq_lens[:R].to(torch.int32),
                    max_q_len=dql)
    cand = None if image_allow is None else image_allow[:nd]
    ops.route(seqs, width=W, block_size=block_size, local_blocks=local_blocks,
              idx_scale=idx_scale, prior_floor=prior_floor, sigma=sigma, topm=int(topm), K=K,
              idx_q=idx_q, kbar=k_bar, block_table=bt, cand=cand,
              out_idx=out_idx[:nd], out_bias=out_bias[:nd], out_width=M, page=page_domain)
    return M
