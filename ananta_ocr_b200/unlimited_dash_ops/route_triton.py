"""Drop-in for the serving path's ``unlimited_dash_ops/route_triton.py``
(WHL sglang/srt/layers/attention/unlimited_dash_ops/route_triton.py).

Same entry points, keyword arguments and caller-owned output buffers; the
routing runs on libdash_b200.so.  Selection semantics follow the torch router
of the same package (dash_router.py:131-174, DashRouterMath.route_and_select):
top-``budget`` blocks by score (ties to the lowest id), entmax prior over the
top-``topm`` candidates, centred log-prior bias; ids packed ascending with -1 /
0.0 in unused slots.  The planning helpers (``kbar_tail_plan``,
``kbar_all_plan``, ``prefill_row2req``) keep the reference's names and
results (route_triton.py:576-620, 682-703) and run as one library kernel
(``dash_serving_plan``) with the sizes given by the caller, so they need no
host sync.
"""
from __future__ import annotations

import torch

from .. import _lib as L
from .. import ops

SCORE_NEG = -1.0e9
ENTMAX_NEG = -1.0e4
ACT_CLAMP = 1.0e4
SCAN_TILE = 128


def _plan_buffers(n_entries, device, out):
    if out is not None and out[0].shape[0] >= n_entries and out[1].shape[0] >= n_entries:
        return out[0][:n_entries], out[1][:n_entries]
    return (torch.empty(n_entries, dtype=torch.int64, device=device),
            torch.empty(n_entries, dtype=torch.int32, device=device))


def _i32(t, device):
    return t.to(device=device, dtype=torch.int32).contiguous()


def _serving_plan(*, block_table, seq_lens, block_size, width, mode, bt_width, context_lens=None,
                  pages=None, ntok=None, cu_seqlens_q=None, row2req=None):
    """One ``dash_serving_plan`` launch on the current stream."""
    device = seq_lens.device
    a = L.DashServingPlanArgs()
    keep = []
    if pages is not None:
        bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
        if bt.stride(-1) != 1:
            bt = bt.contiguous()
        keep.append(bt)
        a.block_table, a.bt_stride = bt.data_ptr(), bt.stride(0)
        a.pages, a.ntok = pages.data_ptr(), ntok.data_ptr()
    sl = _i32(seq_lens, device)
    keep.append(sl)
    a.seq_lens = sl.data_ptr()
    if context_lens is not None:
        ctx = _i32(context_lens, device)
        keep.append(ctx)
        a.context_lens = ctx.data_ptr()
    if row2req is not None:
        cu = _i32(cu_seqlens_q, device)
        keep.append(cu)
        a.cu_seqlens_q, a.row2req = cu.data_ptr(), row2req.data_ptr()
    a.n_req, a.block_size, a.width, a.mode = int(sl.shape[0]), int(block_size), int(width), int(mode)
    a.bt_width = int(bt_width)
    L.call("dash_serving_plan", a)
    del keep


@torch.no_grad()
def kbar_all_plan(*, block_table, seq_lens, context_lens, block_size: int, max_block: int,
                  max_query_len: int, device, out=None):
    """Pages a prefill step changed, per request: the block holding its first
    new token and the following ones up to the longest query span
    (route_triton.py:576-601), with their live token counts; one device launch.
    Returns flat (pages int64, ntok int32) of ``n_req * width`` entries."""
    bt_width = min(int(max_block), int(block_table.shape[1]))
    width = min(bt_width, -(-int(max_query_len) // int(block_size)) + 1)
    pages, ntok = _plan_buffers(int(seq_lens.shape[0]) * width, device, out)
    _serving_plan(block_table=block_table, seq_lens=seq_lens.to(device), block_size=block_size,
                  width=width, mode=0, bt_width=bt_width, context_lens=context_lens,
                  pages=pages, ntok=ntok)
    return pages, ntok


@torch.no_grad()
def prefill_row2req(*, cu_seqlens_q, device, out=None, total_q=None):
    """Request index of every query row (route_triton.py:605-620), filled on the
    device.  ``total_q`` (the row count) avoids reading ``cu_seqlens_q[-1]``
    back to the host; without it that one value is read."""
    cu = cu_seqlens_q.to(device)
    n = int(total_q) if total_q is not None else int(cu[-1])
    row2req = out[:n] if out is not None else torch.empty(n, dtype=torch.int32, device=device)
    _serving_plan(block_table=None, seq_lens=cu[1:] - cu[:-1], block_size=1, width=0, mode=1,
                  bt_width=1, cu_seqlens_q=cu, row2req=row2req)
    return row2req


@torch.no_grad()
def kbar_tail_plan(*, block_table, seq_lens, block_size: int, tail_pages: int, device, out=None):
    """The ``tail_pages`` newest blocks of every request (the ones a decode step
    can still change) and their live token counts (route_triton.py:682-703);
    one device launch.  Returns flat (pages int64, ntok int32)."""
    pages, ntok = _plan_buffers(int(seq_lens.shape[0]) * int(tail_pages), device, out)
    _serving_plan(block_table=block_table, seq_lens=seq_lens.to(device), block_size=block_size,
                  width=int(tail_pages), mode=1, bt_width=int(block_table.shape[1]),
                  pages=pages, ntok=ntok)
    return pages, ntok


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
                        score_buf_win=None, bounds=None, page_domain=None, refresh=None):
    """Decode routing for ``nd = R * decode_query_len`` rows (the last
    ``decode_query_len`` tokens of each request).  The window-narrowing
    arguments of the reference are accepted; the fused kernel scans all
    ``max_block`` columns of a row in one pass.  ``page_domain`` as in
    ``route_prefill_triton``.  ``refresh`` (extension): ``(kv_cache, head_cls,
    plan)`` as given to ``kbar_refresh_tail_triton``, whose refresh then runs
    inside this launch; the plan's pages must be tail pages inside every row's
    local window (``tail_pages <= local_blocks``).  Returns the slot width M."""
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
              out_idx=out_idx[:nd], out_bias=out_bias[:nd], out_width=M, page=page_domain,
              refresh=_refresh_args(refresh, block_size))
    return M


def _refresh_args(refresh, block_size):
    if refresh is None:
        return None
    kv_cache, head_cls, plan = refresh
    pages, tok = plan
    return kv_cache.view(kv_cache.shape[0], block_size, -1), pages, tok, head_cls
