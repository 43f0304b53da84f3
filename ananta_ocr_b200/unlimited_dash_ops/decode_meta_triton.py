"""Drop-in for the page part of the sglang backend's fused one-token decode
metadata (WHL .../unlimited_dash_ops/decode_meta_triton.py), backed by
libdash_b200.so.

``decode_meta_fused`` runs the page bookkeeping of one decode token per request
(``dash_page_state_step`` without a token layout: request r owns token r at
position seq_lens[r] - 1) and, with a ``coord_state`` (``page2d_rope.
PageCoordState``), the Page2D coordinates of those tokens
(``dash_page_coords``); ``cos_sin_2d_fused`` writes their cos/sin table
(``dash_cos_sin_2d``); ``decode_allow_fused`` builds the candidate mask from
the per-block page bounds the page step maintains (``dash_page_allow``).
"""
from __future__ import annotations

import torch

from .. import pages
from .page_state import _MM_PAD_SHIFT_VALUE, _i32, _i64


@torch.no_grad()
def decode_meta_fused(*, input_ids, block_table, seq_lens, slot_mapping, page_state,
                      coord_state=None, num_slots: int, block_size: int, out_q_page=None,
                      out_tok=None, out_page=None):
    """decode_meta_triton.py:247-315: returns (q_page int32 [R], (tok_pos,
    page_pos) int64 [R]) -- the coordinates are None without a coord_state."""
    R = int(seq_lens.shape[0])
    device = input_ids.device
    page_state._ensure(num_slots, device)
    q_page = out_q_page[:R] if out_q_page is not None and out_q_page.shape[0] >= R else \
        torch.empty(R, dtype=torch.int32, device=device)
    pages.page_state_step(
        input_ids=_i64(input_ids[:R]), block_table=_i32(block_table),
        slot_mapping=_i64(slot_mapping[:R]), num_slots=num_slots, block_size=block_size,
        per_page=page_state.per_page_image_tokens, image_token_id=page_state.image_token_id,
        page_token_id=page_state.page_token_id, slots=page_state._slots, q_page=q_page,
        seq_lens=_i32(seq_lens), num_decode_tokens=R, num_reqs=R, num_tokens=R,
        bounds=(page_state._blk_lo, page_state._blk_hi), mm_pad_shift=_MM_PAD_SHIFT_VALUE)
    if coord_state is None:
        return q_page, None
    sl = seq_lens[:R].to(torch.int64)
    tok, page = coord_state.advance(input_ids=input_ids[:R], q_start=None, start_pos=sl - 1,
                                    row_key=block_table[:R, 0], num_decode_tokens=R,
                                    out_tok=out_tok, out_page=out_page)
    return q_page, (tok, page)


@torch.no_grad()
def cos_sin_2d_fused(*, rope, tok_pos, page_pos, dtype, out_cos, out_sin):
    """decode_meta_triton.py:354-389: the Page2D cos/sin table of the given
    coordinates into the caller's fixed buffers."""
    from .page2d_rope import cos_sin_table
    T = int(tok_pos.shape[0])
    return cos_sin_table(rope, tok_pos, page_pos, out_cos[:T], out_sin[:T])


@torch.no_grad()
def decode_allow_fused(*, block_table, page_state, q_page, seq_lens, max_block: int,
                       num_blocks: int, block_size: int, out=None) -> torch.Tensor:
    """decode_meta_triton.py:318-351: page-isolation candidate mask [R, max_block]
    int8 (1 = candidate): blocks before the live length holding the query's
    page, or every column when none does."""
    R = int(q_page.shape[0])
    bt = _i32(block_table)
    W = min(int(max_block), int(bt.shape[1]))
    if out is None or out.shape[0] < R or out.shape[1] < max_block:
        out = torch.zeros(R, max_block, dtype=torch.int8, device=q_page.device)
    view = out[:R, :max_block]
    nb = min(num_blocks, page_state._blk_lo.numel())
    pages.page_allow(q_page, page_state._blk_lo[:nb], page_state._blk_hi[:nb], width=max_block,
                     rows=R, rows_per_seq=1, block_table=bt, desc_width=W,
                     seq_lens=_i32(seq_lens), block_size=block_size, fallback=True, out=view)
    return view


@torch.no_grad()
def local_union_fused(*, allow, seq_lens, out, max_block: int, block_size: int,
                      local_blocks: int) -> torch.Tensor:
    """decode_meta_triton.py:392-425: ``allow`` | the local window blocks
    [clamp(q_blk - local_blocks + 1), clamp(q_blk)] written as int8 into
    ``out``.  (The router's candidates are remote blocks only, so the union
    never changes a route; it is kept for callers that read the mask.)"""
    R = int(seq_lens.shape[0])
    q_blk = (seq_lens[:R].to(torch.int64) - 1) // block_size
    hi = q_blk.clamp(0, max_block - 1)
    lo = (q_blk - (local_blocks - 1)).clamp(0, max_block - 1)
    w = torch.arange(max_block, device=allow.device)
    a = torch.zeros(R, max_block, dtype=torch.bool, device=allow.device)
    n = min(max_block, allow.shape[1])
    a[:, :n] = allow[:R, :n] != 0
    win = (w[None, :] >= lo[:, None]) & (w[None, :] <= hi[:, None])
    n_o = min(max_block, out.shape[1])
    out[:R, :n_o] = (a | win)[:, :n_o].to(out.dtype)
    return out
