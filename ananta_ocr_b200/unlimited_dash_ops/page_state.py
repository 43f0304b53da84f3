"""Drop-in for the sglang backend's page-isolation state
(WHL sglang/srt/layers/attention/unlimited_dash_ops/page_state.py), backed by
libdash_b200.so.

Per physical KV slot the state keeps the token's image page, marker count,
image run and prompt pages, so page ids survive across prefill chunks and
decode steps.  ``PageIsolationState.step`` is one kernel launch
(``dash_page_state_step``: one CTA per request, segmented scans with the carry
read from the slot of the previous token, slot writes, stale-tail clearing)
that also refreshes the [min, max] image page of every physical block it wrote,
so the router can test candidacy from those bounds and the query page without a
dense [tokens, max_block] mask (``candidate_domain``).  ``build_query_allow``
still returns the reference's dense mask.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .. import pages

_INT16_MAX = 32767

# Multimodal placeholders are rewritten above this value; text markers are not.
_MM_PAD_SHIFT_VALUE = 1_000_000


def image_token_mask(ids: torch.Tensor, image_token_id: int) -> torch.Tensor:
    """``True`` where a token is an image placeholder (sentinel or literal id)."""
    return (ids >= _MM_PAD_SHIFT_VALUE) | (ids == image_token_id)


@dataclass
class BatchLayout:
    """Per-step, per-request geometry (page_state.py:35-53)."""
    num_tokens: int
    num_reqs: int
    q_start: torch.Tensor          # [num_reqs + 1] int64
    start_pos: torch.Tensor        # [num_reqs] int64
    block_table: torch.Tensor      # [num_reqs, max_blocks]
    req_of_token: torch.Tensor     # [num_tokens] int64
    num_decode_tokens: int = 0
    gen_start: Optional[torch.Tensor] = None


def _req_of_token(q_start: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Token -> request row (page_state.py:70-75)."""
    tok = torch.arange(num_tokens, device=q_start.device, dtype=torch.int64)
    return torch.searchsorted(q_start[1:].contiguous(), tok, right=True).clamp_(
        max=q_start.shape[0] - 2)


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 and t.is_contiguous() else t.to(torch.int32).contiguous()


def _i64(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int64 and t.is_contiguous() else t.to(torch.int64).contiguous()


class PageIsolationState:
    """Persistent per-slot page bookkeeping + per-query block allow masks."""

    def __init__(self, sparse_cfg: dict, block_size: int) -> None:
        self.block_size = int(block_size)
        self.image_token_id = int(sparse_cfg.get("image_token_id", 128815))
        pt = sparse_cfg.get("page_token_id", None)
        self.page_token_id = int(pt) if pt is not None else None
        self.per_page_image_tokens = max(1, int(sparse_cfg.get("per_page_image_tokens", 273)))
        self._slot_img_page: Optional[torch.Tensor] = None
        self._slot_marker_cum: Optional[torch.Tensor] = None
        self._slot_img_run: Optional[torch.Tensor] = None
        self._slot_prompt_pages: Optional[torch.Tensor] = None
        self._blk_lo: Optional[torch.Tensor] = None
        self._blk_hi: Optional[torch.Tensor] = None
        self._num_slots = 0
        self._last_img_run_max = None

    def _ensure(self, num_slots: int, device: torch.device) -> None:
        if self._slot_img_page is not None and self._num_slots >= num_slots:
            return
        self._slot_img_page = torch.full((num_slots,), -1, dtype=torch.int32, device=device)
        self._slot_marker_cum = torch.zeros(num_slots, dtype=torch.int32, device=device)
        self._slot_img_run = torch.zeros(num_slots, dtype=torch.int32, device=device)
        self._slot_prompt_pages = torch.zeros(num_slots, dtype=torch.int32, device=device)
        nb = max(1, num_slots // self.block_size)
        self._blk_lo = torch.full((nb,), -1, dtype=torch.int32, device=device)
        self._blk_hi = torch.full((nb,), -1, dtype=torch.int32, device=device)
        self._num_slots = num_slots

    @property
    def _slots(self):
        return (self._slot_img_page, self._slot_marker_cum, self._slot_img_run,
                self._slot_prompt_pages)

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor, layout: BatchLayout, slot_mapping: torch.Tensor,
             num_slots: int) -> torch.Tensor:
        """page_state.py:217-313: updates the per-slot state from this step's
        tokens; returns q_page [num_tokens] int32 (-1 = page unknown)."""
        self._ensure(num_slots, input_ids.device)
        T = layout.num_tokens
        q_page = torch.empty(T, dtype=torch.int32, device=input_ids.device)
        pages.page_state_step(
            input_ids=_i64(input_ids[:T]), block_table=_i32(layout.block_table),
            slot_mapping=_i64(slot_mapping[:T]), num_slots=num_slots,
            block_size=self.block_size, per_page=self.per_page_image_tokens,
            image_token_id=self.image_token_id, page_token_id=self.page_token_id,
            slots=self._slots, q_page=q_page, q_start=_i64(layout.q_start),
            start_pos=_i64(layout.start_pos),
            gen_start=None if layout.gen_start is None else _i64(layout.gen_start),
            num_decode_tokens=int(layout.num_decode_tokens), num_reqs=layout.num_reqs,
            num_tokens=T, bounds=(self._blk_lo, self._blk_hi),
            mm_pad_shift=_MM_PAD_SHIFT_VALUE)
        return q_page

    def block_page_bounds(self, num_blocks: int):
        """page_state.py:315-328: per physical block (min, max) image page id
        (-1 == none), int16, recomputed from the slot pages."""
        bs = self.block_size
        lo, hi, _ = pages.page_blocks(self._slot_img_page[: num_blocks * bs].view(num_blocks, bs),
                                      1, bs, bits=False)
        return lo.view(-1).to(torch.int16), hi.view(-1).to(torch.int16)

    def candidate_domain(self, q_page: torch.Tensor):
        """Compact domain for ``ops.route`` on the paged cache (descriptors of
        physical blocks through the route's block table)."""
        return pages.PageDomain(q_page=_i32(q_page), lo=self._blk_lo, hi=self._blk_hi)

    @torch.no_grad()
    def build_query_allow(self, layout: BatchLayout, q_page: torch.Tensor, max_block: int,
                          num_blocks: int) -> torch.Tensor:
        """page_state.py:330-371: [num_tokens, max_block] bool, same page |
        open row."""
        bt = _i32(layout.block_table)
        nb = min(num_blocks, self._blk_lo.numel())
        return pages.page_allow(
            q_page, self._blk_lo[:nb], self._blk_hi[:nb], width=max_block,
            rows=layout.num_tokens, row_seq=_i32(layout.req_of_token), block_table=bt,
            desc_width=min(max_block, bt.shape[1]), fallback=True)
