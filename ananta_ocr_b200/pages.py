"""Tensor-level wrappers of the page-aware candidate kernels (``dash_page_*``,
``dash_block_any`` of libdash_b200.so).

An OCR document is a token sequence whose image placeholders carry the visual
tokens of each page, opened by ``<PAGE>`` markers.  The router restricts a query
token's remote candidates to the blocks holding image tokens of the query's own
page (falling back to every remote block when there is none).  These wrappers
produce that domain on the GPU in its compact form -- a query page per row and
one page descriptor (lo, hi, page bits) per key block -- which ``ops.route``
consumes directly (``page=PageDomain``), and, for API compatibility, the dense
masks the reference builds.  CUDA tensors only; every non-zero library status
raises.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L
from .ops import _need_cuda, _ptr


def _words(block_size: int) -> int:
    return max(1, block_size // 32)


def _call(fn, args):
    L.call(fn, args)


@dataclass
class PageDomain:
    """Compact candidate domain for ``ops.route``: ``q_page`` int32 [rows];
    per-block descriptors ``lo``/``hi`` int32 and optional ``bits`` (int32
    storage of uint32 words) addressed as ``seq * seq_rows + block``
    (contiguous) or by physical block through the route's block table."""
    q_page: torch.Tensor
    lo: torch.Tensor
    hi: torch.Tensor
    bits: Optional[torch.Tensor] = None
    seq_rows: int = 0

    @property
    def words(self) -> int:
        return 0 if self.bits is None else int(self.bits.shape[-1])


def page_ids(token_ids: torch.Tensor, *, image_token_id: int, page_token_id: Optional[int],
             per_page: int, key_length: int, rule: int = 0, page_scope_prefill: bool = False,
             mm_pad_shift: int = 0, block_size: int = 0, n_blocks: int = 0,
             token_outputs: bool = True, page_dtype=torch.int32, bits: bool = True,
             has_image: bool = False, want_image: bool = True):
    """One pass of ``dash_page_ids`` over token ids [B, >=0] (int64).

    Returns a dict: ``image_mask`` bool, ``image_page`` / ``query_page``
    (``page_dtype``) [B, key_length] when ``token_outputs`` (the first two
    only with ``want_image``); ``lo``/``hi``
    int32 [B, n_blocks], ``bits`` int32 [B, n_blocks, words] and ``has_image``
    bool [B, n_blocks] when ``block_size``; ``prompt_pages``, ``marker_count``,
    ``n_image``, ``n_query`` int32 [B]."""
    _need_cuda(token_ids)
    ids = token_ids if token_ids.dtype == torch.int64 else token_ids.to(torch.int64)
    if ids.dim() != 2:
        raise ValueError("token_ids must be [B, S]")
    if ids.stride(-1) != 1:
        ids = ids.contiguous()
    B = ids.shape[0]
    dev = ids.device
    out = {}
    a = L.DashPageIdsArgs()
    a.token_ids, a.ids_stride = ids.data_ptr(), ids.stride(0)
    a.n_seq, a.ids_len, a.key_length = B, min(ids.shape[1], key_length), key_length
    a.per_page = max(1, int(per_page))
    a.image_token_id = int(image_token_id)
    a.has_page_token = int(page_token_id is not None)
    a.page_token_id = int(page_token_id) if page_token_id is not None else -1
    a.mm_pad_shift = int(mm_pad_shift)
    a.rule, a.page_scope_prefill = int(rule), int(bool(page_scope_prefill))
    if token_outputs and page_dtype not in (torch.int32, torch.int64):
        raise ValueError("page_dtype must be int32 or int64")
    # every int32 output in one allocation: [query_page | image_page | lo | hi |
    # bits | per-row x4] (int64 pages get their own)
    w32 = page_dtype == torch.int32
    words = _words(block_size) if block_size else 0
    parts = []
    if token_outputs and rule == 0 and w32:
        parts.append(("query_page", (B, key_length)))
    if token_outputs and want_image and w32:
        parts.append(("image_page", (B, key_length)))
    if block_size:
        parts += [("lo", (B, n_blocks)), ("hi", (B, n_blocks))]
        if bits:
            parts.append(("bits", (B, n_blocks, words)))
    parts.append(("rows", (4, B)))
    n32 = sum(math.prod(sh) for _, sh in parts)
    buf = torch.empty(n32, dtype=torch.int32, device=dev)
    o = 0
    for name, sh in parts:
        n = math.prod(sh)
        out[name] = buf[o:o + n].view(sh)
        o += n
    if token_outputs:
        a.page_elem_bytes = 4 if w32 else 8
        if want_image:
            im = torch.empty(B, key_length, dtype=torch.bool, device=dev)
            if not w32:
                out["image_page"] = torch.empty(B, key_length, dtype=page_dtype, device=dev)
            a.image_mask, a.image_mask_stride = im.data_ptr(), key_length
            a.image_page, a.image_page_stride = out["image_page"].data_ptr(), key_length
            out["image_mask"] = im
        if rule == 0:
            if not w32:
                out["query_page"] = torch.empty(B, key_length, dtype=page_dtype, device=dev)
            a.query_page, a.query_page_stride = out["query_page"].data_ptr(), key_length
    if block_size:
        a.block_size, a.n_blocks = int(block_size), int(n_blocks)
        a.blk_lo, a.blk_hi = out["lo"].data_ptr(), out["hi"].data_ptr()
        if bits:
            a.blk_bits = out["bits"].data_ptr()
        if has_image:
            hb = torch.empty(B, n_blocks, dtype=torch.bool, device=dev)
            a.blk_has_image = hb.data_ptr()
            out["has_image"] = hb
    rows = out.pop("rows")
    a.prompt_pages, a.marker_count = rows[0].data_ptr(), rows[1].data_ptr()
    a.n_image, a.n_query = rows[2].data_ptr(), rows[3].data_ptr()
    out["prompt_pages"], out["marker_count"], out["n_image"], out["n_query"] = rows.unbind(0)
    _call("dash_page_ids", a)
    return out


def page_blocks(pages: torch.Tensor, num_blocks: int, block_size: int, *, length=None,
                bits: bool = True):
    """(lo, hi, bits) int32 descriptors of [rows, >= length] image page ids
    (int32/int64, -1 = none) cut into ``num_blocks`` blocks."""
    _need_cuda(pages)
    if pages.dtype not in (torch.int32, torch.int64):
        pages = pages.to(torch.int64)
    if pages.stride(-1) != 1:
        pages = pages.contiguous()
    R = pages.shape[0]
    dev = pages.device
    a = L.DashPageBlocksArgs()
    a.pages, a.stride, a.elem_bytes = pages.data_ptr(), pages.stride(0), pages.element_size()
    a.rows, a.len = R, int(pages.shape[1] if length is None else min(length, pages.shape[1]))
    a.block_size, a.n_blocks = int(block_size), int(num_blocks)
    lo = torch.empty(R, num_blocks, dtype=torch.int32, device=dev)
    hi = torch.empty(R, num_blocks, dtype=torch.int32, device=dev)
    bt = torch.empty(R, num_blocks, _words(block_size), dtype=torch.int32, device=dev) if bits else None
    a.lo, a.hi, a.bits = lo.data_ptr(), hi.data_ptr(), _ptr(bt)
    _call("dash_page_blocks", a)
    return lo, hi, bt


def page_allow(q_page: torch.Tensor, lo: torch.Tensor, hi: torch.Tensor, *, width: int,
               bits: Optional[torch.Tensor] = None, rows: Optional[int] = None,
               rows_per_seq: int = 1, row_seq: Optional[torch.Tensor] = None,
               desc_width: Optional[int] = None, block_table: Optional[torch.Tensor] = None,
               seq_lens: Optional[torch.Tensor] = None, block_size: int = 0,
               fallback: bool = True, q_pos: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, out_dtype=torch.bool):
    """Dense candidate mask [rows, width] from query pages and descriptors.

    Descriptors: ``block_table`` [n_seq, >= desc_width] int32 of physical
    blocks into ``lo``/``hi`` [num_blocks], or row-major [n_seq, seq_rows]
    ``lo``/``hi``.  ``q_pos`` [rows] int64: the query page of row r is
    ``q_page[seq, clamp(q_pos[r])]`` instead of ``q_page[r]``."""
    _need_cuda(q_page, lo, hi, bits, block_table, seq_lens, q_pos)
    if q_page.dtype not in (torch.int32, torch.int64):
        q_page = q_page.to(torch.int64)
    a = L.DashPageAllowArgs()
    if q_pos is not None:
        qpos = q_pos.reshape(-1).to(torch.int64).contiguous()
        R = qpos.numel() if rows is None else rows
        qsrc = q_page if q_page.stride(-1) == 1 else q_page.contiguous()
        a.q_pos, a.q_stride, a.q_len = qpos.data_ptr(), qsrc.stride(0), qsrc.shape[-1]
        q_page = qsrc
    else:
        q_page = q_page.reshape(-1).contiguous()
        R = q_page.numel() if rows is None else rows
    a.q_page, a.q_elem_bytes = q_page.data_ptr(), q_page.element_size()
    if out is None:
        out = torch.empty(R, width, dtype=out_dtype, device=q_page.device)
    a.rows, a.width = R, int(width)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.row_seq = _ptr(row_seq)
    a.rows_per_seq = int(rows_per_seq)
    lo_c, hi_c = lo.contiguous(), hi.contiguous()
    a.page_lo, a.page_hi = lo_c.data_ptr(), hi_c.data_ptr()
    if bits is not None:
        bits = bits.contiguous()
        a.page_bits, a.page_bits_words = bits.data_ptr(), bits.shape[-1]
    a.num_desc = lo_c.numel()
    if block_table is not None:
        a.block_table, a.bt_stride = block_table.data_ptr(), block_table.stride(0)
        a.desc_width = int(min(width, block_table.shape[1]) if desc_width is None else desc_width)
    else:
        a.desc_seq_rows = lo_c.shape[-1]
        a.desc_width = int(min(width, lo_c.shape[-1]) if desc_width is None else desc_width)
    a.seq_lens, a.block_size = _ptr(seq_lens), int(block_size)
    a.fallback = int(bool(fallback))
    _call("dash_page_allow", a)
    return out


def block_any(mask: torch.Tensor, num_blocks: int, block_size: int) -> torch.Tensor:
    """[rows, num_blocks] bool: any mask token in each block (padding False)."""
    _need_cuda(mask)
    m = mask if mask.dtype in (torch.bool, torch.uint8) else mask != 0
    if m.stride(-1) != 1:
        m = m.contiguous()
    out = torch.empty(m.shape[0], num_blocks, dtype=torch.bool, device=m.device)
    a = L.DashBlockAnyArgs()
    a.mask, a.mask_stride = m.data_ptr(), m.stride(0)
    a.rows, a.len, a.block_size, a.n_blocks = m.shape[0], m.shape[1], int(block_size), int(num_blocks)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    _call("dash_block_any", a)
    return out


def page_decode_query(last_ids: torch.Tensor, marker_count: torch.Tensor,
                      prompt_pages: torch.Tensor, page_token_id: Optional[int],
                      q_page: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode step of the contiguous decoder: marker_count += (last id is a
    page marker) in place; returns the query page int32 [B]."""
    _need_cuda(last_ids, marker_count, prompt_pages)
    ids = last_ids if last_ids.dtype == torch.int64 else last_ids.to(torch.int64)
    B = marker_count.shape[0]
    if q_page is None:
        q_page = torch.empty(B, dtype=torch.int32, device=marker_count.device)
    a = L.DashPageDecodeArgs()
    a.last_ids, a.ids_stride = ids.data_ptr(), ids.stride(0)
    a.n_seq = B
    a.has_page_token = int(page_token_id is not None)
    a.page_token_id = int(page_token_id) if page_token_id is not None else -1
    a.marker_count, a.prompt_pages, a.q_page = (marker_count.data_ptr(), prompt_pages.data_ptr(),
                                                q_page.data_ptr())
    _call("dash_page_decode_query", a)
    return q_page


def page_state_step(*, input_ids, block_table, slot_mapping, num_slots: int, block_size: int,
                    per_page: int, image_token_id: int, page_token_id: Optional[int],
                    slots, q_page, q_start=None, start_pos=None, seq_lens=None,
                    gen_start=None, num_decode_tokens: int = 0, num_reqs: int,
                    num_tokens: int, bounds=None, mm_pad_shift: int = 0):
    """One serving step of per-slot page bookkeeping (``dash_page_state_step``).

    ``slots`` = (img_page, marker_cum, img_run, prompt_pages) int32 [num_slots]
    state, updated in place; ``q_page`` int32 [num_tokens] output; ``bounds``
    = (lo, hi) int32 [num_slots // block_size] refreshed for written blocks."""
    _need_cuda(input_ids, block_table, slot_mapping, q_page)
    a = L.DashPageStateArgs()
    a.input_ids = input_ids.data_ptr()
    a.q_start, a.start_pos = _ptr(q_start), _ptr(start_pos)
    a.seq_lens, a.gen_start = _ptr(seq_lens), _ptr(gen_start)
    a.block_table, a.bt_stride, a.bt_width = (block_table.data_ptr(), block_table.stride(0),
                                              block_table.shape[1])
    a.slot_mapping, a.num_slots = slot_mapping.data_ptr(), int(num_slots)
    a.image_token_id = int(image_token_id)
    a.has_page_token = int(page_token_id is not None)
    a.page_token_id = int(page_token_id) if page_token_id is not None else -1
    a.mm_pad_shift = int(mm_pad_shift)
    a.num_tokens, a.num_reqs, a.num_decode_tokens = int(num_tokens), int(num_reqs), int(num_decode_tokens)
    a.block_size, a.per_page = int(block_size), max(1, int(per_page))
    a.slot_img_page, a.slot_marker_cum, a.slot_img_run, a.slot_prompt_pages = (
        s.data_ptr() for s in slots)
    a.q_page = q_page.data_ptr()
    if bounds is not None:
        a.blk_lo, a.blk_hi = bounds[0].data_ptr(), bounds[1].data_ptr()
    _call("dash_page_state_step", a)
    return q_page
