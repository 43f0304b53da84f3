"""Drop-in for the coordinate part of the serving path's Page2D rotary
(WHL sglang/srt/layers/attention/unlimited_dash_ops/page2d_rope.py).

``PageRope2D`` keeps the reference's frequency tables (token pairs first,
then page pairs, so ``rotate_half`` pairs them the same way) and builds the
cos/sin table on the library (``dash_cos_sin_2d``).  ``PageCoordState`` keeps
the per-request coordinate state (marker count, prompt pages, per-page token
counts) in device tensors and advances it with ``dash_page_coords`` (state
rows matched by the request's first physical KV block, reused least recently
used; one launch for the rows, one for the tokens).  The speculative-decoding
rewind of the reference is not reproduced: ``max_spec_slots`` is accepted and
ignored (the rewind only acts when a step re-submits positions a previous
step already committed).
"""
from __future__ import annotations

import math

import torch

from .. import _lib as L
from .page_state import _MM_PAD_SHIFT_VALUE

MIN_PAGE_TOKENS = 74


def page_capacity(context_len: int) -> int:
    """Page buckets for any prompt of ``context_len`` tokens (page2d_rope.py:23-29)."""
    return max(1, int(context_len)) // MIN_PAGE_TOKENS + 2


def _i64(t):
    return t if t.dtype == torch.int64 and t.is_contiguous() else t.to(torch.int64).contiguous()


class PageRope2D:
    """Frequency tables of the Page2D rotary (page2d_rope.py:32-127): ``dim/2 -
    page_pairs`` token pairs with base ``base_tok`` (``resample``: spread over
    the token pairs; ``truncate``: the 1-D rotary's first pairs), then
    ``page_pairs`` page pairs with base ``base_page``; ``page_mod`` folds the
    page axis."""

    def __init__(self, dim: int, base_tok: float, base_page: float, page_pairs: int,
                 tok_freq_mode: str = "resample", page_mod: int = 0) -> None:
        half = dim // 2
        page_pairs = int(page_pairs)
        if not 0 < page_pairs < half:
            raise ValueError(f"[PageRope2D] page_pairs={page_pairs} must be in (0, {half}); dim={dim}")
        n_tok = half - page_pairs
        k = torch.arange(0, n_tok, dtype=torch.int64).float()
        expo = k * 2 / dim if str(tok_freq_mode).lower() == "truncate" else k / n_tok
        self.inv_tok = 1.0 / (base_tok ** expo)
        self.inv_page = 1.0 / (base_page ** (torch.arange(0, page_pairs, dtype=torch.int64).float() / page_pairs))
        self.dim, self.n_tok, self.page_pairs = dim, n_tok, page_pairs
        self.base_tok, self.base_page = float(base_tok), float(base_page)
        self.tok_freq_mode = str(tok_freq_mode).lower()
        self.page_mod = int(page_mod or 0)
        self._dev_cache = {}

    def _freqs(self, device):
        got = self._dev_cache.get(device)
        if got is None:
            got = (self.inv_tok.to(device), self.inv_page.to(device))
            self._dev_cache[device] = got
        return got

    @property
    def signature(self) -> tuple:
        return (self.dim, self.n_tok, self.page_pairs, self.base_tok, self.base_page,
                self.tok_freq_mode, self.page_mod)

    @property
    def page_mono_range(self) -> float:
        if self.page_mod > 0:
            return float(self.page_mod)
        return self.base_page ** ((self.page_pairs - 1) / self.page_pairs) * math.pi

    @property
    def tok_mono_range(self) -> float:
        return math.pi / float(self.inv_tok[-1])

    @torch.no_grad()
    def cos_sin(self, tok_pos: torch.Tensor, page_pos: torch.Tensor, dtype: torch.dtype):
        """``tok_pos`` / ``page_pos`` [T] int -> cos/sin [T, dim] (fp32 angles)."""
        T = int(tok_pos.shape[0])
        out_dt = torch.bfloat16 if dtype == torch.bfloat16 else torch.float32
        cos = torch.empty(T, self.dim, dtype=out_dt, device=tok_pos.device)
        sin = torch.empty_like(cos)
        cos_sin_table(self, tok_pos, page_pos, cos, sin)
        return cos.to(dtype), sin.to(dtype)


@torch.no_grad()
def cos_sin_table(rope: PageRope2D, tok_pos, page_pos, out_cos, out_sin):
    """``dash_cos_sin_2d`` into caller buffers (fp32 or bf16, rows of ``dim``)."""
    T = int(tok_pos.shape[0])
    if T == 0:
        return out_cos[:0], out_sin[:0]
    inv_tok, inv_page = rope._freqs(tok_pos.device)
    tp, pp = _i64(tok_pos), _i64(page_pos)
    a = L.DashCosSin2DArgs()
    a.tok_pos, a.page_pos = tp.data_ptr(), pp.data_ptr()
    a.inv_tok, a.inv_page = inv_tok.data_ptr(), inv_page.data_ptr()
    assert out_cos.dtype in (torch.float32, torch.bfloat16) and out_sin.dtype == out_cos.dtype
    assert out_cos.stride(-1) == 1 and out_sin.stride() == out_cos.stride()
    a.cos, a.sin, a.stride = out_cos.data_ptr(), out_sin.data_ptr(), out_cos.stride(0)
    a.page_mod, a.num_tokens, a.dim, a.n_tok = rope.page_mod, T, rope.dim, rope.n_tok
    a.out_bf16 = int(out_cos.dtype == torch.bfloat16)
    L.call("dash_cos_sin_2d", a)
    del tp, pp
    return out_cos[:T], out_sin[:T]


class PageCoordState:
    """Streaming ``(tok_pos, page_pos)`` coordinates (page2d_rope.py:327-620)."""

    def __init__(self, sparse_cfg: dict, max_reqs: int, max_pages: int, max_spec_slots: int = 1):
        if max_pages <= 0:
            raise ValueError(f"max_pages must be positive, got {max_pages}")
        self.image_token_id = int(sparse_cfg.get("image_token_id", 128815))
        pt = sparse_cfg.get("page_token_id", None)
        self.page_token_id = int(pt) if pt is not None else None
        self.max_pages = int(max_pages)
        self.max_reqs = int(max_reqs)
        self.max_slots = max(1, int(max_spec_slots))
        self.key = self.stamp = self.st_marker = self.st_pp = self.cnt = None
        self._step_t = self._rows_buf = None

    def _ensure(self, device) -> None:
        if self.key is not None:
            return
        n = self.max_reqs
        self.key = torch.full((n,), -1, dtype=torch.int64, device=device)
        self.stamp = torch.zeros(n, dtype=torch.int64, device=device)
        self.st_marker = torch.zeros(n, dtype=torch.int32, device=device)
        self.st_pp = torch.zeros(n, dtype=torch.int32, device=device)
        self.cnt = torch.zeros(n, self.max_pages, dtype=torch.int32, device=device)
        self._step_t = torch.zeros(1, dtype=torch.int64, device=device)
        self._rows_buf = torch.empty(n, dtype=torch.int32, device=device)

    @torch.no_grad()
    def advance(self, *, input_ids, q_start, start_pos, row_key, num_decode_tokens: int,
                gen_start=None, out_tok=None, out_page=None):
        """One ``dash_page_coords`` call; returns (tok_pos, page_pos) int64 [T]."""
        device = input_ids.device
        self._ensure(device)
        R = int(row_key.shape[0])
        T = int(input_ids.shape[0])
        tok = out_tok[:T] if out_tok is not None and out_tok.shape[0] >= T else \
            torch.empty(T, dtype=torch.int64, device=device)
        page = out_page[:T] if out_page is not None and out_page.shape[0] >= T else \
            torch.empty(T, dtype=torch.int64, device=device)
        keep = [_i64(input_ids), None if q_start is None else _i64(q_start), _i64(start_pos),
                None if gen_start is None else _i64(gen_start), _i64(row_key)]
        ids, qs, sp, gs, rk = keep
        a = L.DashPageCoordArgs()
        a.input_ids, a.q_start, a.start_pos = ids.data_ptr(), None if qs is None else qs.data_ptr(), sp.data_ptr()
        a.gen_start, a.row_key = None if gs is None else gs.data_ptr(), rk.data_ptr()
        a.image_token_id = self.image_token_id
        a.page_token_id = self.page_token_id if self.page_token_id is not None else 0
        a.has_page_token = int(self.page_token_id is not None)
        a.mm_pad_shift = _MM_PAD_SHIFT_VALUE
        a.num_tokens, a.num_reqs, a.num_decode_tokens = T, R, int(num_decode_tokens)
        a.max_rows, a.max_pages = self.max_reqs, self.max_pages
        a.state_key, a.state_stamp, a.step = self.key.data_ptr(), self.stamp.data_ptr(), self._step_t.data_ptr()
        a.c_marker, a.c_pp, a.cnt = self.st_marker.data_ptr(), self.st_pp.data_ptr(), self.cnt.data_ptr()
        a.rows, a.tok_pos, a.page_pos = self._rows_buf.data_ptr(), tok.data_ptr(), page.data_ptr()
        L.call("dash_page_coords", a)
        del keep
        return tok, page

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor, layout):
        """Coordinates of this step's tokens (``layout``: page_state.BatchLayout)."""
        t = int(layout.num_tokens)
        if t <= 0:
            return None
        return self.advance(input_ids=input_ids[:t], q_start=layout.q_start,
                            start_pos=layout.start_pos, row_key=layout.block_table[:, 0],
                            num_decode_tokens=int(layout.num_decode_tokens),
                            gen_start=layout.gen_start)
