"""Serving-side attention front end, backed by libdash_b200.so.

``index_qk_fused`` is the index branch of WHL unlimited_ocr_v2.py:145-162
(``index_q_proj`` / ``index_k_proj`` + ``GemmaRMSNorm`` x2 +
``apply_page2d_rope_pair`` on the index cos/sin table) followed by the index-K
store of WHL memory_pool.py:5573-5591 (``set_index_k_buffer``), as one tcgen05
kernel: the GEMM accumulates in TMEM and the epilogue normalises, rotates and
writes idx_q (fp32, the router's input) and idx_k straight into the paged index
cache at ``slot_mapping``.  On a decode step (one token per request) the same
kernel also refreshes the k-bar summary of each token's page after the write
(``kbar_refresh=``, replacing ``route_triton.kbar_refresh_tail_triton``); a
prefill step keeps the separate refresh, since there a page's tokens can be
written by different CTAs of the kernel.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops


@torch.no_grad()
def index_qk_fused(hidden_states: torch.Tensor, index_q_weight: torch.Tensor,
                   index_k_weight: torch.Tensor, q_norm_weight: torch.Tensor,
                   k_norm_weight: torch.Tensor, eps: float, cos: Optional[torch.Tensor] = None,
                   sin: Optional[torch.Tensor] = None, *, index_cache: Optional[torch.Tensor] = None,
                   slot_mapping: Optional[torch.Tensor] = None, idx_q_out=None,
                   kbar_refresh=None):
    """Returns (idx_q [T, 128] fp32, idx_k).  With ``index_cache`` ([pages,
    page_size, 128] or [slots, 128], fp32 or bf16) and ``slot_mapping``, idx_k
    is written into the cache rows and the cache is returned.
    ``kbar_refresh`` = (k_bar [P, 128], plan, head_cls, block_size) with the
    decode tail plan of ``route_triton.kbar_tail_plan`` (one page per token)
    refreshes those pages' k-bar in the same kernel."""
    T = hidden_states.shape[0]
    kout = None
    if index_cache is not None:
        kout = index_cache.view(-1, index_cache.shape[-1])
    kr = None
    if kbar_refresh is not None:
        kbar, (pages, ntok), head_cls, block_size = kbar_refresh
        assert pages.shape[0] == T, "the fused refresh takes one planned page per token"
        kr = (kbar, pages, ntok, head_cls, block_size)
    q, k = ops.index_proj(hidden_states.reshape(T, -1), index_q_weight, index_k_weight,
                          q_norm_weight, k_norm_weight, eps, cos=cos, sin=sin, norm_clamp=False,
                          idx_q=idx_q_out, idx_k=kout, slot_mapping=slot_mapping,
                          kbar_refresh=kr)
    return q, (index_cache if index_cache is not None else k)


@torch.no_grad()
def apply_page2d_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                      head_dim: int) -> torch.Tensor:
    """WHL page2d_rope.py:192-223: NeoX (rotate-half) RoPE of [T, H * head_dim]
    bf16 with every product and the sum rounded to bf16."""
    out, _ = ops.rope_kv_write(x, None, cos, sin, head_dim=head_dim)
    return out


@torch.no_grad()
def apply_page2d_rope_pair(x: torch.Tensor, y: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor, head_dim: int):
    """WHL page2d_rope.py:301-323: both tensors in one launch."""
    return ops.rope_kv_write(x, y, cos, sin, head_dim=head_dim)


@torch.no_grad()
def rope_and_store_kv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor,
                      sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, head_dim: int = 128) -> torch.Tensor:
    """``apply_page2d_rope_pair(q, k)`` (main branch, WHL unlimited_ocr_v2.py:156-158)
    followed by ``set_kv_buffer(loc, k, v)`` (WHL memory_pool.py:5524-5545) in one
    pass: q is rotated in place, rotated k and v land in the cache rows.
    Returns q."""
    ops.rope_kv_write(q, k, cos, sin, v=v, q_out=q, k_cache=k_cache, v_cache=v_cache,
                      slot_mapping=slot_mapping, head_dim=head_dim)
    return q
