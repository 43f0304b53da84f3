"""Drop-in for the serving path's ``unlimited_dash_ops/attend_triton.py``
(WHL sglang/srt/layers/attention/unlimited_dash_ops/attend_triton.py:523-715).

Same function names, arguments, tensor layouts and in-place output contract;
the work runs on libdash_b200.so (tcgen05 prefill, split-KV decode with fused
combine).  The module name is kept for drop-in imports; no Triton is used.

Layouts: q [total_q, H, D]; k/v cache [num_pages, page_size, Hkv, D]
(page_size == sparse block size); topk_idx / blk_bias [Hkv, total_q, topk]
(usually a stride-0 expansion of one router head); block_table
[num_reqs, max_blocks] int32.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib as L
from .. import ops

SPARSE_BLOCK_SIZE = 128
TARGET_GRID = 256


def _routes_from(topk_idx, blk_bias, num_kv_heads):
    idx = topk_idx if topk_idx.dtype == torch.int32 else topk_idx.to(torch.int32)
    if idx.stride(2) != 1:
        idx = idx.contiguous()
    nih = 1 if idx.stride(0) == 0 or idx.shape[0] == 1 else num_kv_heads
    bias = None
    if blk_bias is not None:
        assert blk_bias.shape == topk_idx.shape, (blk_bias.shape, topk_idx.shape)
        assert blk_bias.dtype == torch.float32, blk_bias.dtype
        bias = blk_bias
        if bias.stride(1) != idx.stride(1) or (nih > 1 and bias.stride(0) != idx.stride(0)):
            bias = bias.contiguous()
            idx = idx.contiguous()
    return ops._routes(idx, bias, idx.stride(1), idx.stride(0) if nih > 1 else 0, nih), idx, bias


def _paged_kv(k_cache, v_cache, block_table, num_kv_heads):
    if k_cache.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"KV cache dtype {k_cache.dtype} not supported (bf16/fp16)")
    return ops._kv(k_cache, v_cache, block_table, num_kv_heads,
                   (k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)))


@torch.no_grad()
def dash_sparse_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     topk_idx: torch.Tensor, blk_bias: Optional[torch.Tensor],
                     block_table: torch.Tensor, cu_seqlens_q: torch.Tensor, seq_lens: torch.Tensor,
                     prefix_lens: torch.Tensor, max_query_len: int, num_kv_heads: int,
                     sm_scale: float, output: torch.Tensor, local_blocks: int = 0,
                     sparse_block_size: int = SPARSE_BLOCK_SIZE,
                     device_error: Optional["ops.DeviceErrorWord"] = None) -> None:
    """Bias-aware block-sparse prefill attention over the paged cache (in place).
    ``device_error`` (extension) receives the first out-of-range block or page
    id the kernels met (they skip it and carry on)."""
    ops._need_cuda(q, k_cache, topk_idx, block_table)
    total_q, H, D = q.shape
    batch = cu_seqlens_q.shape[0] - 1
    routes, idx_keep, bias_keep = _routes_from(topk_idx, blk_bias, num_kv_heads)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    seqs = ops.Seqs(n_seq=batch, q_start=cu_seqlens_q.to(torch.int32),
                    pos0=prefix_lens.to(torch.int32), kv_len_t=seq_lens.to(torch.int32),
                    total_rows=total_q, max_q_len=int(max_query_len))
    a = L.DashPrefillArgs()
    a.seqs = seqs.c()
    a.kv = _paged_kv(k_cache, v_cache, bt, num_kv_heads)
    a.routes = routes
    a.qo = ops._qo(q, output, (0, q.stride(0), q.stride(1)), (0, output.stride(0), output.stride(1)), H)
    a.scale, a.block_size = float(sm_scale), int(sparse_block_size)
    a.local_window = int(local_blocks) * int(sparse_block_size)
    a.device_error = device_error.ptr if device_error is not None else None
    keep = (seqs, idx_keep, bias_keep, bt)
    ops.prefill_attn(a, q.device)
    del keep


@torch.no_grad()
def dash_sparse_attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            topk_idx: torch.Tensor, blk_bias: Optional[torch.Tensor],
                            block_table: torch.Tensor, seq_lens: torch.Tensor, num_kv_heads: int,
                            sm_scale: float, output: torch.Tensor, decode_query_len: int,
                            local_blocks: int = 0, sparse_block_size: int = SPARSE_BLOCK_SIZE,
                            chunk_width: Optional[int] = None, cg_rows: Optional[int] = None,
                            num_splits: int = 0, workspace: Optional[torch.Tensor] = None,
                            device_error: Optional["ops.DeviceErrorWord"] = None) -> None:
    """Bias-aware block-sparse decode with split-KV and fused combine (in place).

    ``chunk_width``/``cg_rows`` are accepted for signature compatibility; the
    split count is chosen from the grid (``num_splits`` overrides it), the
    split scratch comes from ``workspace`` (or a grow-only cache), and
    ``device_error`` receives the first out-of-range block or page id."""
    ops._need_cuda(q, k_cache, topk_idx, block_table, seq_lens)
    total_q, H, D = q.shape
    dql = int(decode_query_len)
    R = seq_lens.shape[0]
    assert total_q == R * dql
    routes, idx_keep, bias_keep = _routes_from(topk_idx, blk_bias, num_kv_heads)
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    sl = seq_lens if seq_lens.dtype == torch.int32 else seq_lens.to(torch.int32)
    seqs = ops.Seqs(n_seq=R, q_len=dql, kv_len=0, kv_len_t=sl, max_q_len=dql)
    a = L.DashDecodeArgs()
    a.seqs = seqs.c()
    a.kv = _paged_kv(k_cache, v_cache, bt, num_kv_heads)
    a.routes = routes
    a.qo = ops._qo(q, output, (dql * q.stride(0), q.stride(0), q.stride(1)),
                   (dql * output.stride(0), output.stride(0), output.stride(1)), H)
    a.scale, a.block_size = float(sm_scale), int(sparse_block_size)
    a.local_window = int(local_blocks) * int(sparse_block_size)
    a.num_splits = int(num_splits)
    a.device_error = device_error.ptr if device_error is not None else None
    keep = (seqs, idx_keep, bias_keep, bt, sl)
    ops.decode_attn(a, q.device, workspace)
    del keep
