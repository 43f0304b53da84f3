"""Drop-in for ANANTA_OCR ``sparse_gather_triton.py`` (forward only).

* ``triton_gather_attention`` (sparse_gather_triton.py:343-392): gather
  attention without bias, ``HI`` index heads ([B,HI,T,S] routes, query head hq
  reads index head hq // (HQ // HI)), sequence packing through a per-token
  segment start ``arange(T) - position_ids``.
* ``triton_block_max_score`` (sparse_gather_triton.py:431-467): indexer
  stage-0 block max of q.k over non-local, causal, same-segment keys (-inf when
  a block has none).
Both run on libdash_b200.so; shapes the reference declines return None.
"""
from __future__ import annotations

import torch

from . import ops
from .sparse_gather_e2e_triton import _as_kernel_dtype

SPARSE_BLOCK_SIZE_SENTINEL = 128


def triton_gather_attention(query_states, key_states, value_states, block_indices, position_ids,
                            attention_mask, block_size, scale, local_window=None):
    if attention_mask is not None:
        return None
    B, HQ, T, D = query_states.shape
    HI = block_indices.shape[1]
    Hkv = key_states.shape[1]
    if HI < 1 or HQ % HI != 0 or Hkv % HI != 0:
        return None
    if key_states.shape[2] != T:
        return None
    if position_ids is None or position_ids.dim() != 2 or position_ids.shape[-1] != T:
        return None
    if D != 128:
        raise NotImplementedError(f"head_dim {D} not supported (B200 kernel: 128)")
    if torch.is_grad_enabled() and any(
            t.requires_grad for t in (query_states, key_states, value_states)):
        raise NotImplementedError("backward is not implemented by the B200 DASH kernels")
    ar = torch.arange(T, device=position_ids.device)
    seg = (ar[None, :] - position_ids).to(torch.int32).contiguous()
    lw = int(block_size) if local_window is None else max(1, int(local_window))
    dt = query_states.dtype
    q = _as_kernel_dtype(query_states)
    k = _as_kernel_dtype(key_states).to(q.dtype)
    v = _as_kernel_dtype(value_states).to(q.dtype)
    out = ops.gather_attention(q, k, v, block_indices, None, block_size=int(block_size),
                               local_window=lw, scale=float(scale), seg_start=seg,
                               n_index_heads=HI)
    return out if out.dtype == dt else out.to(dt)


def triton_block_max_score(q, k, pos, seg, block_size, num_key_blocks, local_window=None):
    """q [B,C,D], k [B,Sk,D], pos/seg [B,C] -> [B,C,num_key_blocks] fp32."""
    assert q.dim() == 3 and k.dim() == 3, "expects [B, C, D] / [B, Sk, D]"
    if q.shape[-1] > 256:
        raise NotImplementedError(f"index dim D={q.shape[-1]} > 256 not supported")
    lw = int(block_size) if local_window is None else max(1, int(local_window))
    return ops.block_max(q, k, pos, seg, int(block_size), int(num_key_blocks), lw,
                         clamp=False, empty=float("-inf"))
