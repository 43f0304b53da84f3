"""Drop-in for ANANTA_OCR ``sparse_gather_triton.py``.

* ``triton_gather_attention`` (sparse_gather_triton.py:343-392): gather
  attention without bias, ``HI`` index heads ([B,HI,T,S] routes, query head hq
  reads index head hq // (HQ // HI)), sequence packing through a per-token
  segment start ``arange(T) - position_ids``.  With inputs that require grad
  it runs through ``_TritonGatherAttnFn`` (sparse_gather_triton.py:320-340):
  the tcgen05 forward keeps the log-sum-exp and the backward is
  ``dash_attn_bwd`` (tensor cores; fp32 inputs are computed in bf16, as the
  forward already does).
* ``triton_block_max_score`` (sparse_gather_triton.py:431-467): indexer
  stage-0 block max of q.k over non-local, causal, same-segment keys (-inf when
  a block has none).
Both run on libdash_b200.so; shapes the reference declines return None.
"""
from __future__ import annotations

import torch

from . import ops
from .sparse_gather_e2e_triton import _as_kernel_dtype, _as_tc_dtype

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
    ar = torch.arange(T, device=position_ids.device)
    seg = (ar[None, :] - position_ids).to(torch.int32).contiguous()
    lw = int(block_size) if local_window is None else max(1, int(local_window))
    if torch.is_grad_enabled() and any(
            t.requires_grad for t in (query_states, key_states, value_states)):
        return _TritonGatherAttnFn.apply(query_states, key_states, value_states, block_indices,
                                         seg, int(block_size), float(scale), lw)
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


class _TritonGatherAttnFn(torch.autograd.Function):
    """sparse_gather_triton.py:320-340.  Layouts here are the public ones
    ([B, heads, T, D]); the backward kernel takes [B, T, heads, D]."""

    @staticmethod
    def forward(ctx, q, k, v, sel, seg, block_size, scale, local_window):
        dt = q.dtype
        # the backward for several index heads / packed segments runs on tensor
        # cores only: fp32 inputs compute forward and backward in bf16 here
        qk = _as_tc_dtype(q)
        B, HQ, T, _ = q.shape
        HI = sel.shape[1]
        lse = torch.empty(B, HQ, T, dtype=torch.float32, device=q.device)
        o = ops.gather_attention(qk, _as_tc_dtype(k).to(qk.dtype), _as_tc_dtype(v).to(qk.dtype),
                                 sel, None, block_size=block_size, local_window=local_window,
                                 scale=scale, seg_start=seg, n_index_heads=HI, lse=lse)
        ctx.save_for_backward(q, k, v, sel, seg, o, lse)
        ctx.cfg = (block_size, scale, local_window)
        return o if o.dtype == dt else o.to(dt)

    @staticmethod
    def backward(ctx, do):
        q, k, v, sel, seg, o, lse = ctx.saved_tensors
        block_size, scale, local_window = ctx.cfg
        dt = o.dtype                                   # the kernel dtype (bf16 / fp16)
        tr = lambda t: t.transpose(1, 2).to(dt).contiguous()      # noqa: E731
        dq, dk, dv, _ = ops.gather_attention_bwd(
            tr(q), tr(k), tr(v), tr(o), tr(do), lse.transpose(1, 2), sel, None,
            block_size=block_size, local_window=local_window, scale=scale, want_d_bias=False,
            seg_start=seg)
        back = lambda g, like: g.transpose(1, 2).to(like.dtype)   # noqa: E731
        return back(dq, q), back(dk, k), back(dv, v), None, None, None, None, None
