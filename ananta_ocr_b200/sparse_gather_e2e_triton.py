"""Drop-in for ANANTA_OCR ``sparse_gather_e2e_triton.py``.

``triton_gather_attention_e2e`` keeps the reference's name, signature, tensor
layouts and "return None on unsupported shape" contract
(sparse_gather_e2e_triton.py:342-391), but runs the B200 kernels of
``libdash_b200.so`` instead of Triton kernels: the tcgen05 forward
(``dash_prefill_attn``, with the log-sum-exp saved) and, when autograd asks
for it, the CUDA-core backward (``dash_attn_bwd``: dq, dk, dv and the slot
bias gradient, sparse_gather_e2e_triton.py:118-262 and the
``_E2EGatherAttnFn.backward`` at :319-337).  Semantics
(sparse_gather_e2e_triton.py:34-115): per query token t and head, keys in the
routed blocks strictly below the local window get the slot's additive bias,
keys in the window (t-LW, t] get none, everything is causal.  Later duplicate
ids of a row are ignored (their slots get no gradient).
"""
from __future__ import annotations

import torch

from . import ops

SPARSE_E2E_SENTINEL = 1


def _as_kernel_dtype(t: torch.Tensor) -> torch.Tensor:
    # bf16/fp16 run on the tensor-core kernel (fp32 accumulation), fp32 on the
    # fp32 CUDA-core kernel (every product and sum fp32); others compute in fp32
    return t if t.dtype in (torch.bfloat16, torch.float16, torch.float32) else t.to(torch.float32)


def _as_tc_dtype(t: torch.Tensor) -> torch.Tensor:
    # tensor-core dtype (bf16 unless fp16), for paths that have no fp32 kernel
    return t if t.dtype in (torch.bfloat16, torch.float16) else t.to(torch.bfloat16)


def triton_gather_attention_e2e(query_states, key_states, value_states, block_indices,
                                blk_bias_slots, position_ids, attention_mask, block_size, scale,
                                local_window=None):
    """Fused e2e gather attention.  query_states [B,HQ,T,D], key/value [B,Hkv,T,D],
    block_indices [B,1,T,K] int (-1 pad), blk_bias_slots [B,T,K] fp32,
    position_ids [B,T] (must be arange).  Returns [B,HQ,T,D] or None when the
    reference would also decline (mask present, q_len != k_len, non-arange
    positions, more than one index head)."""
    if attention_mask is not None:
        return None
    if block_indices.shape[1] != 1:
        return None
    B, HQ, T, D = query_states.shape
    if key_states.shape[2] != T:
        return None
    if position_ids is None or position_ids.dim() != 2 or position_ids.shape[-1] != T:
        return None
    ar = torch.arange(T, device=position_ids.device)
    if not bool((position_ids == ar).all()):
        return None
    if D != 128 or value_states.shape[-1] != 128:
        raise NotImplementedError(f"head_dim {D} not supported (B200 kernel: 128)")
    lw = int(block_size) if local_window is None else max(1, int(local_window))
    if torch.is_grad_enabled() and any(
            t.requires_grad for t in (query_states, key_states, value_states, blk_bias_slots)):
        return _E2EGatherAttnFn.apply(query_states, key_states, value_states,
                                      block_indices[:, 0], blk_bias_slots, int(block_size),
                                      float(scale), lw)
    dt = query_states.dtype
    q = _as_kernel_dtype(query_states)
    k = _as_kernel_dtype(key_states).to(q.dtype)
    v = _as_kernel_dtype(value_states).to(q.dtype)
    out = ops.gather_attention(q, k, v, block_indices, blk_bias_slots[:, None],
                               block_size=int(block_size), local_window=lw, scale=float(scale))
    return out if out.dtype == dt else out.to(dt)


class _E2EGatherAttnFn(torch.autograd.Function):
    """sparse_gather_e2e_triton.py:265-337.  Layouts here are the public ones
    ([B, heads, T, D]); the backward kernel takes [B, T, heads, D]."""

    @staticmethod
    def forward(ctx, q, k, v, sel, bias_slots, block_size, scale, local_window):
        dt = q.dtype
        qk = _as_kernel_dtype(q)
        B, HQ, T, _ = q.shape
        lse = torch.empty(B, HQ, T, dtype=torch.float32, device=q.device)
        o = ops.gather_attention(qk, _as_kernel_dtype(k).to(qk.dtype), _as_kernel_dtype(v).to(qk.dtype),
                                 sel[:, None], bias_slots.detach()[:, None], block_size=block_size,
                                 local_window=local_window, scale=scale, lse=lse)
        o = o if o.dtype == dt else o.to(dt)
        ctx.save_for_backward(q, k, v, sel, bias_slots, o, lse)
        ctx.cfg = (block_size, scale, local_window)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, sel, bias_slots, o, lse = ctx.saved_tensors
        block_size, scale, local_window = ctx.cfg
        dt = q.dtype if q.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
        tr = lambda t: t.transpose(1, 2).to(dt).contiguous()      # noqa: E731
        dq, dk, dv, d_bias = ops.gather_attention_bwd(
            tr(q), tr(k), tr(v), tr(o), tr(do), lse.transpose(1, 2), sel, bias_slots.detach(),
            block_size=block_size, local_window=local_window, scale=scale,
            want_d_bias=ctx.needs_input_grad[4])
        back = lambda g, like: g.transpose(1, 2).to(like.dtype)   # noqa: E731
        return (back(dq, q), back(dk, k), back(dv, v), None,
                None if d_bias is None else d_bias.to(bias_slots.dtype), None, None, None)
