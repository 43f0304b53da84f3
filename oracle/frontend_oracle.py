"""torch restatement of the router front end (index projections + RMSNorm +
RoPE), the floating-point reference of ``dash_index_proj``.

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` and the CPU leg of
``bench.py``, never by the product package.  The same bf16/fp32 torch
operations as the reference, in the reference's order, so on the CPU it
reproduces the reference's outputs (pinned by tests/golden/frontend.npz) and on
a GPU it gives the cuBLAS-based result the kernel is compared with.
"""
from __future__ import annotations

import torch

ACT_CLAMP = 1.0e4   # dash_attention.py:604


def rmsnorm_clamp(x, w, eps):
    """dash_attention.py:680-693 (_RMSNorm.forward)."""
    x32 = torch.nan_to_num(x.float(), nan=0.0, posinf=0.0, neginf=0.0)
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    x32 = x32.clamp(-ACT_CLAMP, ACT_CLAMP)
    return (x32 * (1.0 + w.float())).clamp(-ACT_CLAMP, ACT_CLAMP).to(x.dtype)


def rmsnorm_gemma(x, w, eps):
    """WHL layernorm.py:1126-1130 (GemmaRMSNorm.forward_native)."""
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return (x32 * (1.0 + w.float())).to(x.dtype)


def rope(x, cos, sin):
    """Rotate-half RoPE in the tensors' dtype (transformers' apply_rotary_pos_emb,
    WHL page2d_rope.py:130-141)."""
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), dim=-1)
    return x * cos + rot * sin


def router_qk(hidden, wq, wk, nq, nk, eps, cos=None, sin=None):
    """modeling_deepseekv2.py:336-348 for [T, Hd] hidden: (idx_q, idx_k) fp32."""
    hs = torch.nan_to_num(hidden, nan=0.0, posinf=0.0, neginf=0.0)
    q = rmsnorm_clamp(torch.nn.functional.linear(hs, wq), nq, eps)
    k = rmsnorm_clamp(torch.nn.functional.linear(hs, wk), nk, eps)
    if cos is not None:
        q, k = rope(q, cos, sin), rope(k, cos, sin)
    q = torch.nan_to_num(q.float(), nan=0.0, posinf=0.0, neginf=0.0)
    k = torch.nan_to_num(k.float(), nan=0.0, posinf=0.0, neginf=0.0)
    return q, k


def index_qk(hidden, wq, wk, nq, nk, eps, cos=None, sin=None):
    """WHL unlimited_ocr_v2.py:145-162, index branch: (idx_q, idx_k) as fp32
    values of the bf16 results."""
    q = rmsnorm_gemma(torch.nn.functional.linear(hidden, wq), nq, eps)
    k = rmsnorm_gemma(torch.nn.functional.linear(hidden, wk), nk, eps)
    if cos is not None:
        q, k = rope(q, cos, sin), rope(k, cos, sin)
    return q.float(), k.float()


def rope_rows(x, cos, sin, head_dim=128):
    """WHL page2d_rope.py:130-141 (_rope2d_torch): [T, H * head_dim] rows."""
    T = x.shape[0]
    v = x.view(T, -1, head_dim)
    return rope(v, cos[:, None, :], sin[:, None, :]).view_as(x)
