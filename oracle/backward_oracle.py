"""torch fp32 restatement of the DASH gather attention and of 1.5-entmax with
autograd: the reference for ``dash_attn_bwd`` and ``dash_entmax15_fwd/bwd``.

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` and the CPU leg of
``bench.py``, never by the product package.  The attention is the dense
masked form of dash_attention.py:980-1006 (``_forward_dense``) with the
routed lists of sparse_gather_e2e_triton.py:367-384 (later duplicates
dropped, slot biases scattered onto their blocks); its autograd gradients are
what sparse_gather_e2e_triton.py:118-262 computes blockwise.  Entmax follows
dash_attention.py:623-658 (sort-based threshold; the Jacobian of
``_Entmax15.backward``).  Pinned against the reference's own Triton backward
(interpreted on the CPU) in tests/golden/backward.npz.
"""
from __future__ import annotations

import torch


def kept_slots(idx: torch.Tensor, nblk: int, block_size: int, local_window: int) -> torch.Tensor:
    """[B, T, K] bool: slot holds the first occurrence of a block id in
    [0, nblk) that has a key below the row's local window."""
    B, T, K = idx.shape
    t = torch.arange(T, device=idx.device).view(1, T, 1)
    ok = (idx >= 0) & (idx < nblk) & (idx.long() * block_size < t - local_window + 1)
    first = torch.ones_like(ok)
    for j in range(1, K):
        first[..., j] = ~(idx[..., :j] == idx[..., j:j + 1]).any(-1)
    return ok & first


def gather_attention(q, k, v, idx, bias, block_size: int, local_window: int, scale: float):
    """q [B,T,HQ,D], k/v [B,T,H,D], idx [B,T,K], bias [B,T,K] -> (o [B,T,HQ,D],
    lse [B,T,HQ]); differentiable in q, k, v and bias (fp32)."""
    B, T, HQ, D = q.shape
    H = k.shape[2]
    G = HQ // H
    nblk = (T + block_size - 1) // block_size
    keep = kept_slots(idx, nblk, block_size, local_window)
    dump = torch.where(keep, idx.long(), torch.full_like(idx.long(), nblk))
    b = bias if bias is not None else torch.zeros(idx.shape, device=q.device)
    dense = torch.zeros(B, T, nblk + 1, device=q.device).scatter(-1, dump, b * keep)
    sel = torch.zeros(B, T, nblk + 1, dtype=torch.bool, device=q.device).scatter(-1, dump, keep)
    kb = torch.arange(T, device=q.device) // block_size
    ti = torch.arange(T, device=q.device).view(T, 1)
    kj = torch.arange(T, device=q.device).view(1, T)
    local = (kj <= ti) & (kj > ti - local_window)                       # [T, T]
    remote = (kj < ti - local_window + 1)[None] & sel[:, :, :nblk][:, :, kb]   # [B, T, T]
    add = torch.where(remote, dense[:, :, :nblk][:, :, kb], torch.zeros((), device=q.device))
    allowed = local[None] | remote
    qh = q.permute(0, 2, 1, 3)                                          # [B,HQ,T,D]
    kh = k.permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    vh = v.permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    s = scale * qh @ kh.transpose(-1, -2) + add[:, None]
    s = s.masked_fill(~allowed[:, None], float("-inf"))
    lse = torch.logsumexp(s, -1)                                        # [B,HQ,T]
    o = torch.softmax(s, -1) @ vh
    return o.permute(0, 2, 1, 3), lse.permute(0, 2, 1)


def gather_attention_grads(q, k, v, idx, bias, dout, block_size, local_window, scale):
    """(o, lse, dq, dk, dv, d_bias) in fp32 via autograd."""
    q = q.float().detach().requires_grad_(True)
    k = k.float().detach().requires_grad_(True)
    v = v.float().detach().requires_grad_(True)
    b = (bias.float() if bias is not None else torch.zeros(idx.shape, device=q.device))
    b = b.detach().requires_grad_(True)
    o, lse = gather_attention(q, k, v, idx, b, block_size, local_window, scale)
    o.backward(dout.float())
    return o.detach(), lse.detach(), q.grad, k.grad, v.grad, b.grad


def entmax15(x: torch.Tensor) -> torch.Tensor:
    """dash_attention.py:623-647: y = relu(z - tau)^2, z = (x - max)/2, tau from
    the sorted prefix sums."""
    z = (x - x.max(-1, keepdim=True).values) / 2
    zs, _ = torch.sort(z, descending=True, dim=-1)
    rho = torch.arange(1, z.shape[-1] + 1, device=z.device, dtype=z.dtype)
    mean = zs.cumsum(-1) / rho
    mean_sq = (zs ** 2).cumsum(-1) / rho
    ss = rho * (mean_sq - mean ** 2)
    tau = mean - torch.sqrt(torch.clamp((1 - ss) / rho, min=0))
    support = (tau <= zs).sum(-1, keepdim=True).clamp(min=1)
    tau_star = tau.gather(-1, support - 1)
    return torch.clamp(z - tau_star, min=0) ** 2


def entmax15_backward(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    """dash_attention.py:650-658."""
    g = y.sqrt()
    dx = dy * g
    q = dx.sum(-1, keepdim=True) / g.sum(-1, keepdim=True).clamp_min(1e-12)
    return dx - q * g


def gather_attention_heads(q, k, v, idx, seg, block_size: int, local_window: int, scale: float):
    """sparse_gather_triton.py restated densely: HI index heads (idx
    [B, HI, T, K], query head hq reads index head hq // (HQ / HI)), packed
    sequences (seg [B, T]: row t sees keys in [seg, t]), no bias.  Keys of a
    routed block below max(t - LW + 1, seg) and the window [that bound, t]
    are kept.  Returns (o [B,T,HQ,D], lse [B,T,HQ]); differentiable in q, k, v."""
    B, T, HQ, D = q.shape
    H = k.shape[2]
    G = HQ // H
    HI = idx.shape[1]
    nblk = (T + block_size - 1) // block_size
    dev = q.device
    kb = torch.arange(T, device=dev) // block_size
    ti = torch.arange(T, device=dev).view(1, T, 1)
    kj = torch.arange(T, device=dev).view(1, 1, T)
    sg = seg.long().view(B, T, 1)
    ls = torch.maximum(ti - local_window + 1, sg)
    local = (kj <= ti) & (kj >= ls)                                       # [B, T, T]
    outs, lses = [], []
    for hq in range(HQ):
        ih = hq // (HQ // HI)
        ids = idx[:, ih].long()                                           # [B, T, K]
        valid = (ids >= 0) & (ids < nblk)          # no bias: duplicates change nothing
        dump = torch.where(valid, ids, torch.full_like(ids, nblk))
        sel = torch.zeros(B, T, nblk + 1, dtype=torch.bool, device=dev).scatter(-1, dump, True)
        remote = (kj < ls) & (kj >= sg) & sel[:, :, :nblk][:, :, kb]
        allowed = local | remote
        s = scale * q[:, :, hq].float() @ k[:, :, hq // G].float().transpose(-1, -2)   # [B, T, T]
        s = s.masked_fill(~allowed, float("-inf"))
        lses.append(torch.logsumexp(s, -1))
        outs.append(torch.softmax(s, -1) @ v[:, :, hq // G].float())
    return torch.stack(outs, 2), torch.stack(lses, 2)


def gather_attention_heads_grads(q, k, v, idx, seg, dout, block_size, local_window, scale):
    """(o, lse, dq, dk, dv) of gather_attention_heads in fp32 via autograd."""
    q = q.float().detach().requires_grad_(True)
    k = k.float().detach().requires_grad_(True)
    v = v.float().detach().requires_grad_(True)
    o, lse = gather_attention_heads(q, k, v, idx, seg, block_size, local_window, scale)
    o.backward(dout.float())
    return o.detach(), lse.detach(), q.grad, k.grad, v.grad
