"""torch fp32 restatement of the reference's own CPU inference path for DASH
prefill: head_cls block scores, canonical route selection and the dense masked
attention, in the same tensor form the reference evaluates on a CPU (whole-row
matmuls over every key with masks, chunked over queries).

TEST INFRASTRUCTURE ONLY: used by ``bench.py``'s CPU legs (the timed CPU
baseline in the reference's own arithmetic, fp32) and by ``tests/``; never by
the product package.  Its outputs are checked against the C oracle and the
reference goldens in tests/test_torch_path.py.

Follows:
* ``_block_scores_infer`` head_cls branch, modeling_deepseekv2.py:351-388
  (k-bar = softmax(k . head_cls / sqrt d) weighted block sums; scores
  clamp(q . k-bar / sqrt d); remote iff block <= q_block - local_blocks).
* ``_infer_route_select``, modeling_deepseekv2.py:309-333 (top-M by score,
  1.5-entmax prior, first K, centred log-prior bias).
* ``_entmax_threshold_and_support`` / ``_Entmax15.forward``,
  dash_attention.py:623-648.
* ``DashAttention._forward_dense``, dash_attention.py:980-1006 (per query chunk:
  logit mask of local window, routed remote blocks with their bias, causal).
"""
from __future__ import annotations

import math

import torch

SCORE_NEG = -1.0e9
ENTMAX_NEG = -1.0e4
ACT_CLAMP = 1.0e4
MASK_NEG = -1.0e9


def kbar_headcls(idx_k: torch.Tensor, head_cls: torch.Tensor, block_size: int) -> torch.Tensor:
    """[B, S, d] -> [B, nblk, d]: per block, softmax over its tokens of
    clamp(k . head_cls / sqrt d) (denominator >= 1e-6), weighted key sum."""
    B, S, d = idx_k.shape
    nblk = -(-S // block_size)
    pad = nblk * block_size - S
    kk = torch.nn.functional.pad(idx_k, (0, 0, 0, pad)).view(B, nblk, block_size, d)
    real = (torch.arange(nblk * block_size) < S).view(1, nblk, block_size)
    aw = ((kk * head_cls.view(1, 1, 1, d)).sum(-1) / math.sqrt(d)).clamp(-ACT_CLAMP, ACT_CLAMP)
    aw = aw.masked_fill(~real, float("-inf"))
    mx = aw.amax(-1, keepdim=True)
    w = torch.exp(aw - mx) * real
    w = w / w.sum(-1, keepdim=True).clamp_min(1e-6)
    return torch.nan_to_num((w.unsqueeze(-1) * kk).sum(2), nan=0.0, posinf=0.0, neginf=0.0)


def block_scores(idx_q: torch.Tensor, q_pos: torch.Tensor, kbar: torch.Tensor, block_size: int,
                 local_blocks: int) -> torch.Tensor:
    """[B, L, d] queries at positions q_pos [B, L] -> [B, L, nblk] scores,
    SCORE_NEG where the block is not remote for the query."""
    d = idx_q.shape[-1]
    z = (idx_q @ kbar.transpose(-1, -2) / math.sqrt(d)).clamp(-ACT_CLAMP, ACT_CLAMP)
    blk = torch.arange(kbar.shape[1]).view(1, 1, -1)
    remote = blk <= (q_pos // block_size).unsqueeze(-1) - local_blocks
    return z.masked_fill(~remote, SCORE_NEG)


def entmax15(x: torch.Tensor) -> torch.Tensor:
    """1.5-entmax over the last dim with the sorted-prefix threshold."""
    z = (x - x.amax(-1, keepdim=True)) / 2
    zs = torch.sort(z, descending=True, dim=-1).values
    n = torch.arange(1, z.shape[-1] + 1, dtype=z.dtype)
    mean = zs.cumsum(-1) / n
    msq = (zs * zs).cumsum(-1) / n
    tau = mean - torch.sqrt(torch.clamp((1 - n * (msq - mean * mean)) / n, min=0))
    support = (tau <= zs).sum(-1, keepdim=True).clamp(min=1)
    t = tau.gather(-1, support - 1)
    return torch.clamp(z - t, min=0) ** 2


def route_select(scores: torch.Tensor, idx_scale: float, topm: int, K: int, floor: float,
                 sigma: float):
    """-> (ids [.., K] int64, bias [.., K] fp32, valid [.., K] bool), ids in
    descending score order like the reference."""
    remote = scores > SCORE_NEG * 0.5
    x = torch.where(remote, scores * idx_scale, torch.full_like(scores, ENTMAX_NEG))
    M = max(1, min(topm, x.shape[-1]))
    xv, xi = x.topk(M, dim=-1)
    prior = entmax15(xv)
    K = max(1, min(K, M))
    ids, prior, valid = xi[..., :K], prior[..., :K], remote.gather(-1, xi)[..., :K]
    logp = torch.log(prior.clamp_min(floor))
    cnt = valid.sum(-1, keepdim=True).clamp(min=1)
    mu = torch.where(valid, logp, torch.zeros_like(logp)).sum(-1, keepdim=True) / cnt
    bias = torch.where(valid, (logp - mu) / sigma, torch.zeros_like(logp))
    return ids, bias, valid


def attend_dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor,
                 ids: torch.Tensor, bias: torch.Tensor, valid: torch.Tensor, block_size: int,
                 local_window: int, scale: float, q_chunk: int = 512) -> torch.Tensor:
    """Dense masked attention of query rows ``rows`` (positions) of q [B, H, S, D]
    over all S keys of k/v [B, H, S, D]; ids/bias/valid [B, len(rows), K].
    Returns [B, H, len(rows), D]."""
    B, H, S, D = q.shape
    nblk = -(-S // block_size)
    key_blk = torch.arange(S) // block_size
    kpos = torch.arange(S)
    # per-row additive term per block (MASK_NEG where not routed)
    lp = torch.full((B, rows.numel(), nblk), MASK_NEG)
    lp.scatter_(-1, ids.clamp(min=0), torch.where(valid, bias, torch.full_like(bias, MASK_NEG)))
    out = []
    for c0 in range(0, rows.numel(), q_chunk):
        r = rows[c0:c0 + q_chunk]
        base = lp[:, c0:c0 + q_chunk].index_select(-1, key_blk)             # [B, c, S]
        causal = kpos[None, :] <= r[:, None]
        local = causal & (kpos[None, :] > r[:, None] - local_window)
        keep = causal & (local | (base > MASK_NEG * 0.5))
        add = torch.where(local, torch.zeros_like(base), base).masked_fill(~keep, MASK_NEG)
        out.append(torch.nn.functional.scaled_dot_product_attention(
            q[:, :, r], k, v, attn_mask=add[:, None].clamp_min(MASK_NEG), scale=scale))
    return torch.cat(out, dim=2)


def prefill_rows(q, k, v, idx_q, idx_k, rows, *, block_size, local_blocks, K, topm, idx_scale,
                 floor=1e-4, sigma=1.0, head_cls=None):
    """The whole path for the query positions ``rows`` of every sequence:
    k-bar of all blocks, scores and selection of those rows, their attention.
    Returns (out [B, H, len(rows), D], ids, bias, valid)."""
    d = idx_k.shape[-1]
    hc = torch.zeros(d) if head_cls is None else head_cls
    kb = kbar_headcls(idx_k, hc, block_size)
    B = q.shape[0]
    pos = rows.view(1, -1).expand(B, -1)
    sc = block_scores(idx_q[:, rows], pos, kb, block_size, local_blocks)
    ids, bias, valid = route_select(sc, idx_scale, topm, K, floor, sigma)
    out = attend_dense(q, k, v, rows, ids, bias, valid, block_size, local_blocks * block_size,
                       1.0 / math.sqrt(q.shape[-1]))
    return out, ids, bias, valid
