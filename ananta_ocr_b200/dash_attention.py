"""Drop-in for the 1.5-entmax prior of ANANTA_OCR ``dash_attention.py``.

``entmax15`` / ``_Entmax15`` keep the reference's names and autograd contract
(dash_attention.py:637-662): forward y = relu(z - tau)^2 with z = (x - max)/2
and sum(y) = 1, backward dx = dy*g - g * sum(dy*g) / max(sum g, 1e-12) with
g = sqrt(y).  Both run as kernels of ``libdash_b200.so``
(``dash_entmax15_fwd`` / ``dash_entmax15_bwd``) over the rows of the last
dim of any other dim order (moved last and back).  fp32 (inputs of other
dtypes are computed in fp32 and returned in their dtype).
"""
from __future__ import annotations

import torch

from . import ops


class _Entmax15(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, dim):
        ctx.dim = dim
        x = X.movedim(dim, -1)
        y = ops.entmax15(x).to(X.dtype)
        ctx.save_for_backward(y)
        return y.movedim(-1, dim)

    @staticmethod
    def backward(ctx, dY):
        (y,) = ctx.saved_tensors
        dx = ops.entmax15_backward(y, dY.movedim(ctx.dim, -1)).to(dY.dtype)
        return dx.movedim(-1, ctx.dim), None


def entmax15(X, dim=-1):
    return _Entmax15.apply(X, dim)


# ---------------------------------------------------------------------------
# DashAttention (dash_attention.py:703-1071)
# ---------------------------------------------------------------------------
import math    # noqa: E402
import os      # noqa: E402

import torch.nn as nn             # noqa: E402
import torch.nn.functional as F   # noqa: E402

SCORE_NEG = -1.0e9      # dash_attention.py:602
ACT_CLAMP = 1.0e4       # :604
GRAD_CLAMP = 1.0e4      # :603
ENTMAX_NEG = -1.0e4     # DashAttention._neg, :753


def _bound_grad(g):
    """The reference's gradient guard (dash_attention.py:607-612): non-finite
    entries to 0, then clamp."""
    return None if g is None else torch.nan_to_num(g, nan=0.0, posinf=0.0, neginf=0.0).clamp(
        -GRAD_CLAMP, GRAD_CLAMP)


class _RMSNorm(nn.Module):
    """Gemma-style RMSNorm of the router's index projections (scale 1 + weight,
    weight initialised to 0) with the reference's fp32 finiteness guards and
    clamps (dash_attention.py:680-700)."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.zeros(dim))

    def forward(self, x):
        x32 = torch.nan_to_num(x.float(), nan=0.0, posinf=0.0, neginf=0.0)
        x32 = (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.eps)).clamp(-ACT_CLAMP, ACT_CLAMP)
        out = (x32 * (1.0 + self.weight.float())).clamp(-ACT_CLAMP, ACT_CLAMP).to(x.dtype)
        if out.requires_grad:
            out.register_hook(_bound_grad)
        return out


def _rotate(x, cos, sin):
    """Rotate-half RoPE with cos/sin [B, S, d] broadcast over the head dim
    (transformers' Llama apply_rotary_pos_emb, unsqueeze_dim=1)."""
    h = x.shape[-1] // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), -1)
    return x * cos.unsqueeze(1) + rot * sin.unsqueeze(1)


class DashAttention(nn.Module):
    """The reference's DASH attention module with its router and attention on
    ``libdash_b200``: same constructor (the model config's
    ``sparse_attention_config``), parameters and state_dict keys (``q_proj``,
    ``k_proj``, ``q_norm``, ``k_norm``, ``head_cls``), and ``forward``
    signature and result ([B, H, S, D] before o_proj).

    Per call (dash_attention.py:1008-1071): block scores from the index
    projections (stage 0 ``head_cls``: learned block summaries; ``indexer``:
    block max of token dots), candidates = remote blocks restricted by
    ``block_cand`` (per query) or the image-block mask, with a per-row
    fallback to all remote blocks; 1.5-entmax prior over the candidates; top-K
    blocks by prior with the centred log-prior bias; gather attention.

    Without gradients the router runs on the library: index projections
    (tcgen05, bf16 hidden states), block summaries, and scores + entmax +
    selection + bias in one routing kernel (entmax window
    min(blocks, 256)); the attention is the tcgen05 prefill kernel.  With
    gradients the projections, summaries and scores are torch ops, the prior is
    the library's entmax (its autograd backward is the library's Jacobian
    kernel) and the attention is the library's forward/backward pair, so the
    gradients reach q, k, v, the projections, the norms and ``head_cls``.

    Not reproduced: the training-loop schedulers (the k anneal ``_KS`` and the
    per-layer temperature ``_SCHED``): ``k`` is a plain attribute, initialised
    like the reference's fresh schedule (``DASH_K_START``, default 64), and
    the entmax scale and prior floor are the config's.  A call with an
    ``attention_mask`` raises (the reference falls back to a dense torch path
    there; this library has no dense fallback).

    Selection ties: the library ranks candidates by score (lowest block id on
    equal scores); the reference takes ``topk`` of the masked prior.  Entmax is
    monotone, so the two agree except when a row has fewer than K blocks of
    non-zero prior and more zero-prior candidates than remaining slots: the
    zero-prior blocks each rule picks may differ (they all carry the same
    bias, log(floor) - mean)."""

    def __init__(self, config):
        super().__init__()
        sp = getattr(config, "sparse_attention_config", {}) or {}
        self.num_heads = config.num_attention_heads
        self.head_dim = config.hidden_size // config.num_attention_heads
        self.block_size = int(sp.get("sparse_block_size", 128))
        self.local_blocks = max(1, int(sp.get("sparse_local_block", 1)))
        self.local_window = self.local_blocks * self.block_size
        self.scaling_factor = float(sp.get("dash_scaling_factor", 2.0))
        self.q_chunk = int(sp.get("dash_query_chunk", 2048))
        self.image_only = bool(sp.get("dash_image_only", True))
        self._image_token_id = int(sp.get("image_token_id", 128815))
        self.sigma = float(sp.get("dash_sigma", 1.0))
        self._prior_floor = float(sp.get("dash_prior_floor", 1e-2))
        self.topk_blocks = int(sp.get("sparse_topk_blocks", 16))
        self.remote_blocks = max(1, self.topk_blocks - self.local_blocks)
        self.use_triton = bool(sp.get("dash_use_triton", True))
        self.index_dim = int(sp.get("sparse_index_dim", self.head_dim))
        eps = getattr(config, "rms_norm_eps", 1e-6)
        self.q_proj = nn.Linear(config.hidden_size, self.index_dim, bias=False)
        self.k_proj = nn.Linear(config.hidden_size, self.index_dim, bias=False)
        self.q_norm = _RMSNorm(self.index_dim, eps=eps)
        self.k_norm = _RMSNorm(self.index_dim, eps=eps)
        self.stage0 = os.environ.get("DASH_STAGE0", "indexer").lower()
        self.head_cls = nn.Parameter(torch.zeros(self.index_dim))
        self._scale = 1.0 / math.sqrt(self.head_dim)
        self._idx_scale = self.scaling_factor / math.sqrt(self.index_dim)
        self._neg = ENTMAX_NEG
        self.k = int(os.environ.get("DASH_K_START", "64"))

    # ---- helpers ---------------------------------------------------------
    @torch.no_grad()
    def build_image_block_mask(self, source_input_ids, key_length, nblk, device):
        """[B, nblk] bool: the block holds at least one image token; None when
        there are no ids or no image token (dash_attention.py:778-799).  The
        block test is the library's ``dash_block_any``."""
        from . import pages
        if source_input_ids is None or source_input_ids.ndim != 2:
            return None
        ids = source_input_ids[..., :key_length].to(device)
        if ids.shape[-1] < key_length:
            ids = F.pad(ids, (0, key_length - ids.shape[-1]), value=-1)
        img = ids == self._image_token_id
        if not bool(img.any()):
            return None
        return pages.block_any(img, nblk, self.block_size)

    def _wants_grad(self, *ts):
        return torch.is_grad_enabled() and (any(t is not None and t.requires_grad for t in ts)
                                            or any(p.requires_grad for p in self.parameters()))

    def _index_qk(self, hidden_states, position_embeddings, grad):
        """Router index queries/keys [B, S, d] fp32: RoPE(RMSNorm(W h))
        (dash_attention.py:845-858)."""
        B, S, Hd = hidden_states.shape
        d = self.index_dim
        cos = sin = None
        if position_embeddings is not None:
            cos, sin = position_embeddings
            cos, sin = cos[..., :d].expand(B, S, d), sin[..., :d].expand(B, S, d)
        lib_ok = (not grad and hidden_states.dtype == torch.bfloat16 and d == 128 and
                  self.q_proj.weight.dtype == torch.bfloat16)
        if lib_ok:
            iq, ik = ops.index_proj(
                hidden_states.reshape(B * S, Hd), self.q_proj.weight, self.k_proj.weight,
                self.q_norm.weight, self.k_norm.weight, float(self.q_norm.eps),
                cos=None if cos is None else cos.reshape(B * S, d).to(torch.bfloat16),
                sin=None if sin is None else sin.reshape(B * S, d).to(torch.bfloat16),
                norm_clamp=True)
            return iq.view(B, S, d), ik.view(B, S, d)
        hs = torch.nan_to_num(hidden_states, nan=0.0, posinf=0.0, neginf=0.0)
        iq = self.q_norm(self.q_proj(hs).view(B, S, 1, d)).transpose(1, 2)
        ik = self.k_norm(self.k_proj(hs).view(B, S, 1, d)).transpose(1, 2)
        if cos is not None:
            iq, ik = _rotate(iq, cos.to(iq.dtype), sin.to(iq.dtype)), _rotate(ik, cos.to(ik.dtype), sin.to(ik.dtype))
        iq = torch.nan_to_num(iq[:, 0].float(), nan=0.0, posinf=0.0, neginf=0.0)
        ik = torch.nan_to_num(ik[:, 0].float(), nan=0.0, posinf=0.0, neginf=0.0)
        for t in (iq, ik):
            if t.requires_grad:
                t.register_hook(_bound_grad)
        return iq, ik

    def _block_scores_torch(self, idx_q, idx_k, position_ids, nblk):
        """Differentiable block scores [B, S, nblk] (SCORE_NEG where the block is
        not remote): head_cls (dash_attention.py:860-904) or indexer (:815-835)."""
        B, S, d = idx_k.shape
        bs = self.block_size
        Sp = nblk * bs
        inv = 1.0 / math.sqrt(d)
        if self.stage0 == "head_cls":
            kk = F.pad(idx_k, (0, 0, 0, Sp - S)).view(B, nblk, bs, d)
            real = (torch.arange(Sp, device=idx_k.device) < S).view(1, nblk, bs)
            aw = ((kk * self.head_cls.to(kk.dtype).view(1, 1, 1, d)).sum(-1) * inv).clamp(-ACT_CLAMP, ACT_CLAMP)
            mx = torch.where(real, aw, aw.new_full((), torch.finfo(aw.dtype).min)).amax(-1, keepdim=True)
            e = torch.exp(aw - mx) * real.to(aw.dtype)
            w = e / e.sum(-1, keepdim=True).clamp_min(1e-6)
            kbar = torch.nan_to_num((w.unsqueeze(-1) * kk).sum(2), nan=0.0, posinf=0.0, neginf=0.0)
            z = (idx_q @ kbar.transpose(-1, -2))
            if z.requires_grad:
                z.register_hook(_bound_grad)
            z = (z * inv).clamp(-ACT_CLAMP, ACT_CLAMP)
            remote = (torch.arange(nblk, device=z.device)[None, None] <=
                      (position_ids // bs)[:, :, None] - self.local_blocks)
            return z.masked_fill(~remote, SCORE_NEG)
        kpos = torch.arange(S, device=idx_k.device)
        out = []
        for c0 in range(0, S, self.q_chunk):
            c1 = min(c0 + self.q_chunk, S)
            sc = (idx_q[:, c0:c1] @ idx_k.transpose(-1, -2)).clamp(-ACT_CLAMP, ACT_CLAMP)
            pos = position_ids[:, c0:c1]
            future = kpos[None, None] > pos[:, :, None]
            local = (kpos[None, None] > pos[:, :, None] - self.local_window) & ~future
            sc = F.pad(sc.masked_fill(future | local, SCORE_NEG), (0, Sp - S), value=SCORE_NEG)
            out.append(sc.view(B, c1 - c0, nblk, bs).amax(-1))
        return torch.cat(out, 1)

    def _route(self, block_scores, image_block_mask, block_cand=None):
        """(prior [B, S, nblk], cand) (dash_attention.py:906-930): candidates
        with the per-row fallback, prior = 1.5-entmax on the library."""
        remote = block_scores > SCORE_NEG * 0.5
        cand = remote
        if block_cand is not None:
            cand = remote & block_cand
        elif self.image_only and image_block_mask is not None:
            cand = remote & image_block_mask[:, None, :]
        cand = torch.where(~cand.any(-1, keepdim=True), remote, cand)
        x = torch.where(cand, block_scores * self._idx_scale, block_scores.new_full((), self._neg))
        x = torch.nan_to_num(x, nan=self._neg, posinf=self._neg, neginf=self._neg)
        return entmax15(x, dim=-1), cand

    def _select_and_bias(self, prior, cand, nblk):
        """Top-K of the masked prior and the centred log-prior bias
        (dash_attention.py:932-960)."""
        K = max(1, min(int(self.k), nblk))
        topv, topi = prior.masked_fill(~cand, -1.0).topk(K, dim=-1)
        valid = topv >= 0.0
        logp = torch.log(topv.clamp_min(self._prior_floor))
        cnt = valid.sum(-1, keepdim=True).clamp(min=1)
        mu = torch.where(valid, logp, torch.zeros_like(logp)).sum(-1, keepdim=True) / cnt
        bias = torch.where(valid, (logp - mu) / self.sigma, torch.zeros_like(logp)).clamp(-ACT_CLAMP, ACT_CLAMP)
        return topi, bias, valid

    def _route_library(self, idx_q, idx_k, position_ids, nblk, image_block_mask, block_cand):
        """No-gradient routing on the library: (idx [B, S, K] ascending with -1
        tail, bias [B, S, K])."""
        B, S, d = idx_q.shape
        K = max(1, min(int(self.k), nblk))
        pos0 = position_ids[:, 0].to(torch.int32).contiguous()
        seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, pos0=pos0, max_q_len=S)
        cand, per_seq = None, False
        if block_cand is not None:
            cand = block_cand.reshape(B * S, nblk)
        elif self.image_only and image_block_mask is not None:
            cand, per_seq = image_block_mask, True
        common = dict(width=nblk, block_size=self.block_size, local_blocks=self.local_blocks,
                      idx_scale=self._idx_scale, prior_floor=self._prior_floor, sigma=self.sigma,
                      topm=min(nblk, 256), K=K, cand=cand, cand_per_seq=per_seq)
        if self.stage0 == "head_cls":
            kbar = ops.kbar_pool_contig(idx_k, self.head_cls, self.block_size)
            idx, bias = ops.route(seqs, idx_q=idx_q.reshape(B * S, d), kbar=kbar, **common)
        else:
            sc = ops.block_max(idx_q, idx_k, position_ids, None, self.block_size, nblk,
                               self.local_window, clamp=True, empty=SCORE_NEG)
            idx, bias = ops.route(seqs, scores_in=sc.reshape(B * S, nblk), **common)
        return idx.view(B, S, K), bias.view(B, S, K)

    def forward(self, hidden_states, q, k, v, position_embeddings=None, position_ids=None,
                attention_mask=None, image_block_mask=None, block_cand=None, page_ids=None):
        """hidden_states [B, S, hidden]; q, k, v [B, H, S, D] (RoPE'd, GQA-expanded).
        Returns [B, H, S, D] (before o_proj).  ``page_ids`` feeds only the
        reference's diagnostics and is ignored."""
        from .sparse_gather_e2e_triton import triton_gather_attention_e2e
        if attention_mask is not None:
            raise NotImplementedError("DashAttention on libdash_b200 takes no attention_mask "
                                      "(no dense fallback)")
        B, H, S, D = q.shape
        nblk = (S + self.block_size - 1) // self.block_size
        if position_ids is None:
            position_ids = torch.arange(S, device=q.device)[None].expand(B, -1)
        grad = self._wants_grad(hidden_states, q, k, v)
        arange = bool((position_ids == position_ids[:, :1] + torch.arange(
            S, device=position_ids.device)[None]).all())
        idx_q, idx_k = self._index_qk(hidden_states, position_embeddings, grad)
        if grad or not arange:
            scores = self._block_scores_torch(idx_q, idx_k, position_ids, nblk)
            if scores.requires_grad:
                scores.register_hook(_bound_grad)
            prior, cand = self._route(scores, image_block_mask, block_cand)
            topi, bias, valid = self._select_and_bias(prior, cand, nblk)
            block_indices = topi.masked_fill(~valid, -1).to(torch.int32).unsqueeze(1)
        else:
            idx, bias = self._route_library(idx_q, idx_k, position_ids, nblk, image_block_mask,
                                            block_cand)
            block_indices = idx.unsqueeze(1)
        out = triton_gather_attention_e2e(q, k, v, block_indices, bias, position_ids, None,
                                          self.block_size, self._scale, self.local_window)
        if out is None:
            raise NotImplementedError("DashAttention on libdash_b200 needs consecutive "
                                      "positions per sequence (no dense fallback)")
        return out
