"""Drop-ins for the DASH inference functions of ANANTA_OCR
``modeling_deepseekv2.py`` that the DeepSeek-V2 decoder calls, backed by
libdash_b200.so:

* ``_block_scores_infer`` (modeling_deepseekv2.py:351-400): stage-0 block
  scores, ``head_cls`` (k-bar pooling + scoring) or ``indexer`` (block max).
* ``_infer_route_select`` (modeling_deepseekv2.py:309-333): candidate mask,
  1.5-entmax over the top-``topm`` scores, top-K selection, centred bias.
* ``_decode_attend`` (modeling_deepseekv2.py:424-451): decode gather attention
  over a contiguous cache.
* ``_router_qk`` (modeling_deepseekv2.py:336-348): the router's index
  projections + RMSNorm + RoPE as one tcgen05 GEMM with a fused epilogue.
* ``dash_prefill_forward``: the ``_infer_prefill_attend`` flow
  (modeling_deepseekv2.py:403-421) after the router projections: scores ->
  selection -> gather attention, with the routed lists kept on the device;
  with ``page_domain`` the page-aware candidates of ``_dash_block_cand`` are
  applied inside the router from their compact form (no [B, S, nblk] mask).
* ``_dash_page_ids`` / ``_dash_block_cand`` (modeling_deepseekv2.py:87-114):
  page-aware ids and the per-query candidate domain through the indexer's
  builders (``_sparse_base_impl.DeepseekV2IndexerPages``).
* ``page_domain_from_ids``: token ids -> the compact domain for
  ``dash_prefill_forward`` in one kernel pass.

``router`` arguments only need the attributes the reference reads
(stage0, block_size, local_blocks, local_window, head_cls, _infer_params).
"""
from __future__ import annotations

import math

import torch

from . import ops
from .sparse_gather_e2e_triton import _as_kernel_dtype

_SCORE_NEG = -1.0e9
_MASK_NEG = -1.0e9


def _dash_page_ids(self, idx, src_ids, key_length):
    """modeling_deepseekv2.py:87-96: (image mask, image page ids, query page ids)."""
    if idx.image_bucket_constraint:
        return idx._build_page_aware_ids(src_ids, idx.image_token_id, idx.page_token_id,
                                         key_length)
    itm = idx._build_flat_image_token_mask(src_ids, idx.image_token_id, key_length)
    return itm, None, None


def _dash_block_cand(self, idx, router, pos_ids, itm, ipi, qpi, nblk, bsz, q_len):
    """modeling_deepseekv2.py:99-114: [B, S, nblk] bool per-query candidate
    domain, or None.  One pass: the kernels never build the [B, S, nblk,
    block_size] comparison, so ``router.q_chunk`` slicing is not needed."""
    if itm is None and (ipi is None or qpi is None):
        return None
    cm = idx._build_kl_candidate_mask(pos_ids, nblk, itm, bsz, q_len,
                                      image_token_page_ids=ipi, query_token_page_ids=qpi)
    return cm[:, 0]


@torch.no_grad()
def page_domain_from_ids(token_ids, *, image_token_id, page_token_id, per_page, block_size,
                         nblk, page_scope_prefill=False):
    """Compact page-aware domain of a fresh contiguous prefill (query row t of
    sequence b at position t): query page per row + exact page descriptors per
    block, from one ``dash_page_ids`` pass.  Same candidates as
    ``_dash_block_cand`` with ``image_bucket_constraint``."""
    from .pages import PageDomain, page_ids
    B, S = token_ids.shape
    r = page_ids(token_ids, image_token_id=image_token_id, page_token_id=page_token_id,
                 per_page=per_page, key_length=S, rule=0, page_scope_prefill=page_scope_prefill,
                 block_size=block_size, n_blocks=nblk, want_image=False)
    return PageDomain(q_page=r["query_page"].view(-1), lo=r["lo"], hi=r["hi"], bits=r["bits"],
                      seq_rows=nblk)


@torch.no_grad()
def _router_qk(router, hidden_states, pe):
    """modeling_deepseekv2.py:336-348: router index q/k [B, S, d] fp32 =
    RoPE(_RMSNorm(W hidden)) in one tcgen05 kernel (bf16 GEMM, fp32
    accumulate, the reference's bf16 roundings in the epilogue).  Non-finite
    hidden values are not zeroed before the GEMM (rows holding them come out
    zeroed by the norm instead)."""
    B, S, Hd = hidden_states.shape
    d = router.index_dim
    cos = sin = None
    if pe is not None:
        cos, sin = pe
        cos = cos.expand(B, S, cos.shape[-1]).reshape(B * S, cos.shape[-1])[:, :d]
        sin = sin.expand(B, S, sin.shape[-1]).reshape(B * S, sin.shape[-1])[:, :d]
    idx_q, idx_k = ops.index_proj(hidden_states.reshape(B * S, Hd), router.q_proj.weight,
                                  router.k_proj.weight, router.q_norm.weight,
                                  router.k_norm.weight, float(router.q_norm.eps), cos=cos,
                                  sin=sin, norm_clamp=True)
    return idx_q.view(B, S, d), idx_k.view(B, S, d)


@torch.no_grad()
def _block_scores_infer(router, idx_q, idx_k, q_pos, nblk):
    """[B,Lq,nblk] fp32 remote block scores (SCORE_NEG where not remote)."""
    B, S, d = idx_k.shape
    Lq = idx_q.shape[1]
    bs = router.block_size
    q_pos = torch.as_tensor(q_pos, device=idx_q.device)
    if router.stage0 == "head_cls":
        kbar = ops.kbar_pool_contig(idx_k.float(), router.head_cls, bs)
        nb_k = kbar.shape[1]
        if nb_k < nblk:
            kbar = torch.cat([kbar, kbar.new_zeros(B, nblk - nb_k, d)], 1)
        pos0 = q_pos[:, 0].to(torch.int32).contiguous()
        seqs = ops.Seqs(n_seq=B, q_len=Lq, kv_len=S, pos0=pos0, max_q_len=Lq)
        scores = torch.empty(B * Lq, nblk, dtype=torch.float32, device=idx_q.device)
        ops.route(seqs, width=nblk, block_size=bs, local_blocks=router.local_blocks,
                  idx_scale=1.0, prior_floor=1e-4, sigma=1.0, topm=1, K=1,
                  idx_q=idx_q.reshape(B * Lq, d), kbar=kbar, scores_out=scores)
        return scores.view(B, Lq, nblk)
    return ops.block_max(idx_q, idx_k, q_pos.expand(B, Lq), None, bs, nblk,
                         router.local_window, clamp=True, empty=_SCORE_NEG)


@torch.no_grad()
def _infer_route_select(block_scores, block_cand, p):
    """(topi int64 [B,Lq,K], bias fp32, valid bool).  Valid ids come first in
    ascending order (the reference orders them by descending score; the set
    and the bias of each id are the same)."""
    B, Lq, nblk = block_scores.shape
    M = max(1, min(int(p["topm"]), nblk)) if int(p["topm"]) > 0 else nblk
    K = max(1, min(int(p["K"]), M))
    seqs = ops.Seqs(n_seq=B * Lq, q_len=1, kv_len=0, max_q_len=1)
    cand = None if block_cand is None else block_cand.reshape(B * Lq, nblk)
    idx, bias = ops.route(seqs, width=nblk, block_size=1, local_blocks=0,
                          idx_scale=float(p["idx_scale"]), prior_floor=float(p["floor"]),
                          sigma=float(p["sigma"]), topm=M, K=K,
                          scores_in=block_scores.reshape(B * Lq, nblk).float(), cand=cand)
    idx = idx.view(B, Lq, K)
    valid = idx >= 0
    return idx.clamp_min(0).long(), bias.view(B, Lq, K), valid


@torch.no_grad()
def _decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size, local_window, scale):
    """q [B,H,Lq,D]; k_all/v_all [B,Hkv,S,D] contiguous cache; routes [B,Lq,K]."""
    B, H, Lq, D = q.shape
    S = k_all.shape[2]
    Hkv = k_all.shape[1]
    idx = torch.where(valid, topi, torch.full_like(topi, -1)).to(torch.int32).contiguous()
    bias = torch.where(valid, bias, torch.zeros_like(bias)).float().contiguous()
    qq = _as_kernel_dtype(q)
    kk = _as_kernel_dtype(k_all).to(qq.dtype)
    vv = _as_kernel_dtype(v_all).to(qq.dtype)
    out = torch.empty(B, H, Lq, D, dtype=qq.dtype, device=q.device)
    pos0 = torch.as_tensor(q_pos, device=q.device)[:, 0].to(torch.int32).contiguous()
    seqs = ops.Seqs(n_seq=B, q_len=Lq, kv_len=S, pos0=pos0, max_q_len=Lq)
    from . import _lib as L
    if qq.dtype == torch.float32:
        # fp32 (the reference computes this path in fp32): the fp32 prefill
        # kernel with the Lq query rows at their positions over the whole cache
        a = L.DashPrefillArgs()
        a.seqs = seqs.c()
        a.kv = ops._kv(kk, vv, None, Hkv, (kk.stride(0), kk.stride(2), kk.stride(1)))
        idx2 = idx.view(B * Lq, -1)
        bias2 = bias.view(B * Lq, -1)
        a.routes = ops._routes(idx2, bias2, idx2.stride(0), 0, 1)
        a.qo = ops._qo(qq, out, (qq.stride(0), qq.stride(2), qq.stride(1)),
                       (out.stride(0), out.stride(2), out.stride(1)), H)
        a.scale, a.block_size, a.local_window = float(scale), int(block_size), int(local_window)
        ops.prefill_attn(a, q.device)
        return out
    a = L.DashDecodeArgs()
    a.seqs = seqs.c()
    a.kv = ops._kv(kk, vv, None, Hkv, (kk.stride(0), kk.stride(2), kk.stride(1)))
    a.routes = ops._routes(idx, bias, idx.stride(1), 0, 1)
    a.qo = ops._qo(qq, out, (qq.stride(0), qq.stride(2), qq.stride(1)),
                   (out.stride(0), out.stride(2), out.stride(1)), H)
    a.scale, a.block_size, a.local_window = float(scale), int(block_size), int(local_window)
    ops.decode_attn(a, q.device)
    return out.float()


@torch.no_grad()
def dash_prefill_forward(q, k, v, idx_q, idx_k, *, block_size, local_blocks, head_cls=None,
                         K, topm=None, idx_scale, prior_floor, sigma, scale=None,
                         return_routes=False, page_domain=None, out=None, peers=None):
    """Router + gather attention for a contiguous prefill.

    q [B,H,S,D], k/v [B,Hkv,S,D] (bf16/fp16), idx_q/idx_k [B,S,d] fp32 router
    queries/keys.  Returns out [B,H,S,D] (and the routed lists if asked);
    ``out``/``peers`` as in ``ops.gather_attention`` (fused output gather)."""
    B, H, S, D = q.shape
    d = idx_q.shape[-1]
    nblk = (S + block_size - 1) // block_size
    kbar = ops.kbar_pool_contig(idx_k, head_cls, block_size)
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    idx, bias = ops.route(seqs, width=nblk, block_size=block_size, local_blocks=local_blocks,
                          idx_scale=idx_scale, prior_floor=prior_floor, sigma=sigma,
                          topm=int(topm or K), K=K, idx_q=idx_q.reshape(B * S, d), kbar=kbar,
                          page=page_domain)
    out = ops.gather_attention(q, k, v, idx.view(B, S, K), bias.view(B, S, K),
                               block_size=block_size, local_window=local_blocks * block_size,
                               scale=float(scale if scale is not None else 1.0 / math.sqrt(D)),
                               out=out, peers=peers)
    if return_routes:
        return out, idx.view(B, S, K), bias.view(B, S, K)
    return out
