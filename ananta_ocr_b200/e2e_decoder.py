"""End-to-end DeepSeek-V2-style decoder with the DASH kernels as its attention.

The decoder of ANANTA_OCR (modeling_deepseekv2.py / the sglang
unlimited_ocr_v2.py model) around this library's serving path, used to measure
the attention kernels inside a whole model and to check
that a paged prefill followed by decode steps reproduces a longer prefill.
Weights are random (the trained checkpoint is not available); the layer
structure is the model's: RMSNorm, q/k/v/o projections (10 x 128 heads),
the DASH router's index branch, a dense SwiGLU FFN in the first layer and a
64-expert top-6 MoE with 2 shared experts after it (softmax gate, no top-k
renormalisation, routing scale 1), final norm, LM head on the last token.

Attention per layer, all through libdash_b200:
  rope_and_store_kv   rotate q in place; rotated k and v into the paged cache
  index_qk_fused      index projections + RMSNorm + RoPE; idx_k into the paged
                      index cache
  kbar refresh        k-bar summaries of the pages written this step
  route_*_triton      scores + 1.5-entmax + top-K over the paged k-bar, with
                      page-aware candidates when the token ids are given
                      (PageIsolationState, once per forward for all layers)
  dash_sparse_attn*   paged prefill (tcgen05) / decode (split-KV) attention
The GEMMs and the MoE are PyTorch (cuBLAS).  ``decode_step`` allocates nothing
that changes between steps and is captured in a CUDA graph by the caller.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import torch
import torch.nn.functional as F

from .unlimited_dash_ops import attend_triton as AT
from .unlimited_dash_ops import decode_meta_triton as DM
from .unlimited_dash_ops import index_frontend as IF
from .unlimited_dash_ops import page_state as PS
from .unlimited_dash_ops import route_triton as RT


@dataclass
class DecoderConfig:
    hidden: int = 1280
    heads: int = 10
    kv_heads: int = 10
    head_dim: int = 128
    layers: int = 12
    vocab: int = 129280
    dense_ffn: int = 6848
    moe_ffn: int = 896
    experts: int = 64
    topk: int = 6
    shared: int = 2
    first_dense: int = 1
    eps: float = 1e-6
    rope_theta: float = 500000.0
    # the checkpoint's DASH settings (config.json: sparse_block_size 32,
    # sparse_local_block 4, dash_topk_blocks 12) and the serving router's
    # defaults (WHL dash_router.py:16,101-105: entmax window 16, 16 output
    # slots, the last 4 of them -1)
    block_size: int = 32
    local_blocks: int = 4
    K: int = 12
    topm: int = 16
    slots: int = 16
    index_dim: int = 128
    scaling: float = 128.0
    prior_floor: float = 1e-4
    sigma: float = 1.0


def rmsnorm(x, w, eps):
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return (x32 * w).to(x.dtype)


class DashDecoder:
    """Random-init bf16 decoder with paged caches for ``batch`` sequences of
    up to ``max_len`` tokens."""

    def __init__(self, cfg: DecoderConfig, batch: int, max_len: int, device, seed: int = 0,
                 page_cfg=None, page_mask: bool = False):
        self.cfg = c = cfg
        self.B = batch
        self.dev = device
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape, std):
            return (torch.randn(*shape, generator=g, device=device) * std).to(bf)

        H = c.hidden
        self.embed = rnd(c.vocab, H, std=0.02)
        self.lm_head = rnd(c.vocab, H, std=1.0 / math.sqrt(H))
        self.final_norm = torch.ones(H, device=device)
        self.layers: List[dict] = []
        for li in range(c.layers):
            L = dict(ln1=torch.ones(H, device=device), ln2=torch.ones(H, device=device),
                     wqkv=rnd(3 * H, H, std=1.0 / math.sqrt(H)),
                     wo=rnd(H, H, std=1.0 / math.sqrt(H)),
                     wiq=rnd(c.index_dim, H, std=1.0 / math.sqrt(H)),
                     wik=rnd(c.index_dim, H, std=1.0 / math.sqrt(H)),
                     niq=torch.zeros(c.index_dim, device=device),
                     nik=torch.zeros(c.index_dim, device=device),
                     head_cls=torch.zeros(c.index_dim, device=device))
            if li < c.first_dense:
                L["dense_gu"] = rnd(2 * c.dense_ffn, H, std=1.0 / math.sqrt(H))
                L["dense_d"] = rnd(H, c.dense_ffn, std=1.0 / math.sqrt(c.dense_ffn))
            else:
                L["gate"] = rnd(c.experts, H, std=1.0 / math.sqrt(H))
                L["exp_gu"] = rnd(c.experts, 2 * c.moe_ffn, H, std=1.0 / math.sqrt(H))
                L["exp_d"] = rnd(c.experts, H, c.moe_ffn, std=1.0 / math.sqrt(c.moe_ffn))
                sf = c.shared * c.moe_ffn
                L["sh_gu"] = rnd(2 * sf, H, std=1.0 / math.sqrt(H))
                L["sh_d"] = rnd(H, sf, std=1.0 / math.sqrt(sf))
            self.layers.append(L)
        # paged caches: one block of block_size tokens per page, random block table
        bs = c.block_size
        self.pps = -(-max_len // bs)
        P = batch * self.pps
        self.num_pages = P
        self.block_table = torch.randperm(P, generator=g, device=device).to(torch.int32).view(batch, self.pps).contiguous()
        self.kc = [torch.zeros(P, bs, c.kv_heads, c.head_dim, dtype=bf, device=device) for _ in range(c.layers)]
        self.vc = [torch.zeros_like(self.kc[0]) for _ in range(c.layers)]
        self.ic = [torch.zeros(P, bs, c.index_dim, device=device) for _ in range(c.layers)]
        self.kbar = [torch.zeros(P, c.index_dim, device=device) for _ in range(c.layers)]
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=device)
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim // 2, device=device).float() / (c.head_dim // 2)))
        self.inv_freq = inv
        # decode-step buffers (fixed addresses for graph replay)
        self.tok = torch.zeros(batch, dtype=torch.int64, device=device)
        self.oi = torch.empty(batch, c.slots, dtype=torch.int32, device=device)
        self.ob = torch.empty(batch, c.slots, dtype=torch.float32, device=device)
        self.attn_out = torch.empty(batch, c.heads, c.head_dim, dtype=bf, device=device)
        self.dec_ws = torch.empty(16 << 20, dtype=torch.uint8, device=device)
        self.idx_scale = c.scaling / math.sqrt(c.index_dim)
        # page-aware candidates (image_token_id / page_token_id / per_page_image_tokens)
        self.pst = PS.PageIsolationState(page_cfg, bs) if page_cfg is not None else None
        # page_mask: pass the reference's dense [rows, max_block] allow mask
        # (build_query_allow / decode_allow_fused) instead of the compact domain
        self.page_mask = page_mask
        self.qpage = torch.empty(batch, dtype=torch.int32, device=device)

    # ---------------------------------------------------------------- pieces
    def rope_tables(self, pos):
        ang = pos.float()[:, None] * self.inv_freq[None, :]
        emb = torch.cat([ang, ang], -1)
        return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)

    def slots_of(self, pos, req):
        bs = self.cfg.block_size
        page = self.block_table[req, (pos // bs)].long()
        return page * bs + pos % bs

    def ffn_prefill(self, L, h):
        c = self.cfg
        if "dense_gu" in L:
            g, u = F.linear(h, L["dense_gu"]).chunk(2, -1)
            return F.linear(F.silu(g) * u, L["dense_d"])
        out = torch.zeros(h.shape, dtype=torch.float32, device=h.device)
        g, u = F.linear(h, L["sh_gu"]).chunk(2, -1)
        out += F.linear(F.silu(g) * u, L["sh_d"]).float()
        probs = F.linear(h, L["gate"]).float().softmax(-1)
        w, idx = probs.topk(c.topk, dim=-1)
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=c.experts).tolist()
        tok = order // c.topk
        wt = w.reshape(-1)[order]
        xs = h[tok]
        start = 0
        for e in range(c.experts):
            n = counts[e]
            if n == 0:
                continue
            seg = slice(start, start + n)
            gg, uu = F.linear(xs[seg], L["exp_gu"][e]).chunk(2, -1)
            y = F.linear(F.silu(gg) * uu, L["exp_d"][e]).float() * wt[seg, None]
            out.index_add_(0, tok[seg], y)
            start += n
        return out.to(h.dtype)

    def ffn_decode(self, L, h):
        """Every expert on every decode token, weighted by the (mostly zero)
        gates: static shapes for graph replay; the expert weights are read
        once per step either way."""
        c = self.cfg
        if "dense_gu" in L:
            return self.ffn_prefill(L, h)
        g, u = F.linear(h, L["sh_gu"]).chunk(2, -1)
        out = F.linear(F.silu(g) * u, L["sh_d"]).float()
        probs = F.linear(h, L["gate"]).float().softmax(-1)
        w, idx = probs.topk(c.topk, dim=-1)
        gates = torch.zeros(h.shape[0], c.experts, device=h.device).scatter(1, idx, w)
        gu = torch.matmul(L["exp_gu"], h.t())                       # [E, 2F, B]
        gg, uu = gu.split(c.moe_ffn, dim=1)
        y = torch.matmul(L["exp_d"], F.silu(gg) * uu).float()       # [E, H, B]
        out += (y * gates.t()[:, None, :]).sum(0).t()
        return out.to(h.dtype)

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, embeds: torch.Tensor, attn_events=None, token_ids=None, gen_start=None):
        """embeds [B, S, hidden] bf16 -> logits [B, vocab] of each sequence's
        last token; fills the caches (positions 0..S-1).  With ``token_ids``
        [B, S] and a page configuration, routing is restricted to the blocks of
        each query's own image page; ``gen_start`` [B] marks the positions from
        which tokens count as generated (text pages numbered as responses, as a
        decode step numbers them)."""
        c = self.cfg
        B, S, H = embeds.shape
        T = B * S
        dev = embeds.device
        x = embeds.reshape(T, H).clone()
        req = torch.arange(B, device=dev).repeat_interleave(S)
        pos = torch.arange(S, device=dev).repeat(B)
        cos, sin = self.rope_tables(pos)
        slots = self.slots_of(pos, req)
        self.seq_lens.fill_(S)
        cu = (torch.arange(B + 1, device=dev) * S).to(torch.int32)
        ctx = torch.zeros(B, dtype=torch.int32, device=dev)
        row2req = RT.prefill_row2req(cu_seqlens_q=cu, device=dev, total_q=T)
        plan = RT.kbar_all_plan(block_table=self.block_table, seq_lens=self.seq_lens,
                                context_lens=ctx, block_size=c.block_size, max_block=self.pps,
                                max_query_len=S, device=dev)
        domain = allow = None
        if self.pst is not None and token_ids is not None:
            layout = PS.BatchLayout(num_tokens=T, num_reqs=B,
                                    q_start=torch.arange(B + 1, device=dev) * S,
                                    start_pos=torch.zeros(B, dtype=torch.int64, device=dev),
                                    block_table=self.block_table, req_of_token=req,
                                    gen_start=gen_start)
            q_page = self.pst.step(token_ids.reshape(T), layout, slots,
                                   self.num_pages * c.block_size)
            domain = self.pst.candidate_domain(q_page)
            self.last_q_page = q_page
            if self.page_mask:
                allow = self.pst.build_query_allow(layout, q_page, self.pps, self.num_pages)
                domain = None
        oi = torch.empty(T, c.slots, dtype=torch.int32, device=dev)
        ob = torch.empty(T, c.slots, dtype=torch.float32, device=dev)
        attn = torch.empty(T, c.heads, c.head_dim, dtype=torch.bfloat16, device=dev)
        for li, L in enumerate(self.layers):
            if attn_events is not None:
                attn_events[li][0].record()
            h = rmsnorm(x, L["ln1"], c.eps)
            qkv = F.linear(h, L["wqkv"])
            q, k, v = qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:]
            IF.rope_and_store_kv(q, k, v, cos, sin, self.kc[li], self.vc[li], slots, c.head_dim)
            idx_q, _ = IF.index_qk_fused(h, L["wiq"], L["wik"], L["niq"], L["nik"], c.eps, cos, sin,
                                         index_cache=self.ic[li], slot_mapping=slots)
            RT.kbar_refresh_tail_triton(kv_cache=self.ic[li], k_bar=self.kbar[li],
                                        block_table=self.block_table, seq_lens=self.seq_lens,
                                        head_cls=L["head_cls"], block_size=c.block_size, plan=plan)
            RT.route_prefill_triton(idx_q=idx_q, k_bar=self.kbar[li], block_table=self.block_table,
                                    seq_lens=self.seq_lens, cu_seqlens_q=cu, context_lens=ctx,
                                    row2req=row2req, image_allow=allow, out_idx=oi, out_bias=ob,
                                    max_block=self.pps, block_size=c.block_size,
                                    local_blocks=c.local_blocks, idx_scale=self.idx_scale,
                                    prior_floor=c.prior_floor, sigma=c.sigma, topm=c.topm, budget=c.K,
                                    out_slots=c.slots, page_domain=domain)
            AT.dash_sparse_attn(q.view(T, c.heads, c.head_dim), self.kc[li], self.vc[li],
                                oi[None].expand(c.kv_heads, T, c.slots), ob[None].expand(c.kv_heads, T, c.slots),
                                self.block_table, cu, self.seq_lens, ctx, S, c.kv_heads,
                                1.0 / math.sqrt(c.head_dim), attn, local_blocks=c.local_blocks,
                                sparse_block_size=c.block_size)
            if attn_events is not None:
                attn_events[li][1].record()
            x = x + F.linear(attn.view(T, H), L["wo"])
            x = x + self.ffn_prefill(L, rmsnorm(x, L["ln2"], c.eps))
        self.last_route = (oi, ob)         # the last layer's routes (tests read them)
        last = x.view(B, S, H)[:, -1]
        return F.linear(rmsnorm(last, self.final_norm, c.eps), self.lm_head)

    # ---------------------------------------------------------------- decode
    @torch.no_grad()
    def decode_step(self):
        """One token per sequence: ``self.tok`` at position ``self.seq_lens``;
        returns logits [B, vocab], writes the greedy next token into
        ``self.tok`` and advances ``self.seq_lens``."""
        c = self.cfg
        B, H = self.B, c.hidden
        dev = self.tok.device
        x = self.embed[self.tok]
        pos = self.seq_lens.long()
        req = torch.arange(B, device=dev)
        cos, sin = self.rope_tables(pos)
        slots = self.slots_of(pos, req)
        sl = self.seq_lens + 1
        tail = RT.kbar_tail_plan(block_table=self.block_table, seq_lens=sl,
                                 block_size=c.block_size, tail_pages=1, device=dev)
        domain = allow = None
        if self.pst is not None:
            q_page, _ = DM.decode_meta_fused(input_ids=self.tok, block_table=self.block_table,
                                             seq_lens=sl, slot_mapping=slots, page_state=self.pst,
                                             num_slots=self.num_pages * c.block_size,
                                             block_size=c.block_size, out_q_page=self.qpage)
            domain = self.pst.candidate_domain(q_page)
            if self.page_mask:
                allow = DM.decode_allow_fused(block_table=self.block_table, page_state=self.pst,
                                              q_page=q_page, seq_lens=sl, max_block=self.pps,
                                              num_blocks=self.num_pages, block_size=c.block_size)
                domain = None
        for li, L in enumerate(self.layers):
            h = rmsnorm(x, L["ln1"], c.eps)
            qkv = F.linear(h, L["wqkv"])
            q, k, v = qkv[:, :H], qkv[:, H:2 * H], qkv[:, 2 * H:]
            IF.rope_and_store_kv(q, k, v, cos, sin, self.kc[li], self.vc[li], slots, c.head_dim)
            # index projections + index-K write + k-bar refresh of the tail pages
            idx_q, _ = IF.index_qk_fused(h, L["wiq"], L["wik"], L["niq"], L["nik"], c.eps, cos, sin,
                                         index_cache=self.ic[li], slot_mapping=slots,
                                         kbar_refresh=(self.kbar[li], tail, L["head_cls"],
                                                       c.block_size))
            RT.route_decode_triton(idx_q=idx_q, k_bar=self.kbar[li], block_table=self.block_table,
                                   seq_lens=sl, image_allow=allow, out_idx=self.oi, out_bias=self.ob,
                                   max_block=self.pps, block_size=c.block_size,
                                   local_blocks=c.local_blocks, decode_query_len=1,
                                   idx_scale=self.idx_scale, prior_floor=c.prior_floor,
                                   sigma=c.sigma, topm=c.topm, budget=c.K, out_slots=c.slots,
                                   page_domain=domain)
            AT.dash_sparse_attn_decode(q.view(B, c.heads, c.head_dim), self.kc[li], self.vc[li],
                                       self.oi[None].expand(c.kv_heads, B, c.slots),
                                       self.ob[None].expand(c.kv_heads, B, c.slots), self.block_table,
                                       sl, c.kv_heads, 1.0 / math.sqrt(c.head_dim), self.attn_out, 1,
                                       local_blocks=c.local_blocks, sparse_block_size=c.block_size,
                                       workspace=self.dec_ws)
            x = x + F.linear(self.attn_out.view(B, H), L["wo"])
            x = x + self.ffn_decode(L, rmsnorm(x, L["ln2"], c.eps))
        logits = F.linear(rmsnorm(x, self.final_norm, c.eps), self.lm_head)
        self.tok.copy_(logits.argmax(-1))
        self.seq_lens.add_(1)
        return logits
