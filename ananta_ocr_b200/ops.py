"""Tensor-level wrappers around the C ABI (torch tensors in, kernels launched on
the current CUDA stream).  Every function requires CUDA tensors and raises on
any non-zero library status; there is no CPU path.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L

_DT = {torch.bfloat16: L.DTYPE_BF16, torch.float16: L.DTYPE_F16, torch.float32: L.DTYPE_F32}


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("DASH B200 kernels need CUDA tensors (no CPU fallback)")


@dataclass
class Seqs:
    """Query/sequence packing (mirrors DashSeqs).

    fixed: ``n_seq`` sequences of ``q_len`` query rows each, keys ``kv_len``.
    varlen: ``q_start`` int32 [n_seq+1] (cu_seqlens_q), optional ``pos0`` and
    ``kv_len_t`` int32 [n_seq] device tensors, ``total_rows`` and ``max_q_len``
    given by the caller (no host sync)."""
    n_seq: int
    q_len: int = 0
    kv_len: int = 0
    q_start: Optional[torch.Tensor] = None
    pos0: Optional[torch.Tensor] = None
    kv_len_t: Optional[torch.Tensor] = None
    total_rows: int = 0
    max_q_len: int = 0

    @property
    def rows(self) -> int:
        return self.total_rows if self.q_start is not None else self.n_seq * self.q_len

    def c(self) -> L.DashSeqs:
        s = L.DashSeqs()
        s.n_seq = self.n_seq
        if self.q_start is not None:
            s.q_len_fixed = self.total_rows
            s.max_q_len = self.max_q_len
        else:
            s.q_len_fixed = self.q_len
            s.max_q_len = max(self.max_q_len, self.q_len)
        s.kv_len_fixed = self.kv_len
        s.q_start = _ptr(self.q_start)
        s.pos0 = _ptr(self.pos0)
        s.kv_len = _ptr(self.kv_len_t)
        return s


class DeviceErrorWord:
    """16 bytes of device memory the kernels write DASH_DEV_* codes into."""

    def __init__(self, device):
        self.t = torch.zeros(2, dtype=torch.int64, device=device)

    @property
    def ptr(self):
        return self.t.data_ptr()

    def read(self):
        v = self.t.cpu()
        code = int(v[0] & 0xFFFFFFFF)
        where = int((v[0] >> 32) & 0xFFFFFFFF)
        return code, where, int(v[1])

    def check(self):
        code, where, info = self.read()
        if code:
            raise RuntimeError(f"DASH device error {code} at site {where} (value {info})")

    def clear(self):
        self.t.zero_()


def selftest_bounded_wait(device_error: DeviceErrorWord, limit_ms: float = 50.0) -> None:
    """Runs the library's bounded-wait self-test on the current stream: a
    kernel waits for a barrier phase that never completes and must give up
    after ``limit_ms`` with DASH_DEV_TIMEOUT in ``device_error``."""
    rc = L.load().dash_selftest_bounded_wait(int(limit_ms * 1e6), device_error.ptr, L.current_stream())
    if rc != L.DASH_OK:
        raise L.DashError(rc, L.last_error())


# ---------------------------------------------------------------------------
# stage-0 pooling
# ---------------------------------------------------------------------------
def kbar_pool_contig(idx_k: torch.Tensor, head_cls: Optional[torch.Tensor], block_size: int,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """idx_k [B,S,d] (fp32/bf16, unit inner stride) -> k-bar [B,nblk,d] fp32."""
    _need_cuda(idx_k)
    B, S, d = idx_k.shape
    if idx_k.stride(2) != 1:
        idx_k = idx_k.contiguous()
    nblk = (S + block_size - 1) // block_size
    if out is None:
        out = torch.empty(B, nblk, d, dtype=torch.float32, device=idx_k.device)
    hc = None if head_cls is None else head_cls.detach().to(idx_k.device, torch.float32).contiguous()
    a = L.DashKbarArgs()
    a.keys = idx_k.data_ptr()
    a.dtype = _DT[idx_k.dtype]
    a.d, a.block_size, a.n_seq, a.seq_len, a.n_plan = d, block_size, B, S, 0
    a.tok_stride, a.seq_stride, a.page_stride = idx_k.stride(1), idx_k.stride(0), 0
    a.kbar_seq_rows = out.stride(0) // out.stride(1)
    a.head_cls = _ptr(hc)
    a.pages = a.ntok = None
    a.kbar = out.data_ptr()
    a.kbar_row_stride = out.stride(1)
    L.call("dash_kbar_pool", a)
    return out


def _kbar_paged_args(index_cache, pages, ntok, head_cls, kbar):
    """DashKbarArgs of a paged refresh plan, with the tensors it points into."""
    _need_cuda(index_cache, pages, ntok, kbar)
    P, bs, d = index_cache.shape
    pages = pages.to(torch.int64).contiguous()
    ntok = ntok.to(torch.int32).contiguous()
    hc = None if head_cls is None else head_cls.detach().to(index_cache.device, torch.float32).contiguous()
    a = L.DashKbarArgs()
    a.keys = index_cache.data_ptr()
    a.dtype = _DT[index_cache.dtype]
    a.d, a.block_size, a.n_seq, a.seq_len, a.n_plan = d, bs, 0, 0, int(pages.numel())
    a.tok_stride, a.seq_stride, a.page_stride = index_cache.stride(1), 0, index_cache.stride(0)
    a.kbar_seq_rows = 0
    a.head_cls = _ptr(hc)
    a.pages, a.ntok = pages.data_ptr(), ntok.data_ptr()
    a.kbar, a.kbar_row_stride = kbar.data_ptr(), kbar.stride(0)
    return a, (pages, ntok, hc)


def kbar_pool_paged(index_cache: torch.Tensor, pages: torch.Tensor, ntok: torch.Tensor,
                    head_cls: Optional[torch.Tensor], kbar: torch.Tensor) -> torch.Tensor:
    """Refresh kbar[page] from index_cache [P, bs, d] for each (page, ntok) entry."""
    a, keep = _kbar_paged_args(index_cache, pages, ntok, head_cls, kbar)
    if a.n_plan:
        L.call("dash_kbar_pool", a)
    return kbar


# ---------------------------------------------------------------------------
# routing
# ---------------------------------------------------------------------------
def route(seqs: Seqs, *, width: int, block_size: int, local_blocks: int, idx_scale: float,
          prior_floor: float, sigma: float, topm: int, K: int,
          idx_q: Optional[torch.Tensor] = None, kbar: Optional[torch.Tensor] = None,
          block_table: Optional[torch.Tensor] = None, scores_in: Optional[torch.Tensor] = None,
          cand: Optional[torch.Tensor] = None, cand_per_seq: bool = False,
          out_idx: Optional[torch.Tensor] = None, out_bias: Optional[torch.Tensor] = None,
          out_width: Optional[int] = None, scores_out: Optional[torch.Tensor] = None,
          out_count: Optional[torch.Tensor] = None, device_error: Optional[DeviceErrorWord] = None,
          page=None, refresh=None):
    """Fused DASH routing for ``seqs.rows`` query rows.

    Either ``scores_in`` [rows, width] (precomputed block scores) or ``idx_q``
    [rows, d] + ``kbar`` (contiguous [n_seq, nblk, d] or a page cache [P, d]
    addressed through ``block_table`` [n_seq, W]).  ``page`` (a
    ``pages.PageDomain``) restricts the candidates to the blocks holding image
    tokens of each row's page (instead of ``cand``).  ``refresh`` (index_cache
    [P, bs, d], pages, ntok, head_cls) refreshes those k-bar rows of the page
    cache in the same launch (``dash_route_refresh``); the rows must not be
    scored by this call (a decode step's tail pages, inside every row's local
    window).  Returns (idx int32 [rows, out_width] ascending with -1 tail, bias
    fp32 [rows, out_width])."""
    ref = scores_in if scores_in is not None else idx_q
    _need_cuda(ref, kbar, block_table, cand)
    dev = ref.device
    rows = seqs.rows
    ow = out_width or K
    if out_idx is None:
        out_idx = torch.empty(rows, ow, dtype=torch.int32, device=dev)
    if out_bias is None:
        out_bias = torch.empty(rows, ow, dtype=torch.float32, device=dev)
    a = L.DashRouteArgs()
    a.seqs = seqs.c()
    if scores_in is None:
        if idx_q.dtype != torch.float32 or idx_q.stride(-1) != 1:
            idx_q = idx_q.float().contiguous()
        a.idx_q, a.q_row_stride = idx_q.data_ptr(), idx_q.stride(0)
        a.d = idx_q.shape[-1]
        if block_table is not None:
            a.kbar, a.kbar_row_stride = kbar.data_ptr(), kbar.stride(0)
            a.block_table, a.bt_stride = block_table.data_ptr(), block_table.stride(0)
            a.num_kbar_rows = kbar.shape[0]
        else:
            a.kbar, a.kbar_row_stride = kbar.data_ptr(), kbar.stride(1)
            a.kbar_seq_rows = kbar.stride(0) // kbar.stride(1)
            a.num_kbar_rows = kbar.shape[0] * a.kbar_seq_rows
    else:
        scores_in = scores_in if scores_in.stride(-1) == 1 else scores_in.contiguous()
        a.scores_in, a.scores_in_stride = scores_in.data_ptr(), scores_in.stride(0)
        a.d = 128
    a.width = width
    if scores_out is not None:
        a.scores_out, a.scores_out_stride = scores_out.data_ptr(), scores_out.stride(0)
    if cand is not None:
        cand = cand.to(torch.uint8).contiguous()
        a.cand, a.cand_row_stride, a.cand_per_seq = cand.data_ptr(), cand.stride(0), int(cand_per_seq)
    a.block_size, a.local_blocks, a.topm, a.K, a.out_width = block_size, local_blocks, topm, K, ow
    a.idx_scale, a.prior_floor, a.inv_sigma = float(idx_scale), float(prior_floor), float(1.0 / sigma)
    a.out_idx, a.out_bias, a.out_stride = out_idx.data_ptr(), out_bias.data_ptr(), out_idx.stride(0)
    assert out_bias.stride(0) == out_idx.stride(0)
    a.out_count = _ptr(out_count)
    a.device_error = device_error.ptr if device_error is not None else None
    if page is not None:
        _need_cuda(page.q_page, page.lo, page.hi, page.bits)
        for t in (page.q_page, page.lo, page.hi):
            if t.dtype != torch.int32 or not t.is_contiguous():
                raise ValueError("page domain tensors must be contiguous int32")
        a.page_q, a.page_lo, a.page_hi = page.q_page.data_ptr(), page.lo.data_ptr(), page.hi.data_ptr()
        if page.bits is not None:
            a.page_bits, a.page_bits_words = page.bits.data_ptr(), page.bits.shape[-1]
        a.page_seq_rows = page.seq_rows if block_table is None else 0
        a.num_page_desc = page.lo.numel()
    if refresh is None:
        L.call("dash_route", a)
        return out_idx, out_bias
    if block_table is None:
        raise ValueError("the folded k-bar refresh needs the paged k-bar cache (block_table)")
    ka, keep = _kbar_paged_args(*refresh, kbar)
    lib = L.load()
    rc = lib.dash_route_refresh(ctypes.byref(a), ctypes.byref(ka) if ka.n_plan else None, L.current_stream())
    if rc != L.DASH_OK:
        raise L.DashError(rc, L.last_error())
    return out_idx, out_bias


def block_max(q: torch.Tensor, k: torch.Tensor, pos: torch.Tensor, seg: Optional[torch.Tensor],
              block_size: int, nblk: int, local_window: int, clamp: bool, empty: float):
    """Indexer stage-0 block-max scores: q [B,C,d], k [B,Sk,d] fp32 -> [B,C,nblk]."""
    _need_cuda(q, k, pos, seg)
    q = q.float().contiguous()
    k = k.float().contiguous()
    B, Cq, d = q.shape
    pos = pos.to(torch.int32).contiguous()
    seg = None if seg is None else seg.to(torch.int32).contiguous()
    out = torch.empty(B, Cq, nblk, dtype=torch.float32, device=q.device)
    a = L.DashBlockMaxArgs()
    a.q, a.q_stride_b, a.q_stride_c = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_b, a.k_stride_j = k.data_ptr(), k.stride(0), k.stride(1)
    a.pos, a.pos_stride_b, a.pos_stride_c = pos.data_ptr(), pos.stride(0), pos.stride(1)
    if seg is not None:
        a.seg, a.seg_stride_b, a.seg_stride_c = seg.data_ptr(), seg.stride(0), seg.stride(1)
    a.B, a.C, a.Sk, a.d = B, Cq, k.shape[1], d
    a.block_size, a.nblk, a.local_window, a.clamp = block_size, nblk, local_window, int(clamp)
    a.empty = float(empty)
    a.out, a.out_stride_b, a.out_stride_c = out.data_ptr(), out.stride(0), out.stride(1)
    L.call("dash_block_max", a)
    return out


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def _kv(k, v, block_table, n_kv_heads, paged_layout):
    """DashKV from tensors.  contiguous: k/v indexable as [seq, tok, head, d] via
    strides; paged: caches [P, page, Hkv, d]."""
    kv = L.DashKV()
    kv.k, kv.v = k.data_ptr(), v.data_ptr()
    kv.dtype = _DT[k.dtype]
    kv.n_kv_heads = n_kv_heads
    kv.head_dim = k.shape[-1]
    st = paged_layout
    assert k.stride() == v.stride(), "K and V must share strides"
    kv.stride_seq, kv.stride_tok, kv.stride_head = st
    if block_table is not None:
        kv.block_table, kv.bt_stride = block_table.data_ptr(), block_table.stride(0)
        kv.num_pages = k.shape[0]
    return kv


def _routes(idx, bias, row_stride, ihead_stride, n_index_heads):
    r = L.DashRoutes()
    r.idx = _ptr(idx)
    r.bias = _ptr(bias)
    r.row_stride, r.ihead_stride = row_stride, ihead_stride
    r.K = 0 if idx is None else idx.shape[-1]
    r.n_index_heads = n_index_heads
    return r


def _qo(q, out, q_strides, o_strides, n_heads, lse=None, lse_strides=(0, 0, 0)):
    qo = L.DashQO()
    qo.q, qo.out = q.data_ptr(), out.data_ptr()
    qo.q_stride_seq, qo.q_stride_tok, qo.q_stride_head = q_strides
    qo.o_stride_seq, qo.o_stride_tok, qo.o_stride_head = o_strides
    qo.n_heads = n_heads
    qo.lse = _ptr(lse)
    qo.lse_stride_seq, qo.lse_stride_tok, qo.lse_stride_head = lse_strides
    return qo


_WS = {}


def _workspace(device, nbytes, key):
    """Grow-only workspace cache per (device, current stream, key): kernels on
    different streams may run at the same time, so each stream has its own
    scratch (a buffer is only ever reused in its stream's order).  Callers that
    must not allocate pass their own buffer instead."""
    sid = torch.cuda.current_stream(device).cuda_stream
    buf = _WS.get((device, sid, key))
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _WS[(device, sid, key)] = buf
    return buf


# Prefill work split (DashPrefillArgs.mode) for calls that leave it at 0:
# 0 automatic, 1 tile-major, 2 routed part gathered by key block.
PREFILL_MODE = 0


@contextlib.contextmanager
def prefill_mode(mode: int, part_budget_mib: int = 0):
    """Within the block, prefill calls use ``mode`` (and the gathered mode's
    partial scratch budget in MiB, 0 = the library default)."""
    global PREFILL_MODE, PREFILL_PART_MIB
    old = PREFILL_MODE, PREFILL_PART_MIB
    PREFILL_MODE, PREFILL_PART_MIB = int(mode), int(part_budget_mib)
    try:
        yield
    finally:
        PREFILL_MODE, PREFILL_PART_MIB = old


PREFILL_PART_MIB = 0


def _apply_prefill_mode(args: L.DashPrefillArgs) -> None:
    if args.mode == 0:
        args.mode = PREFILL_MODE
    if args.part_budget_mib == 0:
        args.part_budget_mib = PREFILL_PART_MIB


def prefill_attn(args: L.DashPrefillArgs, device, workspace: Optional[torch.Tensor] = None):
    L.load()
    _apply_prefill_mode(args)
    need = L.load().dash_prefill_workspace_size(args)
    if workspace is None:
        workspace = _workspace(device, need, "prefill")
    args.workspace, args.workspace_bytes = workspace.data_ptr(), workspace.numel()
    L.call("dash_prefill_attn", args)


def decode_attn(args: L.DashDecodeArgs, device, workspace: Optional[torch.Tensor] = None):
    need = L.load().dash_decode_workspace_size(args)
    if need:
        if workspace is None:
            workspace = _workspace(device, need, "decode")
        args.workspace, args.workspace_bytes = workspace.data_ptr(), workspace.numel()
    L.call("dash_decode_attn", args)


def gather_attention(q, k, v, idx, bias, *, block_size: int, local_window: int, scale: float,
                     out=None, lse=None, seg_start=None, n_index_heads: int = 1,
                     device_error: Optional[DeviceErrorWord] = None, workspace=None,
                     peers: Optional[torch.Tensor] = None):
    """Contiguous prefill: q [B,HQ,T,D], k/v [B,Hkv,T,D] (any strides with unit
    inner stride), idx/bias routes [B,HI,T,K] (or [B,T,K]).  Returns out
    [B,HQ,T,D] (a new tensor unless ``out`` is given).  ``peers`` (int64 device
    array, ``peer.PeerGather.peers_for(out)``) also stores every output row
    into the other ranks' copies of ``out``."""
    _need_cuda(q, k, v, idx)
    B, HQ, T, D = q.shape
    Hkv = k.shape[1]
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if idx.dim() == 3:
        idx = idx[:, None]
        bias = None if bias is None else bias[:, None]
    HI = idx.shape[1]
    # rows are (b, t) pairs addressed as row * row_stride + ih * ihead_stride:
    # view the routes as [B, T, HI, K] with equally spaced rows
    idx4 = idx.to(torch.int32).permute(0, 2, 1, 3)
    bias4 = None if bias is None else bias.to(torch.float32).permute(0, 2, 1, 3)

    def _rowable(t):
        return t.stride(3) == 1 and t.stride(0) == T * t.stride(1)

    if not _rowable(idx4) or (bias4 is not None and
                              (not _rowable(bias4) or bias4.stride() != idx4.stride())):
        idx4 = idx4.contiguous()
        bias4 = None if bias4 is None else bias4.contiguous()
    a = L.DashPrefillArgs()
    a.seqs = Seqs(n_seq=B, q_len=T, kv_len=T, max_q_len=T).c()
    a.kv = _kv(k, v, None, Hkv, (k.stride(0), k.stride(2), k.stride(1)))
    a.routes = _routes(idx4, bias4, idx4.stride(1), idx4.stride(2), HI)
    lse_strides = (0, 0, 0) if lse is None else (lse.stride(0), lse.stride(2), lse.stride(1))
    a.qo = _qo(q, out, (q.stride(0), q.stride(2), q.stride(1)),
               (out.stride(0), out.stride(2), out.stride(1)), HQ, lse, lse_strides)
    if seg_start is not None:
        seg_start = seg_start.to(torch.int32).contiguous()
        a.seg_start = seg_start.data_ptr()
    a.scale, a.block_size, a.local_window = float(scale), int(block_size), int(local_window)
    a.device_error = device_error.ptr if device_error is not None else None
    if peers is not None and peers.numel():
        a.out_peers, a.n_peers = peers.data_ptr(), int(peers.numel())
    prefill_attn(a, q.device, workspace)
    return out


def gather_attention_workspace_bytes(B: int, HQ: int, Hkv: int, T: int, K: int, *,
                                     block_size: int, local_window: int,
                                     n_index_heads: int = 1,
                                     dtype: torch.dtype = torch.bfloat16) -> int:
    """Scratch bytes ``gather_attention`` needs for these shapes (under the
    current prefill mode), for callers that size a workspace once."""
    a = L.DashPrefillArgs()
    a.seqs = Seqs(n_seq=B, q_len=T, kv_len=T, max_q_len=T).c()
    a.kv.dtype, a.kv.n_kv_heads, a.kv.head_dim = _DT[dtype], int(Hkv), 128
    a.qo.n_heads = int(HQ)
    a.routes.K, a.routes.n_index_heads = int(K), int(n_index_heads)
    a.block_size, a.local_window = int(block_size), int(local_window)
    _apply_prefill_mode(a)
    return int(L.load().dash_prefill_workspace_size(a))


# ---------------------------------------------------------------------------
# training backward
# ---------------------------------------------------------------------------
def gather_attention_bwd(q, k, v, o, dout, lse, idx, bias, *, block_size: int,
                         local_window: int, scale: float, want_d_bias: bool = True,
                         seg_start: Optional[torch.Tensor] = None,
                         device_error: Optional[DeviceErrorWord] = None):
    """Backward of the contiguous gather attention (``dash_attn_bwd``).

    q, o, dout [B, T, HQ, D]; k, v [B, T, Hkv, D] (made contiguous, one dtype);
    lse [B, T, HQ] fp32 (natural log, from the forward); idx [B, T, K] int
    (-1 unused) or [B, HI, T, K] for HI index heads, bias of the same shape
    fp32 or None; seg_start [B, T] int (packed sequences: row t sees keys
    [seg_start, t]) or None.  Returns (dq, dk, dv, d_bias) with d_bias shaped
    like idx, fp32 (None unless ``want_d_bias``)."""
    _need_cuda(q, k, v, o, dout, lse, idx)
    dt = q.dtype
    q, o, dout = (t.to(dt).contiguous() for t in (q, o, dout))
    k, v = k.to(dt).contiguous(), v.to(dt).contiguous()
    B, T, HQ, D = q.shape
    Hkv = k.shape[2]
    idx = idx.to(torch.int32).contiguous()
    K = idx.shape[-1]
    HI = idx.shape[1] if idx.dim() == 4 else 1
    seg_start = None if seg_start is None else seg_start.to(torch.int32).contiguous()
    bias = None if bias is None else bias.to(torch.float32).contiguous()
    lse = lse.to(torch.float32).contiguous()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    d_bias = torch.empty(idx.shape, dtype=torch.float32, device=q.device) if want_d_bias else None
    delta = torch.empty(B, T, HQ, dtype=torch.float32, device=q.device)
    a = L.DashAttnBwdArgs()
    a.n_seq, a.seq_len, a.n_heads, a.n_kv_heads, a.head_dim = B, T, HQ, Hkv, D
    a.dtype, a.block_size, a.local_window, a.K = _DT[dt], int(block_size), int(local_window), K
    a.scale = float(scale)
    a.n_index_heads = HI
    a.seg_start = _ptr(seg_start)
    words = L.load().dash_attn_bwd_flag_words(ctypes.byref(a))
    if words < 0:
        raise L.DashError(L.DASH_ERR_UNSUPPORTED, L.last_error())
    flags = torch.empty(max(1, words), dtype=torch.int32, device=q.device)
    dq_acc = (torch.empty(B, T, HQ, D, dtype=torch.float32, device=q.device)
              if dt in (torch.bfloat16, torch.float16) else None)
    a.q, a.k, a.v, a.o, a.dout = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr()
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.lse, a.idx, a.bias = lse.data_ptr(), idx.data_ptr(), _ptr(bias)
    a.d_bias, a.delta, a.flags = _ptr(d_bias), delta.data_ptr(), flags.data_ptr()
    a.dq_acc = _ptr(dq_acc)
    a.device_error = device_error.ptr if device_error is not None else None
    L.call("dash_attn_bwd", a)
    return dq, dk, dv, d_bias


def entmax15(x: torch.Tensor) -> torch.Tensor:
    """1.5-entmax over the last dim (``dash_entmax15_fwd``), fp32."""
    _need_cuda(x)
    x = x.to(torch.float32).contiguous()
    y = torch.empty_like(x)
    a = L.DashEntmaxArgs()
    n = x.shape[-1] if x.dim() else 1
    a.x, a.y, a.rows, a.n, a.stride = x.data_ptr(), y.data_ptr(), x.numel() // max(1, n), n, n
    L.call("dash_entmax15_fwd", a)
    return y


def entmax15_backward(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    """Jacobian-vector product of 1.5-entmax (``dash_entmax15_bwd``), fp32."""
    _need_cuda(y, dy)
    y = y.to(torch.float32).contiguous()
    dy = dy.to(torch.float32).contiguous()
    dx = torch.empty_like(y)
    a = L.DashEntmaxArgs()
    n = y.shape[-1]
    a.y, a.dy, a.dx, a.rows, a.n, a.stride = y.data_ptr(), dy.data_ptr(), dx.data_ptr(), y.numel() // max(1, n), n, n
    L.call("dash_entmax15_bwd", a)
    return dx


# ---------------------------------------------------------------------------
# router front end
# ---------------------------------------------------------------------------
def index_proj(hidden: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor,
               norm_q: torch.Tensor, norm_k: torch.Tensor, eps: float, *,
               cos: Optional[torch.Tensor] = None, sin: Optional[torch.Tensor] = None,
               norm_clamp: bool = False, idx_q: Optional[torch.Tensor] = None,
               idx_k: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None,
               device_error: Optional[DeviceErrorWord] = None, kbar_refresh=None):
    """Index projections + RMSNorm + RoPE on tcgen05 (``dash_index_proj``).

    hidden [T, hidden_dim] bf16; w_q/w_k [128, hidden_dim] bf16 (nn.Linear
    weights); norm_q/norm_k [128] (Gemma weights, scale 1 + w); cos/sin
    [T, >=128] bf16 or None.  Returns (idx_q [T, 128] fp32, idx_k): idx_k is
    [T, 128] fp32 unless ``idx_k`` is given -- with ``slot_mapping`` [T] int64
    it is a cache of rows [num_slots, 128] (fp32 or bf16) written at the
    tokens' slots.  ``kbar_refresh`` = (kbar [P, 128] fp32, pages [T] int64,
    ntok [T] int32, head_cls or None, block_size) recomputes, after the write,
    the k-bar row of each token's page (one token per page in this call)."""
    _need_cuda(hidden, w_q, w_k, cos, sin, idx_k, slot_mapping)
    if hidden.dtype != torch.bfloat16 or w_q.dtype != torch.bfloat16 or w_k.dtype != torch.bfloat16:
        raise NotImplementedError("index projections run on bf16 hidden states and weights")
    T, Hd = hidden.shape
    dev = hidden.device
    if hidden.stride(-1) != 1:
        hidden = hidden.contiguous()
    w_q = w_q if w_q.stride(-1) == 1 else w_q.contiguous()
    w_k = w_k if w_k.stride(-1) == 1 else w_k.contiguous()
    if w_q.stride(0) != w_k.stride(0):
        w_k = w_k.contiguous()
        w_q = w_q.contiguous()
    nq = norm_q.to(device=dev, dtype=torch.float32).contiguous()
    nk = norm_k.to(device=dev, dtype=torch.float32).contiguous()
    if idx_q is None:
        idx_q = torch.empty(T, w_q.shape[0], dtype=torch.float32, device=dev)
    if idx_k is None:
        idx_k = torch.empty(T, w_k.shape[0], dtype=torch.float32, device=dev)
    a = L.DashIndexProjArgs()
    a.hidden, a.hidden_stride = hidden.data_ptr(), hidden.stride(0)
    a.w_q, a.w_k, a.w_stride = w_q.data_ptr(), w_k.data_ptr(), w_q.stride(0)
    a.norm_q, a.norm_k = nq.data_ptr(), nk.data_ptr()
    if cos is not None:
        if cos.dtype != torch.bfloat16 or sin.dtype != torch.bfloat16:
            raise NotImplementedError("cos/sin must be bf16 (the model dtype)")
        if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
            cos, sin = cos.contiguous(), sin.contiguous()
        a.cos, a.sin, a.cs_stride = cos.data_ptr(), sin.data_ptr(), cos.stride(0)
    a.eps, a.norm_clamp = float(eps), int(bool(norm_clamp))
    a.T, a.hidden_dim, a.d = T, Hd, w_q.shape[0]
    a.k_dtype = _DT[idx_k.dtype]
    a.idx_q, a.q_stride = idx_q.data_ptr(), idx_q.stride(0)
    a.idx_k, a.k_stride = idx_k.data_ptr(), idx_k.stride(0)
    if slot_mapping is not None:
        sm = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
        a.slot_mapping, a.k_rows = sm.contiguous().data_ptr(), idx_k.shape[0]
    a.device_error = device_error.ptr if device_error is not None else None
    keep = None
    if kbar_refresh is not None:
        kbar, pages, ntok, head_cls, block_size = kbar_refresh
        _need_cuda(kbar, pages, ntok)
        pages = pages.to(torch.int64).contiguous()
        ntok = ntok.to(torch.int32).contiguous()
        hc = None if head_cls is None else head_cls.detach().to(dev, torch.float32).contiguous()
        keep = (pages, ntok, hc)
        a.kbar_page, a.kbar_ntok, a.kbar_head_cls = pages.data_ptr(), ntok.data_ptr(), _ptr(hc)
        a.kbar, a.kbar_row_stride, a.kbar_block_size = kbar.data_ptr(), kbar.stride(0), int(block_size)
    L.call("dash_index_proj", a)
    del keep
    return idx_q, idx_k


def rope_kv_write(q: Optional[torch.Tensor], k: Optional[torch.Tensor], cos: Optional[torch.Tensor],
                  sin: Optional[torch.Tensor], *, v: Optional[torch.Tensor] = None,
                  q_out: Optional[torch.Tensor] = None, k_cache: Optional[torch.Tensor] = None,
                  v_cache: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None,
                  head_dim: int = 128, device_error: Optional[DeviceErrorWord] = None):
    """Rotate-half RoPE of q [T, Hq*D] and k [T, Hkv*D] (bf16, every product and
    the sum rounded to bf16) with k (rotated) and v written to the cache rows
    ``slot_mapping`` (``dash_rope_kv_write``).  Without caches, k goes to a
    new [T, Hkv*D] tensor.  Returns (q_out, k_dest)."""
    _need_cuda(q, k, v, cos, sin, k_cache, v_cache, slot_mapping)
    ref = q if q is not None else k
    T = ref.shape[0]
    a = L.DashRopeKVArgs()
    a.T, a.head_dim = T, head_dim
    if q is not None:
        if q.stride(-1) != 1:
            q = q.contiguous()
        if q_out is None:
            q_out = torch.empty_like(q)
        a.q, a.q_stride, a.q_out, a.q_out_stride = q.data_ptr(), q.stride(0), q_out.data_ptr(), q_out.stride(0)
        a.n_q_heads = q.shape[1] // head_dim
    if k is not None:
        if k.stride(-1) != 1:
            k = k.contiguous()
        a.k, a.k_stride, a.n_kv_heads = k.data_ptr(), k.stride(0), k.shape[1] // head_dim
        if k_cache is None:
            k_cache = torch.empty_like(k)
        kc = k_cache if k_cache.dim() == 2 else k_cache.reshape(-1, a.n_kv_heads * head_dim)
        a.k_cache, a.cache_row_stride, a.num_slots = kc.data_ptr(), kc.stride(0), kc.shape[0]
        if v is not None:
            if v.stride(-1) != 1:
                v = v.contiguous()
            vc = v_cache.reshape(kc.shape) if v_cache.dim() != 2 else v_cache
            if vc.stride(0) != kc.stride(0):
                raise ValueError("k_cache and v_cache rows must share a stride")
            a.v, a.v_stride, a.v_cache = v.data_ptr(), v.stride(0), vc.data_ptr()
    if cos is not None:
        if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
            cos, sin = cos.contiguous(), sin.contiguous()
        a.cos, a.sin, a.cs_stride = cos.data_ptr(), sin.data_ptr(), cos.stride(0)
    if slot_mapping is not None:
        sm = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
        a.slot_mapping = sm.contiguous().data_ptr()
    a.device_error = device_error.ptr if device_error is not None else None
    L.call("dash_rope_kv_write", a)
    return q_out, k_cache
