"""The allocation-free decode entry point (dash_decode_attn_noalloc).

It serves callers that cannot allocate device memory for the split scratch
(a host whose device memory is owned by its own pool, or a bare FFI consumer
with no allocator): the scratch is a fixed array inside the library.  This
file is collected last on purpose; the test must pass both alone in a fresh
process and after every other test.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from ananta_ocr_b200 import _lib as L
from ananta_ocr_b200 import ops
from dash_testutil import assert_close_bf16
from oracle import dash_oracle as O

pytestmark = pytest.mark.gpu


def _decode_args(q, kc, vc, bt, sl, idx, bias, out, H, Hkv, bs, lw, splits):
    R = q.shape[0]
    a = L.DashDecodeArgs()
    a.seqs = ops.Seqs(n_seq=R, q_len=1, kv_len=0, kv_len_t=sl, max_q_len=1).c()
    a.kv = ops._kv(kc, vc, bt, Hkv, (kc.stride(0), kc.stride(1), kc.stride(2)))
    a.routes = ops._routes(idx, bias, idx.stride(0), 0, 1)
    a.qo = ops._qo(q, out, (q.stride(0), q.stride(0), q.stride(1)),
                   (out.stride(0), out.stride(0), out.stride(1)), H)
    a.scale, a.block_size, a.local_window, a.num_splits = 1.0 / math.sqrt(128), bs, lw, splits
    return a


def _problem():
    g = torch.Generator(device="cuda").manual_seed(5)
    R, H, D, bs, lb, K = 24, 4, 128, 64, 4, 16
    seq = torch.randint(300, 4000, (R,), generator=g, device="cuda").to(torch.int32)
    nb = -(-4000 // bs)
    P = R * nb
    kc = (torch.randn(P, bs, H, D, generator=g, device="cuda") * 0.5).bfloat16()
    vc = (torch.randn(P, bs, H, D, generator=g, device="cuda") * 0.5).bfloat16()
    bt = torch.randperm(P, generator=g, device="cuda").to(torch.int32).view(R, nb).contiguous()
    q = torch.randn(R, H, D, generator=g, device="cuda").bfloat16()
    idx = torch.full((R, K), -1, dtype=torch.int32, device="cuda")
    sl = seq.cpu().numpy()
    rng = np.random.default_rng(0)
    for r in range(R):
        hi = (int(sl[r]) - 1 - lb * bs) // bs
        c = rng.choice(hi + 1, size=min(K, hi + 1), replace=False)
        idx[r, :len(c)] = torch.from_numpy(np.sort(c).astype(np.int32))
    bias = torch.randn(R, K, generator=g, device="cuda")
    return q, kc, vc, bt, seq, idx, bias, H, bs, lb * bs


def _oracle(q, kc, vc, bt, sl, idx, bias, bs, lw):
    """The CPU restatement of the reference's paged decode on the same inputs."""
    R = q.shape[0]
    return O.attend_paged(q.float().cpu().numpy(), kc.float().cpu().numpy(),
                          vc.float().cpu().numpy(), idx.cpu().numpy(), bias.cpu().numpy(),
                          bt.cpu().numpy(), np.arange(R), sl.cpu().numpy().astype(np.int64) - 1,
                          bs, lw, 1.0 / math.sqrt(128))


@pytest.mark.parametrize("splits", [4, 0])
def test_noalloc_decode_matches_workspace_entry_point(splits):
    """Two allocation-free calls in a row (the second sees the first one's
    leftovers in the shared scratch) against the workspace entry point and the
    oracle; splits 0 lets the library choose the split count."""
    lib = L.load()
    stream = L.current_stream()
    q, kc, vc, bt, sl, idx, bias, H, bs, lw = _problem()
    ref = torch.empty_like(q)
    a = _decode_args(q, kc, vc, bt, sl, idx, bias, ref, H, H, bs, lw, splits)
    need = lib.dash_decode_workspace_size(C.byref(a))
    assert need <= lib.dash_noalloc_scratch_bytes()
    if splits:
        assert need > 0
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    assert lib.dash_decode_attn(C.byref(a), stream) == L.DASH_OK, L.last_error()
    outs = []
    for _ in range(2):                       # two calls in a row share the static scratch
        out = torch.full_like(q, float("nan"))
        b = _decode_args(q, kc, vc, bt, sl, idx, bias, out, H, H, bs, lw, splits)
        assert lib.dash_decode_attn_noalloc(C.byref(b), stream) == L.DASH_OK, L.last_error()
        outs.append(out)
    torch.cuda.synchronize()
    want = _oracle(q, kc, vc, bt, sl, idx, bias, bs, lw)
    assert_close_bf16(ref.float().cpu().numpy(), want)
    for out in outs:
        assert_close_bf16(out.float().cpu().numpy(), ref.float().cpu().numpy())
        assert_close_bf16(out.float().cpu().numpy(), want)


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    lib = L.load()
    q, kc, vc, bt, sl, idx, bias, H, bs, lw = _problem()
    out = torch.empty_like(q)
    a = _decode_args(q, kc, vc, bt, sl, idx, bias, out, H, H, bs, lw, 64)
    a.seqs.n_seq = 4096                       # host-side size check only; nothing launches
    a.seqs.kv_len = None
    a.seqs.kv_len_fixed = 4000
    assert lib.dash_decode_workspace_size(C.byref(a)) > lib.dash_noalloc_scratch_bytes()
    rc = lib.dash_decode_attn_noalloc(C.byref(a), L.current_stream())
    assert rc == L.DASH_ERR_WORKSPACE
    assert "fixed" in L.last_error()


def test_noalloc_decode_replays_in_a_cuda_graph():
    """The documented serving pattern: one call on the device first (outside
    any capture), then the call captured in a CUDA graph and replayed with new
    queries written in place; each replay equals the workspace entry point on
    the same queries."""
    lib = L.load()
    q, kc, vc, bt, sl, idx, bias, H, bs, lw = _problem()
    out = torch.empty_like(q)
    a = _decode_args(q, kc, vc, bt, sl, idx, bias, out, H, H, bs, lw, 0)
    assert lib.dash_decode_attn_noalloc(C.byref(a), L.current_stream()) == L.DASH_OK, L.last_error()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rc = lib.dash_decode_attn_noalloc(C.byref(a), L.current_stream())
    assert rc == L.DASH_OK, L.last_error()
    gen = torch.Generator(device="cuda").manual_seed(11)
    for _ in range(2):
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda").bfloat16())
        out.fill_(float("nan"))
        g.replay()
        ref = torch.empty_like(q)
        b = _decode_args(q, kc, vc, bt, sl, idx, bias, ref, H, H, bs, lw, 0)
        need = lib.dash_decode_workspace_size(C.byref(b))
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda")
        b.workspace, b.workspace_bytes = ws.data_ptr(), ws.numel()
        assert lib.dash_decode_attn(C.byref(b), L.current_stream()) == L.DASH_OK, L.last_error()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), "graph replay differs from the workspace entry point"
    del g
