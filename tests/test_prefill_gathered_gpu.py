"""Prefill with the routed part gathered by key block (DashPrefillArgs.mode 2:
the routed kernel's partials merged into the window kernel's epilogue)
against the oracle: block sizes 32/64/128, 1/2/4 query heads per kv head,
messy route lists, windows longer than the sequence, partial budgets small
enough to split the work into chunks of sequences, tile pairs and kv heads,
packing with two index heads, the paged serving layout with prefixes, and
the log-sum-exp output.  The same inputs through mode 1 (tile-major) must
agree with mode 2 to bf16 rounding."""
import math

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from ananta_ocr_b200 import ops
from ananta_ocr_b200.sparse_gather_triton import triton_gather_attention
from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn
from dash_testutil import assert_close_bf16, bf16_round, random_routes

pytestmark = pytest.mark.gpu

CASES = [
    # B, H, Hkv, T, bs, LW, K
    (2, 2, 2, 700, 64, 256, 4),
    (1, 4, 2, 1000, 128, 256, 3),     # G=2, block 128
    (1, 1, 1, 129, 64, 64, 2),        # tiny, ragged tail
    (1, 2, 2, 100, 64, 256, 4),       # window longer than the sequence: no partials
    (2, 4, 1, 777, 64, 192, 6),       # G=4
    (2, 2, 2, 700, 32, 128, 12),      # 32-token blocks
    (1, 4, 2, 1000, 32, 128, 16),
    (1, 1, 1, 129, 32, 128, 3),
    (2, 3, 3, 777, 32, 100, 12),      # window ends inside a block
    (1, 8, 2, 900, 32, 96, 5),        # G=4, 32-token blocks
    (1, 2, 1, 1500, 128, 1024, 64),   # config-4 window / K on a short sequence
    (1, 2, 2, 2100, 64, 256, 40),     # K > 32: two list registers per lane
]


def _inputs(seed, B, H, Hkv, T, D=128):
    rng = np.random.default_rng(seed)
    q = bf16_round((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32))
    k = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    v = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    return rng, q, k, v


def _run(q, k, v, idx, bias, bs, LW, mode, budget=0, lse=None):
    D = q.shape[-1]
    with ops.prefill_mode(mode, budget):
        return ops.gather_attention(torch.from_numpy(q).cuda().bfloat16(),
                                    torch.from_numpy(k).cuda().bfloat16(),
                                    torch.from_numpy(v).cuda().bfloat16(),
                                    torch.from_numpy(idx).cuda(),
                                    None if bias is None else torch.from_numpy(bias).cuda(),
                                    block_size=bs, local_window=LW, scale=1.0 / math.sqrt(D),
                                    lse=lse)


@pytest.mark.parametrize("B,H,Hkv,T,bs,LW,K", CASES)
def test_gathered_vs_oracle(B, H, Hkv, T, bs, LW, K):
    rng, q, k, v = _inputs(B * 1000 + T + K, B, H, Hkv, T)
    idx, bias = random_routes(rng, B, T, K, bs, LW)
    out = _run(q, k, v, idx, bias, bs, LW, 2)
    ref = O.attend_contig(q, k, v, idx[:, 0], bias[:, 0], bs, LW, 1.0 / math.sqrt(q.shape[-1]))
    assert_close_bf16(out.float().cpu().numpy(), ref)
    # the tile-major split gives the same result up to bf16 rounding
    out1 = _run(q, k, v, idx, bias, bs, LW, 1)
    assert_close_bf16(out.float().cpu().numpy(), out1.float().cpu().numpy())


@pytest.mark.parametrize("budget", [1, 3, 16, 40])
def test_gathered_chunks(budget):
    """Budgets of 1/3/16/40 MiB split the work into chunks of one tile pair,
    two tile pairs, one sequence, and every sequence of one kv head."""
    B, H, Hkv, T, bs, LW, K = 3, 4, 2, 1300, 64, 192, 16
    rng, q, k, v = _inputs(budget, B, H, Hkv, T)
    idx, bias = random_routes(rng, B, T, K, bs, LW)
    out = _run(q, k, v, idx, bias, bs, LW, 2, budget)
    ref = O.attend_contig(q, k, v, idx[:, 0], bias[:, 0], bs, LW, 1.0 / math.sqrt(q.shape[-1]))
    assert_close_bf16(out.float().cpu().numpy(), ref)


def test_gathered_no_bias_and_lse():
    B, H, Hkv, T, bs, LW, K = 2, 4, 4, 900, 64, 128, 8
    rng, q, k, v = _inputs(11, B, H, Hkv, T)
    idx, _ = random_routes(rng, B, T, K, bs, LW)
    lse = torch.empty(B, H, T, device="cuda")
    out = _run(q, k, v, idx, None, bs, LW, 2, lse=lse)
    ref, ref_lse = O.attend_contig(q, k, v, idx[:, 0], None, bs, LW, 1.0 / math.sqrt(128),
                                   return_lse=True)
    assert_close_bf16(out.float().cpu().numpy(), ref)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


def test_gathered_index_heads_and_packing():
    """Two index heads (one per kv head) and two packed segments per row:
    routed keys before a row's segment start are masked in the partials."""
    rng = np.random.default_rng(4)
    B, H, Hkv, T, D, bs, LW, K = 1, 4, 2, 1400, 128, 64, 128, 5
    q = bf16_round((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32))
    k = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    v = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    idx, _ = random_routes(rng, B, T, K, bs, LW, n_index_heads=2)
    split = 650
    pos = np.concatenate([np.arange(split), np.arange(T - split)])[None]
    with ops.prefill_mode(2):
        out = triton_gather_attention(torch.from_numpy(q).cuda().bfloat16(),
                                      torch.from_numpy(k).cuda().bfloat16(),
                                      torch.from_numpy(v).cuda().bfloat16(),
                                      torch.from_numpy(idx).cuda(), torch.from_numpy(pos).cuda(),
                                      None, bs, 1.0 / math.sqrt(D), LW)
    seg = (np.arange(T)[None] - pos)
    got = out.float().cpu().numpy()
    for ih in range(2):
        hs = slice(ih * 2, ih * 2 + 2)
        ref = O.attend_contig(q[:, hs], k[:, ih:ih + 1], v[:, ih:ih + 1], idx[:, ih], None, bs,
                              LW, 1.0 / math.sqrt(D), seg=seg)
        assert_close_bf16(got[:, hs], ref)


@pytest.mark.parametrize("bs,lb,G", [(64, 4, 2), (128, 2, 1), (32, 4, 4), (32, 1, 2)])
def test_gathered_paged_with_prefix(bs, lb, G):
    rng = np.random.default_rng(bs + G)
    D, Hkv, K = 128, 2, 6
    H = Hkv * G
    seq_lens = np.array([2300, 300, 3100])
    ctx = np.array([200, 0, 1000])
    R = len(seq_lens)
    W = int(-(-seq_lens.max() // bs))
    P = 3 * W + 5
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((R, W), np.int32)
    n = 0
    for r in range(R):
        nb = -(-int(seq_lens[r]) // bs)
        bt[r, :nb] = perm[n:n + nb]
        n += nb
    kc = bf16_round((rng.standard_normal((P, bs, Hkv, D)) * 0.5).astype(np.float32))
    vc = bf16_round((rng.standard_normal((P, bs, Hkv, D)) * 0.5).astype(np.float32))
    q_lens = seq_lens - ctx
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    total_q = int(cu[-1])
    q = bf16_round((rng.standard_normal((total_q, H, D)) * 0.5).astype(np.float32))
    row_req = np.repeat(np.arange(R), q_lens)
    row_pos = np.concatenate([np.arange(ctx[r], seq_lens[r]) for r in range(R)])
    idx = np.full((total_q, K), -1, np.int32)
    bias = (rng.standard_normal((total_q, K))).astype(np.float32)
    for i in range(total_q):
        hi = (row_pos[i] - lb * bs) // bs
        if hi >= 0:
            c = rng.choice(hi + 1, size=min(K, hi + 1), replace=False)
            idx[i, :len(c)] = c                     # unsorted on purpose
    out = torch.zeros(total_q, H, D, dtype=torch.bfloat16, device="cuda")
    ti = torch.from_numpy(idx).cuda()[None].expand(Hkv, -1, -1)
    tb = torch.from_numpy(bias).cuda()[None].expand(Hkv, -1, -1)
    with ops.prefill_mode(2):
        dash_sparse_attn(torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(kc).cuda().bfloat16(),
                         torch.from_numpy(vc).cuda().bfloat16(), ti, tb, torch.from_numpy(bt).cuda(),
                         torch.from_numpy(cu).cuda(), torch.from_numpy(seq_lens.astype(np.int32)).cuda(),
                         torch.from_numpy(ctx.astype(np.int32)).cuda(), int(q_lens.max()), Hkv,
                         1.0 / math.sqrt(D), out, local_blocks=lb, sparse_block_size=bs)
    ref = O.attend_paged(q, kc, vc, idx, bias, bt, row_req, row_pos, bs, lb * bs, 1.0 / math.sqrt(D))
    assert_close_bf16(out.float().cpu().numpy(), ref)


def test_gathered_rejects_unsupported():
    """Mode 2 with 8 query heads per kv head (tiles of 16 tokens) is refused."""
    B, H, Hkv, T, bs, LW, K = 1, 8, 1, 300, 64, 128, 4
    rng, q, k, v = _inputs(1, B, H, Hkv, T)
    idx, bias = random_routes(rng, B, T, K, bs, LW)
    from ananta_ocr_b200 import _lib as L
    with pytest.raises(L.DashError):
        _run(q, k, v, idx, bias, bs, LW, 2)
