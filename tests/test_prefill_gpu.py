"""Prefill gather attention (tcgen05 kernel) against the oracle and the
reference goldens: contiguous (HF layout), multi index head, packing, paged
(serving layout), and BASELINE config 2 at full size on sampled rows."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from ananta_ocr_b200 import ops
from ananta_ocr_b200 import modeling_deepseekv2 as MD
from ananta_ocr_b200.sparse_gather_e2e_triton import triton_gather_attention_e2e
from ananta_ocr_b200.sparse_gather_triton import triton_gather_attention
from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn
from dash_testutil import assert_close_bf16, bf16_round, random_routes, sample_rows

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_c1_golden_e2e():
    """BASELINE config 1 with the reference's own routes: bf16 kernel vs the
    reference fp32 output."""
    g = np.load(os.path.join(GOLD, "c1_headcls.npz"))
    q, k, v, iq, ik = O.make_prefill_inputs(0, 1, 10, 1348, 128, 0, 273, 0.0)
    topi, valid = g["topi"], g["valid"]
    bi = np.where(valid, topi, -1).astype(np.int32)[:, None]
    bias = np.where(valid, g["bias"], 0).astype(np.float32)
    out = triton_gather_attention_e2e(
        torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(k).cuda().bfloat16(),
        torch.from_numpy(v).cuda().bfloat16(), torch.from_numpy(bi).cuda(),
        torch.from_numpy(bias).cuda(), torch.arange(1348, device="cuda")[None], None, 64,
        1.0 / math.sqrt(128), 256)
    rows = g["rows"]
    assert_close_bf16(out.float().cpu().numpy()[:, :, rows], g["out_rows"])


def test_checkpoint_block_size_golden():
    """The checkpoint's DASH settings (block 32, window 4 blocks, K=12) on the
    config-1 shape with page offsets: router + attention on the GPU against the
    reference's own _infer_route_select routes and _forward_dense output."""
    g = np.load(os.path.join(GOLD, "c1_bs32.npz"))
    B, H, S, bs, lb, K = (int(g[x]) for x in ("B", "H", "S", "bs", "lb", "K"))
    q, k, v, iq, ik = O.make_prefill_inputs(int(g["seed"]), B, H, S, 128, int(g["n_pages"]),
                                            int(g["page_tokens"]), float(g["off_std"]))
    out, idx, bias = MD.dash_prefill_forward(
        torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(k).cuda().bfloat16(),
        torch.from_numpy(v).cuda().bfloat16(), torch.from_numpy(iq).cuda(),
        torch.from_numpy(ik).cuda(), block_size=bs, local_blocks=lb, K=K,
        idx_scale=float(g["idx_scale"]), prior_floor=float(g["floor"]), sigma=float(g["sigma"]),
        return_routes=True)
    topi, valid = g["topi"], g["valid"]
    ri = np.sort(np.where(valid, topi, np.iinfo(np.int32).max), -1)
    ri = np.where(ri == np.iinfo(np.int32).max, -1, ri).astype(np.int32)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    rows = g["rows"]
    assert_close_bf16(out.float().cpu().numpy()[:, :, rows], g["out_rows"])


@pytest.mark.parametrize("name", ["triton_interp", "triton_interp_bs32"])
def test_reference_triton_golden(name):
    """The reference's Triton kernels (interpreted on the CPU, fp32) against the
    B200 kernels on the same inputs: e2e contiguous, paged prefill, decode.
    The 16-token-block golden exercises decode only (the tensor-core prefill
    takes blocks of 32 tokens or multiples of 64; it refuses 16)."""
    g = np.load(os.path.join(GOLD, name + ".npz"))
    q, k, v, idx, bias = g["q"], g["k"], g["v"], g["idx"], g["bias"]
    bs, lb = int(g["bs"]), int(g["lb"])
    B, H, T, D = q.shape
    prefill = bs == 32 or bs % 64 == 0
    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda().bfloat16()   # noqa: E731
    if prefill:
        out = triton_gather_attention_e2e(bf(q), bf(k), bf(v),
                                          torch.from_numpy(idx).cuda()[:, None],
                                          torch.from_numpy(bias).cuda(),
                                          torch.arange(T, device="cuda")[None], None, bs,
                                          1.0 / math.sqrt(D), lb * bs)
        assert_close_bf16(out.float().cpu().numpy(), g["out_e2e"])
    bt = g["block_table"]
    P = int(bt.max()) + 1
    kc = np.zeros((P, bs, H, D), np.float32)
    vc = np.zeros_like(kc)
    for b, pg in enumerate(bt[0]):
        kc[pg] = k[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
        vc[pg] = v[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
    qp = q[0].transpose(1, 0, 2)
    ti = torch.from_numpy(idx[0]).cuda()[None].expand(H, -1, -1)
    tb = torch.from_numpy(bias[0]).cuda()[None].expand(H, -1, -1)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device="cuda")        # noqa: E731
    if prefill:
        outp = torch.zeros(T, H, D, dtype=torch.bfloat16, device="cuda")
        dash_sparse_attn(bf(qp), bf(kc), bf(vc), ti, tb, torch.from_numpy(bt).cuda(),
                         i32([0, T]), i32([T]), i32([0]), T, H, 1.0 / math.sqrt(D), outp,
                         local_blocks=lb, sparse_block_size=bs)
        assert_close_bf16(outp.float().cpu().numpy(), g["out_paged"])
    from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn_decode
    outd = torch.zeros(1, H, D, dtype=torch.bfloat16, device="cuda")
    dash_sparse_attn_decode(bf(qp[-1:]), bf(kc), bf(vc), ti[:, -1:], tb[:, -1:],
                            torch.from_numpy(bt).cuda(), i32([T]), H, 1.0 / math.sqrt(D), outd, 1,
                            local_blocks=lb, sparse_block_size=bs)
    assert_close_bf16(outd.float().cpu().numpy(), g["out_decode"])


def test_e2e_declines_like_reference():
    x = torch.zeros(1, 2, 64, 128, device="cuda", dtype=torch.bfloat16)
    bi = torch.zeros(1, 1, 64, 2, dtype=torch.int32, device="cuda")
    b = torch.zeros(1, 64, 2, device="cuda")
    pos = torch.arange(64, device="cuda")[None]
    assert triton_gather_attention_e2e(x, x, x, bi, b, pos, torch.zeros(1), 64, 0.1, 64) is None
    assert triton_gather_attention_e2e(x, x, x, bi.expand(1, 2, 64, 2), b, pos, None, 64, 0.1) is None
    assert triton_gather_attention_e2e(x, x, x, bi, b, pos + 1, None, 64, 0.1, 64) is None


CASES = [
    # B, H, Hkv, T, bs, LW, K
    (2, 2, 2, 700, 64, 256, 4),
    (1, 4, 2, 1000, 128, 256, 3),     # GQA G=2, block 128
    (1, 1, 1, 129, 64, 64, 2),        # tiny, ragged tail
    (1, 2, 2, 100, 64, 256, 4),       # window longer than the sequence
    (1, 8, 1, 600, 64, 128, 5),       # G=8
    (2, 3, 3, 777, 64, 192, 6),       # window not a multiple of ... 64-aligned but 3 blocks
    # 32-token blocks (the checkpoint's sparse_block_size): two blocks per key tile
    (2, 2, 2, 700, 32, 128, 12),
    (1, 4, 2, 1000, 32, 128, 16),     # GQA G=2
    (1, 1, 1, 129, 32, 128, 3),       # tiny, ragged tail
    (1, 8, 1, 600, 32, 96, 5),        # G=8, window of 3 blocks
    (2, 3, 3, 777, 32, 100, 12),      # window ends inside a block
]


@pytest.mark.parametrize("B,H,Hkv,T,bs,LW,K", CASES)
def test_prefill_random_vs_oracle(B, H, Hkv, T, bs, LW, K):
    rng = np.random.default_rng(B * 1000 + T)
    D = 128
    q = bf16_round((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32))
    k = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    v = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    idx, bias = random_routes(rng, B, T, K, bs, LW)
    out = ops.gather_attention(torch.from_numpy(q).cuda().bfloat16(),
                               torch.from_numpy(k).cuda().bfloat16(),
                               torch.from_numpy(v).cuda().bfloat16(),
                               torch.from_numpy(idx).cuda(), torch.from_numpy(bias).cuda(),
                               block_size=bs, local_window=LW, scale=1.0 / math.sqrt(D))
    ref = O.attend_contig(q, k, v, idx[:, 0], bias[:, 0], bs, LW, 1.0 / math.sqrt(D))
    assert_close_bf16(out.float().cpu().numpy(), ref)


def test_prefill_strided_layout_and_lse():
    """[B,T,H,D] storage viewed as [B,H,T,D] (the reference kernel layout)."""
    rng = np.random.default_rng(3)
    B, H, T, D, bs, LW, K = 2, 4, 513, 128, 64, 256, 4
    base = lambda: bf16_round((rng.standard_normal((B, T, H, D)) * 0.5).astype(np.float32))
    q, k, v = base(), base(), base()
    idx, bias = random_routes(rng, B, T, K, bs, LW, messy=False)
    tq = torch.from_numpy(q).cuda().bfloat16().transpose(1, 2)
    tk = torch.from_numpy(k).cuda().bfloat16().transpose(1, 2)
    tv = torch.from_numpy(v).cuda().bfloat16().transpose(1, 2)
    lse = torch.empty(B, H, T, device="cuda")
    out = ops.gather_attention(tq, tk, tv, torch.from_numpy(idx).cuda(),
                               torch.from_numpy(bias).cuda(), block_size=bs, local_window=LW,
                               scale=1.0 / math.sqrt(D), lse=lse)
    qq = q.transpose(0, 2, 1, 3)
    ref, ref_lse = O.attend_contig(qq, k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3),
                                   idx[:, 0], bias[:, 0], bs, LW, 1.0 / math.sqrt(D),
                                   return_lse=True)
    assert_close_bf16(out.float().cpu().numpy(), ref)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=2e-3)


def test_multi_index_head_and_packing():
    """triton_gather_attention: HI=2 index heads, two packed segments per row."""
    rng = np.random.default_rng(4)
    B, H, Hkv, T, D, bs, LW, K = 1, 4, 2, 640, 128, 64, 128, 3
    q = bf16_round((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32))
    k = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    v = bf16_round((rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32))
    idx, _ = random_routes(rng, B, T, K, bs, LW, n_index_heads=2)
    split = 300
    pos = np.concatenate([np.arange(split), np.arange(T - split)])[None]
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


@pytest.mark.parametrize("bs,lb", [(64, 4), (128, 2), (32, 4), (32, 1)])
def test_paged_prefill_with_prefix(bs, lb):
    rng = np.random.default_rng(bs)
    D, H, Hkv, K = 128, 4, 2, 4
    seq_lens = np.array([700, 300, 1500])
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
            idx[i, :len(c)] = np.sort(c)
    out = torch.zeros(total_q, H, D, dtype=torch.bfloat16, device="cuda")
    ti = torch.from_numpy(idx).cuda()[None].expand(Hkv, -1, -1)
    tb = torch.from_numpy(bias).cuda()[None].expand(Hkv, -1, -1)
    dash_sparse_attn(torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(kc).cuda().bfloat16(),
                     torch.from_numpy(vc).cuda().bfloat16(), ti, tb, torch.from_numpy(bt).cuda(),
                     torch.from_numpy(cu).cuda(), torch.from_numpy(seq_lens.astype(np.int32)).cuda(),
                     torch.from_numpy(ctx.astype(np.int32)).cuda(), int(q_lens.max()), Hkv,
                     1.0 / math.sqrt(D), out, local_blocks=lb, sparse_block_size=bs)
    ref = O.attend_paged(q, kc, vc, idx, bias, bt, row_req, row_pos, bs, lb * bs, 1.0 / math.sqrt(D))
    assert_close_bf16(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("H,S", [(16, 32768), (4, 131072)])
def test_prefill_config4_geometry_sampled_rows(H, S):
    """BASELINE config 4 geometry (block 128, window 8 blocks = 1024 tokens,
    k=64) on one sequence of 32,768 tokens (16 heads) and of the full 131,072
    tokens (4 heads, 1,024 blocks): router + attention on the GPU, routes
    bit-exact, output vs the oracle on sampled rows."""
    B, D, bs, lb, K = 1, 128, 128, 8, 64
    q, k, v, iq, ik = O.make_prefill_inputs(8, B, H, S, D, S // 273, 273, 0.2)
    out, idx, bias = MD.dash_prefill_forward(
        torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(k).cuda().bfloat16(),
        torch.from_numpy(v).cuda().bfloat16(), torch.from_numpy(iq).cuda(),
        torch.from_numpy(ik).cuda(), block_size=bs, local_blocks=lb, K=K,
        idx_scale=128.0 / math.sqrt(128), prior_floor=1e-4, sigma=1.0, return_routes=True)
    rows = sample_rows(np.random.default_rng(2), S, 40)
    gi = idx.cpu().numpy()
    kb = O.kbar_contig(ik, np.zeros(128, np.float32), bs)
    nblk = kb.shape[1]
    osc = O.scores_paged(iq[0, rows], rows, np.zeros(len(rows), np.int64), np.array([S]), kb[0],
                         np.arange(nblk, dtype=np.int32)[None], bs, lb, nblk)
    oi, _, _ = O.route_select(osc, None, 128.0 / math.sqrt(128), K, K, 1e-4, 1.0)
    np.testing.assert_array_equal(gi[0, rows], oi)
    ref = O.attend_contig(bf16_round(q), bf16_round(k), bf16_round(v), gi, bias.cpu().numpy(), bs,
                          lb * bs, 1.0 / math.sqrt(D), rows=rows)
    assert_close_bf16(out.float().cpu().numpy()[:, :, rows], ref)


def test_prefill_config2_full_size_sampled_rows():
    """BASELINE config 2 (B=4, H=10, S=9248, bs=64, window 4, K=16, page
    offsets): router + attention on the GPU; routes checked bit-exact and the
    output checked against the oracle on sampled rows of every sequence/head."""
    B, H, S, D, bs, lb, K = 4, 10, 9248, 128, 64, 4, 16
    q, k, v, iq, ik = O.make_prefill_inputs(0, B, H, S, D, 32, 273, 0.2)
    tq = torch.from_numpy(q).cuda().bfloat16()
    tk = torch.from_numpy(k).cuda().bfloat16()
    tv = torch.from_numpy(v).cuda().bfloat16()
    out, idx, bias = MD.dash_prefill_forward(
        tq, tk, tv, torch.from_numpy(iq).cuda(), torch.from_numpy(ik).cuda(), block_size=bs,
        local_blocks=lb, K=K, idx_scale=128.0 / math.sqrt(128), prior_floor=1e-4, sigma=1.0,
        return_routes=True)
    gi = idx.cpu().numpy()
    osc = O.block_scores_headcls(iq, ik, np.arange(S)[None], bs, lb, np.zeros(128, np.float32))
    oi, ob, _ = O.route_select(osc, None, 128.0 / math.sqrt(128), K, K, 1e-4, 1.0)
    np.testing.assert_array_equal(gi, oi)
    rows = sample_rows(np.random.default_rng(0), S, 120)
    ref = O.attend_contig(bf16_round(q), bf16_round(k), bf16_round(v), gi, bias.cpu().numpy(),
                          bs, lb * bs, 1.0 / math.sqrt(D), rows=rows)
    assert_close_bf16(out.float().cpu().numpy()[:, :, rows], ref)


def test_two_streams_share_no_scratch():
    """Two prefills issued on two streams at once (each library call takes
    its cached scratch from its own stream) give exactly the single-stream
    outputs."""
    torch.manual_seed(5)
    B, H, T, D, bs = 2, 2, 1500, 128, 64
    ins = []
    for _ in range(2):
        q = (torch.randn(B, H, T, D, device="cuda") * 0.5).bfloat16()
        k = (torch.randn(B, H, T, D, device="cuda") * 0.5).bfloat16()
        v = (torch.randn(B, H, T, D, device="cuda") * 0.5).bfloat16()
        iq = torch.randn(B, T, 128, device="cuda") * 0.5
        ik = torch.randn(B, T, 128, device="cuda") * 0.5
        ins.append((q, k, v, iq, ik))

    def run(x):
        return MD.dash_prefill_forward(*x, block_size=bs, local_blocks=4, K=4,
                                       idx_scale=128.0 / math.sqrt(128), prior_floor=1e-4, sigma=1.0)

    ref = [run(x) for x in ins]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream() for _ in range(2)]
    outs = [None, None]
    for _ in range(3):
        for s in streams:
            s.wait_stream(torch.cuda.current_stream())
        for j in range(2):
            with torch.cuda.stream(streams[j]):
                outs[j] = run(ins[j])
        for s in streams:
            torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        for j in range(2):
            assert torch.equal(outs[j], ref[j])


# ---------------------------------------------------------------------------
# fp32 inputs: the fp32 CUDA-core kernel (every product and sum in fp32)
# ---------------------------------------------------------------------------
F32_ATOL = 2e-5      # fp32 kernel vs fp32/fp64 references


def test_c1_golden_fp32():
    """BASELINE config 1 is fp32: with the reference's own routes the output
    matches the reference's fp32 _forward_dense to fp32 rounding."""
    g = np.load(os.path.join(GOLD, "c1_headcls.npz"))
    q, k, v, iq, ik = O.make_prefill_inputs(0, 1, 10, 1348, 128, 0, 273, 0.0)
    bi = np.where(g["valid"], g["topi"], -1).astype(np.int32)[:, None]
    bias = np.where(g["valid"], g["bias"], 0).astype(np.float32)
    out = triton_gather_attention_e2e(
        torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
        torch.from_numpy(bi).cuda(), torch.from_numpy(bias).cuda(),
        torch.arange(1348, device="cuda")[None], None, 64, 1.0 / math.sqrt(128), 256)
    assert out.dtype == torch.float32
    np.testing.assert_allclose(out.cpu().numpy()[:, :, g["rows"]], g["out_rows"], atol=F32_ATOL, rtol=0)


F32_CASES = [
    # B, H, Hkv, T, bs, LW, K
    (2, 2, 2, 700, 64, 256, 4),
    (1, 6, 2, 900, 32, 128, 12),      # G=3, 32-token blocks
    (1, 2, 2, 333, 16, 48, 5),        # 16-token blocks, window of 3 blocks
    (2, 4, 4, 500, 100, 200, 3),      # a block size no tile shape divides
    (1, 1, 1, 40, 64, 256, 2),        # shorter than a block and the window
]


@pytest.mark.parametrize("B,H,Hkv,T,bs,LW,K", F32_CASES)
def test_prefill_fp32_vs_oracle(B, H, Hkv, T, bs, LW, K):
    rng = np.random.default_rng(B * 7 + T)
    D = 128
    q = (rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32)
    idx, bias = random_routes(rng, B, T, K, bs, LW)
    lse = torch.empty(B, H, T, device="cuda")
    out = ops.gather_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                               torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda(),
                               torch.from_numpy(bias).cuda(), block_size=bs, local_window=LW,
                               scale=1.0 / math.sqrt(D), lse=lse)
    ref, ref_lse = O.attend_contig(q, k, v, idx[:, 0], bias[:, 0], bs, LW, 1.0 / math.sqrt(D),
                                   return_lse=True)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=F32_ATOL, rtol=0)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=1e-4, rtol=0)


def test_prefill_fp32_index_heads_and_packing():
    """fp32 through triton_gather_attention (no grad): two index heads, two
    packed segments per row."""
    rng = np.random.default_rng(41)
    B, H, Hkv, T, D, bs, LW, K = 1, 4, 2, 640, 128, 64, 128, 3
    q = (rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, Hkv, T, D)) * 0.5).astype(np.float32)
    idx, _ = random_routes(rng, B, T, K, bs, LW, n_index_heads=2)
    split = 300
    pos = np.concatenate([np.arange(split), np.arange(T - split)])[None]
    with torch.no_grad():
        out = triton_gather_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                      torch.from_numpy(v).cuda(), torch.from_numpy(idx).cuda(),
                                      torch.from_numpy(pos).cuda(), None, bs, 1.0 / math.sqrt(D), LW)
    assert out.dtype == torch.float32
    seg = (np.arange(T)[None] - pos)
    got = out.cpu().numpy()
    for ih in range(2):
        hs = slice(ih * 2, ih * 2 + 2)
        ref = O.attend_contig(q[:, hs], k[:, ih:ih + 1], v[:, ih:ih + 1], idx[:, ih], None, bs,
                              LW, 1.0 / math.sqrt(D), seg=seg)
        np.testing.assert_allclose(got[:, hs], ref, atol=F32_ATOL, rtol=0)
