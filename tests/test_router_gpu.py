"""Router parity on the GPU (k-bar pooling, block scores, selection + bias)
against the CPU oracle (bit-exact scores and indices) and the reference goldens."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from ananta_ocr_b200 import ops
from ananta_ocr_b200 import modeling_deepseekv2 as MD
from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
from ananta_ocr_b200.unlimited_dash_ops.dash_router import DashRouterMath

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
IDX_SCALE = 128.0 / math.sqrt(128)


def canon(topi, bias, valid):
    big = 1 << 30
    ti = np.where(valid, topi, big)
    o = np.argsort(ti, -1, kind="stable")
    ii = np.take_along_axis(ti, o, -1)
    bb = np.take_along_axis(np.where(valid, bias, 0.0), o, -1)
    return np.where(ii == big, -1, ii).astype(np.int32), bb.astype(np.float32)


@pytest.mark.parametrize("hc_std", [0.0, 1.0])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("S,bs", [(300, 16), (1348, 64), (1000, 128)])
def test_kbar_bitwise(hc_std, dtype, S, bs):
    rng = np.random.default_rng(7)
    ik = (rng.standard_normal((2, S, 128)) * 0.5).astype(np.float32)
    ik = torch.from_numpy(ik).to(dtype).float().numpy()
    hc = (rng.standard_normal(128) * hc_std).astype(np.float32)
    got = ops.kbar_pool_contig(torch.from_numpy(ik).to(dtype).cuda(), torch.from_numpy(hc).cuda(), bs)
    ref = O.kbar_contig(ik, hc, bs)
    assert np.array_equal(got.cpu().numpy(), ref)


def _route_case(iq, ik, hc, bs, lb, K, topm):
    B, S, d = iq.shape
    nblk = (S + bs - 1) // bs
    kbar = ops.kbar_pool_contig(torch.from_numpy(ik).cuda(), torch.from_numpy(hc).cuda(), bs)
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    scores = torch.empty(B * S, nblk, dtype=torch.float32, device="cuda")
    idx, bias = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                          prior_floor=1e-4, sigma=1.0, topm=topm, K=K,
                          idx_q=torch.from_numpy(iq).cuda().view(B * S, d), kbar=kbar,
                          scores_out=scores)
    osc = O.block_scores_headcls(iq, ik, np.arange(S)[None], bs, lb, hc).reshape(B * S, nblk)
    oi, ob, _ = O.route_select(osc, None, IDX_SCALE, topm, K, 1e-4, 1.0)
    return scores.cpu().numpy(), idx.cpu().numpy(), bias.cpu().numpy(), osc, oi, ob


@pytest.mark.parametrize("B,S,bs,lb,K,topm,hc_std,off", [
    (1, 1348, 64, 4, 8, 8, 0.0, 0.0),        # BASELINE config 1 shapes
    (2, 700, 16, 2, 4, 6, 1.0, 0.3),
    (2, 2000, 64, 4, 16, 16, 0.0, 0.2),
    (1, 5000, 128, 8, 32, 40, 0.5, 0.2),
])
def test_route_bitwise_vs_oracle(B, S, bs, lb, K, topm, hc_std, off):
    iq, ik = O.make_router_inputs(11, B, S, max(1, S // 273), 273, off)
    hc = (np.random.default_rng(3).standard_normal(128) * hc_std).astype(np.float32)
    gs, gi, gb, osc, oi, ob = _route_case(iq, ik, hc, bs, lb, K, topm)
    assert np.array_equal(gs, osc), "block scores differ from the oracle"
    np.testing.assert_array_equal(gi, oi)
    np.testing.assert_allclose(gb, ob, atol=1e-4, rtol=0)


@pytest.mark.parametrize("name", ["c1_headcls", "small_headcls", "small_indexer"])
def test_select_on_reference_scores(name):
    g = np.load(os.path.join(GOLD, name + ".npz"))
    p = dict(idx_scale=float(g["idx_scale"]), floor=float(g["floor"]), sigma=float(g["sigma"]),
             K=int(g["K"]), topm=int(g["topm"]))
    topi, bias, valid = MD._infer_route_select(torch.from_numpy(g["scores"]).cuda(), None, p)
    gi = np.where(valid.cpu().numpy(), topi.cpu().numpy(), -1)
    ri, rb = canon(g["topi"], g["bias"], g["valid"])
    np.testing.assert_array_equal(gi, ri)
    np.testing.assert_allclose(bias.cpu().numpy(), rb, atol=1e-4)


def test_block_max_indexer_vs_oracle():
    rng = np.random.default_rng(5)
    B, C, Sk, bs, lw = 2, 300, 300, 32, 64
    q = (rng.standard_normal((B, C, 128)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, Sk, 128)) * 0.5).astype(np.float32)
    pos = np.broadcast_to(np.arange(C), (B, C)).copy()
    seg = np.zeros((B, C), np.int64)
    seg[1, 150:] = 150
    nblk = (Sk + bs - 1) // bs
    from ananta_ocr_b200.sparse_gather_triton import triton_block_max_score
    got = triton_block_max_score(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                 torch.from_numpy(pos).cuda(), torch.from_numpy(seg).cuda(), bs,
                                 nblk, lw).cpu().numpy()
    ref = O.block_scores_indexer(q, k, pos, bs, lw, nblk, q_seg=seg, clamp=False, empty=-np.inf)
    assert np.array_equal(got, ref)
    # HF indexer branch (clamped, SCORE_NEG sentinel) on the golden
    g = np.load(os.path.join(GOLD, "small_indexer.npz"))
    iq, ik = O.make_router_inputs(0, 1, 4, 1, 4, 0.0)  # placeholder shapes, replaced below
    qq, kk, vv, iq, ik = O.make_prefill_inputs(int(g["seed"]), int(g["B"]), int(g["H"]), int(g["S"]),
                                               128, int(g["n_pages"]), int(g["page_tokens"]),
                                               float(g["off_std"]))
    router = type("R", (), dict(stage0="indexer", block_size=int(g["bs"]), local_blocks=int(g["lb"]),
                                local_window=int(g["lb"]) * int(g["bs"]), head_cls=None))
    S = int(g["S"])
    sc = MD._block_scores_infer(router, torch.from_numpy(iq).cuda(), torch.from_numpy(ik).cuda(),
                                torch.arange(S, device="cuda")[None], (S + int(g["bs"]) - 1) // int(g["bs"]))
    osc = O.block_scores_indexer(iq, ik, np.arange(S)[None], int(g["bs"]), int(g["lb"]) * int(g["bs"]))
    assert np.array_equal(sc.cpu().numpy(), osc)


def test_paged_router_golden():
    g = np.load(os.path.join(GOLD, "paged_router.npz"))
    d, bs, lb = int(g["d"]), int(g["bs"]), int(g["lb"])
    seq_lens, ctx, cu, bt = g["seq_lens"], g["ctx_lens"], g["cu"], g["block_table"]
    R, W = bt.shape
    P = g["cache"].shape[0]
    dev = "cuda"
    cache = torch.from_numpy(g["cache"]).to(dev)
    kbar = torch.zeros(P, d, dtype=torch.float32, device=dev)
    btd = torch.from_numpy(bt).to(dev)
    sl = torch.from_numpy(seq_lens).to(dev)
    plan = RT.kbar_all_plan(block_table=btd, seq_lens=sl, context_lens=torch.zeros_like(sl),
                            block_size=bs, max_block=W, max_query_len=int(seq_lens.max()), device=dev)
    RT.kbar_refresh_tail_triton(kv_cache=cache, k_bar=kbar, block_table=btd, seq_lens=sl,
                                head_cls=torch.from_numpy(g["head_cls"]).to(dev), block_size=bs,
                                plan=plan)
    kb = kbar.cpu().numpy()
    ref_kbar = np.zeros_like(g["kbar"])
    pages, ntok = [], []
    for r in range(R):
        nb = -(-int(seq_lens[r]) // bs)
        for b in range(nb):
            pages.append(bt[r, b])
            ntok.append(min(bs, int(seq_lens[r]) - b * bs))
    O.kbar_paged(g["cache"], np.array(pages), np.array(ntok), g["head_cls"], ref_kbar)
    used = np.array(pages)
    assert np.array_equal(kb[used], ref_kbar[used])
    slots, budget, topm = int(g["out_slots"]), int(g["budget"]), int(g["topm"])
    total_q = int(cu[-1])
    out_idx = torch.empty(total_q, slots, dtype=torch.int32, device=dev)
    out_bias = torch.empty(total_q, slots, dtype=torch.float32, device=dev)
    RT.route_prefill_triton(idx_q=torch.from_numpy(g["idx_q"]).to(dev), k_bar=kbar, block_table=btd,
                            seq_lens=sl, cu_seqlens_q=torch.from_numpy(cu).to(dev),
                            context_lens=torch.from_numpy(ctx).to(dev), row2req=None,
                            image_allow=None, out_idx=out_idx, out_bias=out_bias, max_block=W,
                            block_size=bs, local_blocks=lb, idx_scale=float(g["idx_scale"]),
                            prior_floor=1e-4, sigma=1.0, topm=topm, budget=budget,
                            out_slots=slots)
    ref_i = g["idx_prefill"][:, :slots]
    ri, rb = canon(ref_i, g["bias_prefill"][:, :slots], ref_i >= 0)
    np.testing.assert_array_equal(out_idx.cpu().numpy(), ri)
    np.testing.assert_allclose(out_bias.cpu().numpy(), rb, atol=1e-4)
    # decode
    oi = torch.empty(R, slots, dtype=torch.int32, device=dev)
    ob = torch.empty(R, slots, dtype=torch.float32, device=dev)
    RT.route_decode_triton(idx_q=torch.from_numpy(g["iq_dec"]).to(dev), k_bar=kbar, block_table=btd,
                           seq_lens=sl, image_allow=None, out_idx=oi, out_bias=ob, max_block=W,
                           block_size=bs, local_blocks=lb, decode_query_len=1,
                           idx_scale=float(g["idx_scale"]), prior_floor=1e-4, sigma=1.0, topm=topm,
                           budget=budget, out_slots=slots)
    ref_i = g["idx_decode"][:, :slots]
    ri, rb = canon(ref_i, g["bias_decode"][:, :slots], ref_i >= 0)
    np.testing.assert_array_equal(oi.cpu().numpy(), ri)
    np.testing.assert_allclose(ob.cpu().numpy(), rb, atol=1e-4)
    # DashRouterMath on the reference scores
    router = DashRouterMath(index_dim=d, block_size=bs, local_blocks=lb, topk_blocks=8,
                            scaling_factor=128.0, sigma=1.0, prior_floor=1e-4, budget_remote=budget,
                            topm=topm)
    ti, tb = router.route_and_select(torch.from_numpy(g["scores_decode"]).to(dev), W)
    ref_i = g["idx_decode"]
    ri, rb = canon(ref_i, g["bias_decode"], ref_i >= 0)
    np.testing.assert_array_equal(ti.cpu().numpy(), ri)
    np.testing.assert_allclose(tb.cpu().numpy(), rb, atol=1e-4)


def test_candidate_mask_and_fallback():
    rng = np.random.default_rng(9)
    rows, W = 64, 40
    sc = (rng.standard_normal((rows, W))).astype(np.float32)
    sc[:, 30:] = -1e9                                    # not remote
    cand = rng.random((rows, W)) < 0.3
    cand[:8] = False                                     # empty mask -> fallback to remote
    p = dict(idx_scale=IDX_SCALE, floor=1e-4, sigma=1.0, K=6, topm=10)
    topi, bias, valid = MD._infer_route_select(torch.from_numpy(sc).cuda()[None],
                                               torch.from_numpy(cand).cuda()[None], p)
    gi = np.where(valid.cpu().numpy(), topi.cpu().numpy(), -1)[0]
    oi, ob, _ = O.route_select(sc, cand, IDX_SCALE, 10, 6, 1e-4, 1.0)
    np.testing.assert_array_equal(gi, oi)
    np.testing.assert_allclose(bias.cpu().numpy()[0], ob, atol=1e-4)


def test_router_full_size_config2():
    """BASELINE config 2 router (B=4, S=9248, bs=64, window 4, K=16): every row."""
    B, S, bs, lb, K = 4, 9248, 64, 4, 16
    iq, ik = O.make_router_inputs(0, B, S, 32, 273, 0.2)
    hc = np.zeros(128, np.float32)
    gs, gi, gb, osc, oi, ob = _route_case(iq, ik, hc, bs, lb, K, K)
    assert np.array_equal(gs, osc)
    np.testing.assert_array_equal(gi, oi)
    np.testing.assert_allclose(gb, ob, atol=1e-4)


def test_router_config4_sampled_rows():
    """BASELINE config 4 router (S=131072, bs=128, nblk=1024, K=64) on 2 of the 8
    sequences; oracle checks sampled rows (scores bitwise, indices exact)."""
    B, S, bs, lb, K = 2, 131072, 128, 8, 64
    iq, ik = O.make_router_inputs(4, B, S, 480, 273, 0.2)
    hc = np.zeros(128, np.float32)
    nblk = S // bs
    kbar = ops.kbar_pool_contig(torch.from_numpy(ik).cuda(), None, bs)
    ref_kbar = O.kbar_contig(ik, hc, bs)
    assert np.array_equal(kbar.cpu().numpy(), ref_kbar)
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    idx, bias = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                          prior_floor=1e-4, sigma=1.0, topm=K, K=K,
                          idx_q=torch.from_numpy(iq).cuda().view(B * S, 128), kbar=kbar)
    rng = np.random.default_rng(1)
    rows = np.concatenate([rng.integers(0, S, 96), [S - 1, 1024, 1025, 2047]])
    for b in range(B):
        row_req = np.full(len(rows), b)
        bt = np.broadcast_to(np.arange(nblk, dtype=np.int32) + b * nblk, (B, nblk)).copy()
        osc = O.scores_paged(iq[b, rows], rows, row_req, np.full(B, S), ref_kbar.reshape(-1, 128),
                             bt, bs, lb, nblk)
        oi, ob, _ = O.route_select(osc, None, IDX_SCALE, K, K, 1e-4, 1.0)
        np.testing.assert_array_equal(idx.cpu().numpy()[b * S + rows], oi)
        np.testing.assert_allclose(bias.cpu().numpy()[b * S + rows], ob, atol=1e-4)
