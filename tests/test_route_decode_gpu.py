"""Decode routing (the cluster kernel: slices scored across 8 CTAs, CTA-wide
selection) against the CPU oracle, bitwise: scores, indices, and the k-bar
rows of the tail refresh folded into the same launch."""
import math

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from ananta_ocr_b200 import _lib, ops
from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT

pytestmark = pytest.mark.gpu
IDX_SCALE = 128.0 / math.sqrt(128)


def _decode_inputs(seed, R, W, bs, lb, ties):
    rng = np.random.default_rng(seed)
    P = R * W + 8
    kbar = rng.standard_normal((P, 128)).astype(np.float32) * 0.5
    iq = rng.standard_normal((R, 128)).astype(np.float32) * 0.5
    if ties:
        # coarse values: many equal dot products, so the tie rule decides
        kbar = np.round(kbar * 2) / 2
        iq = np.sign(np.round(iq * 2)).astype(np.float32)
    bt = rng.permutation(P)[:R * W].astype(np.int32).reshape(R, W)
    lo = bs * (lb + 1)
    seq_lens = rng.integers(lo, W * bs + 1, R).astype(np.int32)
    seq_lens[0] = W * bs                       # one row with every block remote-able
    seq_lens[1] = lo                           # one with a single remote block
    return kbar, iq, bt, seq_lens


def _route(kbar, iq, bt, seq_lens, bs, lb, K, topm, cand=None):
    R, W = bt.shape
    dev = "cuda"
    seqs = ops.Seqs(n_seq=R, q_len=1, kv_len=0, kv_len_t=torch.from_numpy(seq_lens).to(dev),
                    max_q_len=1)
    scores = torch.empty(R, W, dtype=torch.float32, device=dev)
    idx, bias = ops.route(seqs, width=W, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                          prior_floor=1e-4, sigma=1.0, topm=topm, K=K,
                          idx_q=torch.from_numpy(iq).to(dev), kbar=torch.from_numpy(kbar).to(dev),
                          block_table=torch.from_numpy(bt).to(dev),
                          cand=None if cand is None else torch.from_numpy(cand).to(dev),
                          scores_out=scores)
    return scores.cpu().numpy(), idx.cpu().numpy(), bias.cpu().numpy()


@pytest.mark.parametrize("W,K,topm,ties", [
    (37, 8, 8, False),          # 1 block per selecting thread
    (200, 16, 24, False),       # 2
    (431, 32, 32, False),       # 4: BASELINE config 3 (27,556 tokens, block 64)
    (431, 32, 32, True),        # ties at the threshold
    (1000, 64, 64, False),      # 8
    (1000, 16, 16, True),
    (100, 16, 0, False),        # topm 0: the entmax window is every block
    (1500, 32, 32, False),      # wider than the CTA-wide form: one-warp selection
])
def test_decode_route_vs_oracle(W, K, topm, ties):
    bs, lb, R = 64, 4, 24
    kbar, iq, bt, seq_lens = _decode_inputs(W + K, R, W, bs, lb, ties)
    gs, gi, gb = _route(kbar, iq, bt, seq_lens, bs, lb, K, topm)
    osc = O.scores_paged(iq, seq_lens.astype(np.int64) - 1, np.arange(R), seq_lens, kbar, bt, bs, lb, W)
    assert np.array_equal(gs, osc), "block scores differ from the oracle"
    oi, ob, _ = O.route_select(osc, None, IDX_SCALE, topm, K, 1e-4, 1.0)
    np.testing.assert_array_equal(gi[:, :K], oi)
    np.testing.assert_allclose(gb[:, :K], ob, atol=1e-4, rtol=0)


@pytest.mark.parametrize("W", [60, 431])
def test_decode_route_candidates_and_fallback(W):
    bs, lb, R, K = 64, 4, 24, 12
    kbar, iq, bt, seq_lens = _decode_inputs(5, R, W, bs, lb, False)
    cand = np.random.default_rng(6).random((R, W)) < 0.2
    cand[:4] = False                           # no candidate: every remote block
    gs, gi, gb = _route(kbar, iq, bt, seq_lens, bs, lb, K, K, cand)
    oi, ob, _ = O.route_select(gs, cand, IDX_SCALE, K, K, 1e-4, 1.0)
    np.testing.assert_array_equal(gi, oi)
    np.testing.assert_allclose(gb, ob, atol=1e-4, rtol=0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hc_std", [0.0, 1.0])
def test_decode_route_with_folded_refresh(dtype, hc_std):
    """route_decode_triton(refresh=...) equals kbar_refresh_tail_triton followed
    by route_decode_triton (same k-bar bits, same routes) in one launch."""
    bs, lb, R, W, K = 64, 4, 16, 300, 16
    dev = "cuda"
    rng = np.random.default_rng(21)
    _, iq, bt, seq_lens = _decode_inputs(8, R, W, bs, lb, False)
    P = int(bt.max()) + 1
    cache = torch.from_numpy(rng.standard_normal((P, bs, 128)).astype(np.float32) * 0.5).to(dtype).to(dev)
    hc = torch.from_numpy((rng.standard_normal(128) * hc_std).astype(np.float32)).to(dev)
    btd, sl = torch.from_numpy(bt).to(dev), torch.from_numpy(seq_lens).to(dev)
    kbar0 = torch.zeros(P, 128, device=dev)
    plan = RT.kbar_all_plan(block_table=btd, seq_lens=sl, context_lens=torch.zeros_like(sl),
                            block_size=bs, max_block=W, max_query_len=int(seq_lens.max()), device=dev)
    RT.kbar_refresh_tail_triton(kv_cache=cache, k_bar=kbar0, block_table=btd, seq_lens=sl,
                                head_cls=hc, block_size=bs, plan=plan)
    # a decode step has appended to every tail page: new keys there
    cache2 = cache.clone()
    tail = RT.kbar_tail_plan(block_table=btd, seq_lens=sl, block_size=bs, tail_pages=1, device=dev)
    cache2[tail[0]] = (torch.randn(tail[0].numel(), bs, 128, device=dev) * 0.5).to(dtype)
    iqd = torch.from_numpy(iq).to(dev)
    outs = []
    for fused in (False, True):
        kb = kbar0.clone()
        oi = torch.empty(R, K, dtype=torch.int32, device=dev)
        ob = torch.empty(R, K, device=dev)
        kw = dict(idx_q=iqd, k_bar=kb, block_table=btd, seq_lens=sl, image_allow=None, out_idx=oi,
                  out_bias=ob, max_block=W, block_size=bs, local_blocks=lb, decode_query_len=1,
                  idx_scale=IDX_SCALE, prior_floor=1e-4, sigma=1.0, topm=K, budget=K, out_slots=K)
        n0 = _lib.launches()
        if fused:
            RT.route_decode_triton(refresh=(cache2, hc, tail), **kw)
        else:
            RT.kbar_refresh_tail_triton(kv_cache=cache2, k_bar=kb, block_table=btd, seq_lens=sl,
                                        head_cls=hc, block_size=bs, plan=tail)
            RT.route_decode_triton(**kw)
        torch.cuda.synchronize()
        outs.append((kb.cpu().numpy(), oi.cpu().numpy(), ob.cpu().numpy(), _lib.launches() - n0))
    (ka, ia, ba, la), (kf, i_f, bf, lf) = outs
    assert lf == 1 and la == 2, (la, lf)
    assert np.array_equal(ka, kf), "k-bar rows differ"
    np.testing.assert_array_equal(ia, i_f)
    assert np.array_equal(ba, bf)
    # the refreshed rows against the oracle
    ref = kbar0.cpu().numpy().copy()
    pages, ntok = tail[0].cpu().numpy(), tail[1].cpu().numpy()
    O.kbar_paged(cache2.float().cpu().numpy(), pages, ntok, hc.cpu().numpy(), ref)
    assert np.array_equal(kf, ref)
