"""Decode gather attention (split-KV + fused combine) against the oracle and
the reference golden; BASELINE config 3 end to end (k-bar refresh, routing,
attention) at full size on sampled sequences."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from ananta_ocr_b200 import ops
from ananta_ocr_b200 import modeling_deepseekv2 as MD
from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn_decode
from dash_testutil import assert_close_bf16, bf16_round

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_decode_golden_contiguous():
    g = np.load(os.path.join(GOLD, "decode_small.npz"))
    B, H, S, bs, lb = (int(g[x]) for x in ("B", "H", "S", "bs", "lb"))
    q, k, v, iq, ik = O.make_prefill_inputs(int(g["seed"]), B, H, S, 128, 0, 273, 0.0)
    pos = torch.full((B, 1), S - 1, device="cuda")
    out = MD._decode_attend(torch.from_numpy(g["qd"]).cuda(), torch.from_numpy(k).cuda(),
                            torch.from_numpy(v).cuda(), torch.from_numpy(g["topi"]).cuda(),
                            torch.from_numpy(g["bias"]).cuda(), torch.from_numpy(g["valid"]).cuda(),
                            pos, bs, lb * bs, 1.0 / math.sqrt(128))
    # fp32 inputs: computed in fp32 (the reference's _decode_attend is fp32)
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], atol=2e-5, rtol=0)
    # the same query in bf16 takes the split-KV decode kernel
    bf = lambda x: torch.from_numpy(x).cuda().bfloat16()      # noqa: E731
    out16 = MD._decode_attend(bf(g["qd"]), bf(k), bf(v), torch.from_numpy(g["topi"]).cuda(),
                              torch.from_numpy(g["bias"]).cuda(), torch.from_numpy(g["valid"]).cuda(),
                              pos, bs, lb * bs, 1.0 / math.sqrt(128))
    assert_close_bf16(out16.cpu().numpy(), g["out"])


def _paged_setup(rng, R, seq_lens, bs, Hkv, D, extra_pages=7):
    W = int(-(-max(seq_lens) // bs))
    nb = [int(-(-s // bs)) for s in seq_lens]
    P = sum(nb) + extra_pages
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((R, W), np.int32)
    n = 0
    for r in range(R):
        bt[r, :nb[r]] = perm[n:n + nb[r]]
        n += nb[r]
    return bt, P


@pytest.mark.parametrize("splits", [1, 3, 0])
@pytest.mark.parametrize("bs,lb,G", [(64, 4, 1), (32, 2, 2), (128, 1, 1)])
def test_paged_decode_vs_oracle(splits, bs, lb, G):
    rng = np.random.default_rng(bs + splits)
    D, Hkv, K = 128, 2, 8
    H = Hkv * G
    seq_lens = [1, 63, 64, 65, 300, 1000, 2500]
    R = len(seq_lens)
    bt, P = _paged_setup(rng, R, seq_lens, bs, Hkv, D)
    kc = bf16_round((rng.standard_normal((P, bs, Hkv, D)) * 0.5).astype(np.float32))
    vc = bf16_round((rng.standard_normal((P, bs, Hkv, D)) * 0.5).astype(np.float32))
    q = bf16_round(rng.standard_normal((R, H, D)).astype(np.float32))
    idx = np.full((R, K), -1, np.int32)
    bias = rng.standard_normal((R, K)).astype(np.float32)
    for r, s in enumerate(seq_lens):
        hi = (s - 1 - lb * bs) // bs
        if hi >= 0:
            c = rng.choice(hi + 1, size=min(K, hi + 1), replace=False)
            idx[r, :len(c)] = c                      # unsorted on purpose
    out = torch.zeros(R, H, D, dtype=torch.bfloat16, device="cuda")
    ti = torch.from_numpy(idx).cuda()[None].expand(Hkv, -1, -1)
    tb = torch.from_numpy(bias).cuda()[None].expand(Hkv, -1, -1)
    dash_sparse_attn_decode(torch.from_numpy(q).cuda().bfloat16(),
                            torch.from_numpy(kc).cuda().bfloat16(),
                            torch.from_numpy(vc).cuda().bfloat16(), ti, tb,
                            torch.from_numpy(bt).cuda(),
                            torch.tensor(seq_lens, dtype=torch.int32, device="cuda"), Hkv,
                            1.0 / math.sqrt(D), out, 1, local_blocks=lb, sparse_block_size=bs,
                            num_splits=splits)
    ref = O.attend_paged(q, kc, vc, idx, bias, bt, np.arange(R), np.array(seq_lens) - 1, bs,
                         lb * bs, 1.0 / math.sqrt(D))
    assert_close_bf16(out.float().cpu().numpy(), ref)


def test_decode_config3_full_size():
    """batch 64, 10 heads, 27,556-token paged cache (bs=64,
    random block table), window 4, K=32.  Full GPU step (k-bar, route, attend);
    the oracle checks 6 sequences (routes bit-exact, output within tolerance)."""
    R, H, D, S, bs, lb, K = 64, 10, 128, 27556, 64, 4, 32
    nb = -(-S // bs)
    P = R * nb + 28
    g = torch.Generator(device="cuda").manual_seed(0)
    dev = "cuda"
    kc = (torch.randn(P, bs, H, D, generator=g, device=dev) * 0.5).bfloat16()
    vc = (torch.randn(P, bs, H, D, generator=g, device=dev) * 0.5).bfloat16()
    icache = torch.randn(P, bs, 128, generator=g, device=dev) * 0.5
    q = torch.randn(R, H, D, generator=g, device=dev).bfloat16()
    iq = torch.randn(R, 128, generator=g, device=dev) * 0.5
    perm = torch.randperm(P, generator=g, device=dev)[:R * nb].to(torch.int32)
    bt = perm.view(R, nb).contiguous()
    sl = torch.full((R,), S, dtype=torch.int32, device=dev)
    kbar = torch.zeros(P, 128, device=dev)
    plan = RT.kbar_all_plan(block_table=bt, seq_lens=sl, context_lens=torch.zeros_like(sl),
                            block_size=bs, max_block=nb, max_query_len=S, device=dev)
    RT.kbar_refresh_tail_triton(kv_cache=icache, k_bar=kbar, block_table=bt, seq_lens=sl,
                                head_cls=None, block_size=bs, plan=plan)
    oi = torch.empty(R, K, dtype=torch.int32, device=dev)
    ob = torch.empty(R, K, dtype=torch.float32, device=dev)
    RT.route_decode_triton(idx_q=iq, k_bar=kbar, block_table=bt, seq_lens=sl, image_allow=None,
                           out_idx=oi, out_bias=ob, max_block=nb, block_size=bs, local_blocks=lb,
                           decode_query_len=1, idx_scale=128.0 / math.sqrt(128), prior_floor=1e-4,
                           sigma=1.0, topm=K, budget=K, out_slots=K)
    out = torch.zeros(R, H, D, dtype=torch.bfloat16, device=dev)
    dash_sparse_attn_decode(q, kc, vc, oi[None].expand(H, -1, -1), ob[None].expand(H, -1, -1), bt,
                            sl, H, 1.0 / math.sqrt(D), out, 1, local_blocks=lb, sparse_block_size=bs)
    torch.cuda.synchronize()
    bt_np = bt.cpu().numpy()
    for r in [0, 1, 17, 31, 48, 63]:
        pages = bt_np[r]
        cache_r = icache[pages.astype(np.int64)].cpu().numpy()           # [nb, bs, 128]
        kb = np.zeros((nb, 128), np.float32)
        O.kbar_paged(cache_r, np.arange(nb), np.array([min(bs, S - b * bs) for b in range(nb)]),
                     np.zeros(128, np.float32), kb)
        osc = O.scores_paged(iq[r:r + 1].cpu().numpy(), np.array([S - 1]), np.array([0]),
                             np.array([S]), kb, np.arange(nb, dtype=np.int32)[None], bs, lb, nb)
        ri, rb, _ = O.route_select(osc, None, 128.0 / math.sqrt(128), K, K, 1e-4, 1.0)
        np.testing.assert_array_equal(oi[r].cpu().numpy(), ri[0])
        np.testing.assert_allclose(ob[r].cpu().numpy(), rb[0], atol=1e-4)
        need = sorted(set(ri[0][ri[0] >= 0].tolist()) | set(range((S - 1 - lb * bs) // bs, nb)))
        remap = np.full(nb, 0, np.int32)
        remap[need] = np.arange(len(need), dtype=np.int32)
        sub = pages[need].astype(np.int64)
        kc_r = kc[sub].float().cpu().numpy()
        vc_r = vc[sub].float().cpu().numpy()
        ref = O.attend_paged(q[r:r + 1].float().cpu().numpy(), kc_r, vc_r, ri, rb, remap[None],
                             np.array([0]), np.array([S - 1]), bs, lb * bs, 1.0 / math.sqrt(D))
        assert_close_bf16(out[r:r + 1].float().cpu().numpy(), ref)
