"""Page-aware candidate domain on the GPU: the page kernels against the numpy
oracle (oracle/page_oracle.py, itself pinned to the reference by
test_page_oracle_golden.py) and against the reference's golden outputs, and
the router's compact page mode against the dense candidate mask (bit-exact
block lists; biases bit-exact between the two GPU paths, within 1e-4 of the
oracle, whose host log() may differ by an ulp)."""
import math
import os
import types

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from oracle import page_oracle as P
from ananta_ocr_b200 import ops, pages
from ananta_ocr_b200 import modeling_deepseekv2 as MD
from ananta_ocr_b200 import modeling_anantaocr as MA
from ananta_ocr_b200._sparse_base_impl import DeepseekV2IndexerPages
import ananta_ocr_b200._sparse_base_impl as SB
from ananta_ocr_b200.unlimited_dash_ops import page_state as PS
from ananta_ocr_b200.unlimited_dash_ops import decode_meta_triton as DM

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
IMG, PG = P.IMAGE_TOKEN_ID, P.PAGE_TOKEN_ID
IDX_SCALE = 128.0 / math.sqrt(128)


def golden():
    return np.load(os.path.join(GOLD, "page_aware.npz"))


def unpack(a, n):
    return np.unpackbits(a, axis=-1)[..., :n].astype(bool)


def docs(seed, S, variants=None):
    rng = np.random.default_rng(seed)
    variants = variants or [
        dict(n_pages=max(1, S // 400), page_tokens=273, text_in_page=3, empty_pages=1,
             response_pages=2),
        dict(n_pages=max(1, S // 300), page_tokens=200, markers=False),
        dict(n_pages=max(1, S // 40), page_tokens=20, empty_pages=6, lead_images=10,
             response_pages=3),
        dict(n_pages=0, page_tokens=10, response_pages=2),            # text only
    ]
    return np.stack([P.make_document_ids(rng, S, **v) for v in variants])


class Indexer(DeepseekV2IndexerPages):
    def __init__(self, bs, per=100, bucket=True):
        self.block_size = bs
        self.per_page_image_tokens = per
        self.image_bucket_constraint = bucket
        self.image_token_id = IMG
        self.page_token_id = PG


# ---------------------------------------------------------------------------
# dash_page_ids
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("S", [1, 700, 4096, 4097, 70_000])
@pytest.mark.parametrize("scope", [False, True])
def test_page_ids_rule0_match_oracle(S, scope):
    ids = docs(11 + S, S)
    r = pages.page_ids(torch.from_numpy(ids).cuda(), image_token_id=IMG, page_token_id=PG,
                       per_page=100, key_length=S, rule=0, page_scope_prefill=scope,
                       page_dtype=torch.int64)
    img, ipi, qpi, pp, mcum = P.page_aware_ids(ids, IMG, PG, 100, S, scope)
    assert np.array_equal(r["image_mask"].cpu().numpy(), img)
    assert np.array_equal(r["image_page"].cpu().numpy(), ipi)
    assert np.array_equal(r["query_page"].cpu().numpy(), qpi)
    assert np.array_equal(r["prompt_pages"].cpu().numpy(), pp)
    assert np.array_equal(r["marker_count"].cpu().numpy(), mcum)
    assert np.array_equal(r["n_image"].cpu().numpy(), img.sum(-1))
    assert np.array_equal(r["n_query"].cpu().numpy(), (qpi >= 0).sum(-1))


@pytest.mark.parametrize("kl", [0, 500, 1000, 1700])
def test_page_ids_key_length_pad_and_truncate(kl):
    ids = docs(5, 1000)
    r = pages.page_ids(torch.from_numpy(ids).cuda(), image_token_id=IMG, page_token_id=PG,
                       per_page=100, key_length=kl, rule=0)
    img, ipi, qpi, pp, mcum = P.page_aware_ids(ids, IMG, PG, 100, kl)
    assert np.array_equal(r["image_page"].cpu().numpy(), ipi)
    assert np.array_equal(r["query_page"].cpu().numpy(), qpi)
    assert np.array_equal(r["prompt_pages"].cpu().numpy(), pp)


@pytest.mark.parametrize("bs", [16, 64, 128, 256])
@pytest.mark.parametrize("S", [1000, 9000])
def test_page_descriptors_match_oracle(bs, S):
    ids = docs(3 + bs, S)
    nblk = -(-S // bs)
    for n_blocks in (nblk, nblk + 3, max(1, nblk - 2)):
        r = pages.page_ids(torch.from_numpy(ids).cuda(), image_token_id=IMG, page_token_id=PG,
                           per_page=100, key_length=S, rule=0, block_size=bs, n_blocks=n_blocks,
                           has_image=True)
        _, ipi, _, _, _ = P.page_aware_ids(ids, IMG, PG, 100, S)
        lo, hi, bits = P.page_descriptors(ipi, n_blocks, bs)
        assert np.array_equal(r["lo"].cpu().numpy(), lo)
        assert np.array_equal(r["hi"].cpu().numpy(), hi)
        assert np.array_equal(r["bits"].cpu().numpy().view(np.uint32), bits)
        img = P.pad_ids(ids, S) == IMG
        assert np.array_equal(r["has_image"].cpu().numpy(), P.image_block_allow_mask(img, n_blocks, bs))
        # the separate descriptor kernel from page ids gives the same
        lo2, hi2, bits2 = pages.page_blocks(torch.from_numpy(ipi).cuda(), n_blocks, bs,
                                            length=min(S, n_blocks * bs))
        assert np.array_equal(lo2.cpu().numpy(), lo)
        assert np.array_equal(hi2.cpu().numpy(), hi)
        assert np.array_equal(bits2.cpu().numpy().view(np.uint32), bits)


def test_page_ids_rule1_decode_state_matches_oracle():
    ids = docs(9, 1300)
    bs = 64
    nblk = -(-1300 // bs)
    r = pages.page_ids(torch.from_numpy(ids).cuda(), image_token_id=IMG, page_token_id=PG,
                       per_page=100, key_length=1300, rule=1, block_size=bs, n_blocks=nblk,
                       bits=False)
    st = P.decode_allow_prefill(ids, IMG, PG, 100, bs)
    assert np.array_equal(r["lo"].cpu().numpy(), st["bmin"])
    assert np.array_equal(r["hi"].cpu().numpy(), st["bmax"])
    assert np.array_equal(r["prompt_pages"].cpu().numpy(), st["pp"])
    assert np.array_equal(r["marker_count"].cpu().numpy(), st["mcum"])


# ---------------------------------------------------------------------------
# reference-named mirrors against the reference's golden outputs
# ---------------------------------------------------------------------------
def test_indexer_mirrors_match_reference_golden():
    G = golden()
    ids, S, bs, nblk = G["ids"], int(G["S"]), int(G["bs"]), int(G["nblk"])
    B = ids.shape[0]
    idx = Indexer(bs, int(G["per_page"]))
    tid = torch.from_numpy(ids).cuda()
    pos = torch.arange(S, device="cuda")[None].expand(B, -1)
    for scope in (0, 1):
        SB._PAGE_SCOPE_PREFILL = bool(scope)
        try:
            itm, ipi, qpi = idx._build_page_aware_ids(tid, IMG, PG, S)
        finally:
            SB._PAGE_SCOPE_PREFILL = False
        assert ipi.dtype == torch.int64 and qpi.dtype == torch.int64 and itm.dtype == torch.bool
        assert np.array_equal(itm.cpu().numpy(), G[f"itm_{scope}"])
        assert np.array_equal(ipi.cpu().numpy(), G[f"ipi_{scope}"])
        assert np.array_equal(qpi.cpu().numpy(), G[f"qpi_{scope}"])
        cm = idx._build_kl_candidate_mask(pos, nblk, itm, B, S, ipi, qpi)
        assert cm.shape == (B, 1, S, nblk)
        assert np.array_equal(cm[:, 0].cpu().numpy(), unpack(G[f"cand_page_{scope}"], nblk))
    for kl in (1000, 1700):
        _, ipi, qpi = idx._build_page_aware_ids(tid, IMG, PG, kl)
        assert np.array_equal(ipi.cpu().numpy(), G[f"ipi_kl{kl}"])
        assert np.array_equal(qpi.cpu().numpy(), G[f"qpi_kl{kl}"])
    flat = idx._build_flat_image_token_mask(tid, IMG, S)
    assert np.array_equal(idx._build_image_block_allow_mask(flat, nblk).cpu().numpy(), G["img_blk"])
    assert np.array_equal(idx._build_image_block_allow_mask(flat, nblk - 5).cpu().numpy(),
                          G["img_blk_short"])
    idx.image_bucket_constraint = False
    cm = idx._build_kl_candidate_mask(pos[:, :300], nblk, flat, B, 300)
    assert np.array_equal(cm[:, 0].cpu().numpy(), unpack(G["cand_flat"], nblk))
    idx.image_bucket_constraint = True
    itm, ipi, qpi = MD._dash_page_ids(None, idx, tid, S)
    bc = MD._dash_block_cand(None, idx, types.SimpleNamespace(q_chunk=512), pos, itm, ipi, qpi,
                             nblk, B, S)
    assert np.array_equal(bc.cpu().numpy(), unpack(G["block_cand"], nblk))
    pos2 = torch.clamp(pos + 37, max=S + 20)
    cm = idx._build_kl_candidate_mask(pos2, nblk, itm, B, S, ipi, qpi)
    assert np.array_equal(cm[:, 0].cpu().numpy(), unpack(G["cand_pos_shift"], nblk))


def test_page_aware_ids_none_contract():
    idx = Indexer(64)
    text = torch.randint(0, 1000, (2, 300), device="cuda")
    assert idx._build_page_aware_ids(text, IMG, PG, 300) == (None, None, None)
    assert idx._build_page_aware_ids(None, IMG, PG, 300) == (None, None, None)
    assert idx._build_page_aware_ids(text, IMG, None, 300) == (None, None, None)
    assert idx._build_flat_image_token_mask(text, IMG, 300) is None


def test_decode_allow_mirror_matches_reference_golden():
    G = golden()
    ids, bs = G["ids"], int(G["bs"])
    idx = Indexer(bs, int(G["per_page"]))

    class Cache:
        n = 0

        def get_seq_length(self):
            return self.n
    cache = Cache()
    assert MA._uocr_dash_decode_allow(idx, torch.from_numpy(ids[:, :1300]).cuda(), cache) is None
    st = cache._uocr_pg
    for k in ("bmin", "bmax", "pp", "mcum"):
        assert np.array_equal(st[k].cpu().numpy(), G[f"dec_{k}"]), k
    cache.n = 1300
    for k, last in enumerate(G["dec_ids"]):
        allow = MA._uocr_dash_decode_allow(idx, torch.from_numpy(last[:, None]).cuda(), cache)
        assert np.array_equal(allow.cpu().numpy(), unpack(G["dec_allow"][k], allow.shape[1]))
        cache.n += 1


def test_serving_mirrors_match_reference_golden():
    G = golden()
    bs, per, Pn, W = int(G["sg_bs"]), int(G["sg_per"]), int(G["sg_P"]), int(G["sg_W"])
    bt = G["sg_bt"]
    pst = PS.PageIsolationState({"image_token_id": IMG, "page_token_id": PG,
                                 "per_page_image_tokens": per}, bs)
    for i in range(int(G["sg_steps"])):
        g = {k[len(f"sg{i}_"):]: G[k] for k in G.files if k.startswith(f"sg{i}_")}
        rows = g["rows"]
        q_start = torch.from_numpy(g["q_start"]).cuda()
        T = int(g["q_start"][-1])
        layout = PS.BatchLayout(num_tokens=T, num_reqs=len(rows), q_start=q_start,
                                start_pos=torch.from_numpy(g["start_pos"]).cuda(),
                                block_table=torch.from_numpy(bt[rows]).cuda(),
                                req_of_token=PS._req_of_token(q_start, T),
                                num_decode_tokens=int(g["n_dec"]))
        q_page = pst.step(torch.from_numpy(g["ids"]).cuda(), layout,
                          torch.from_numpy(g["slots"]).cuda(), Pn * bs)
        assert np.array_equal(q_page.cpu().numpy(), g["q_page"]), i
        for name in ("img_page", "marker_cum", "img_run", "prompt_pages"):
            got = getattr(pst, f"_slot_{name}").cpu().numpy()
            assert np.array_equal(got, g[f"slot_{name}"]), (i, name)
        # the bounds the step maintains equal a full recompute
        lo, hi = pst.block_page_bounds(Pn)
        assert np.array_equal(pst._blk_lo.cpu().numpy(), lo.cpu().numpy().astype(np.int32))
        assert np.array_equal(pst._blk_hi.cpu().numpy(), hi.cpu().numpy().astype(np.int32))
        allow = pst.build_query_allow(layout, q_page, W, Pn)
        assert np.array_equal(allow.cpu().numpy(), g["allow"]), i
        if "decode_allow" in g:
            sl = torch.from_numpy(g["seq_lens"]).cuda()
            da = DM.decode_allow_fused(block_table=layout.block_table, page_state=pst,
                                       q_page=q_page, seq_lens=sl, max_block=W, num_blocks=Pn,
                                       block_size=bs)
            assert np.array_equal(da.cpu().numpy(), g["decode_allow"]), i
            lu = DM.local_union_fused(allow=da, seq_lens=sl,
                                      out=torch.zeros(len(rows), W, dtype=torch.int8, device="cuda"),
                                      max_block=W, block_size=bs, local_blocks=2)
            assert np.array_equal(lu.cpu().numpy(), g["local_union"]), i


def test_decode_meta_fused_equals_step():
    """The one-token-per-request form (no token layout) gives the layout form's
    pages and slot state."""
    rng = np.random.default_rng(4)
    bs, per, Pn, R = 16, 24, 64, 4
    cfg = {"image_token_id": IMG, "page_token_id": PG, "per_page_image_tokens": per}
    a, b = PS.PageIsolationState(cfg, bs), PS.PageIsolationState(cfg, bs)
    bt = torch.from_numpy(rng.permutation(Pn)[: R * 8].reshape(R, 8)).cuda()
    lens = np.zeros(R, np.int64)
    for step in range(40):
        tok = rng.choice([IMG, PG, 5, 77, P.MM_PAD_SHIFT + 3], size=R, p=[.5, .1, .2, .1, .1])
        pos = lens.copy()
        slots = np.array([int(bt[r, pos[r] // bs]) * bs + pos[r] % bs for r in range(R)])
        lens += 1
        q_start = torch.arange(R + 1, device="cuda")
        layout = PS.BatchLayout(num_tokens=R, num_reqs=R, q_start=q_start,
                                start_pos=torch.from_numpy(pos).cuda(), block_table=bt,
                                req_of_token=PS._req_of_token(q_start, R), num_decode_tokens=R)
        ids = torch.from_numpy(tok).cuda()
        sm = torch.from_numpy(slots).cuda()
        qa = a.step(ids, layout, sm, Pn * bs)
        qb, _ = DM.decode_meta_fused(input_ids=ids, block_table=bt,
                                     seq_lens=torch.from_numpy(lens).cuda().to(torch.int32),
                                     slot_mapping=sm, page_state=b, num_slots=Pn * bs,
                                     block_size=bs)
        assert torch.equal(qa, qb)
        for name in ("img_page", "marker_cum", "img_run", "prompt_pages"):
            assert torch.equal(getattr(a, f"_slot_{name}"), getattr(b, f"_slot_{name}"))
        assert torch.equal(a._blk_lo, b._blk_lo) and torch.equal(a._blk_hi, b._blk_hi)


# ---------------------------------------------------------------------------
# router page mode == dense candidate mask
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("S,bs,lb,K,topm", [(1500, 64, 4, 8, 8), (3000, 64, 4, 16, 24),
                                            (2600, 128, 2, 8, 8)])
def test_route_page_mode_contiguous_bitexact(S, bs, lb, K, topm):
    ids = docs(21 + S, S)
    B = ids.shape[0]
    rng = np.random.default_rng(S)
    iq = (rng.standard_normal((B, S, 128)) * 0.5).astype(np.float32)
    ik = (rng.standard_normal((B, S, 128)) * 0.5).astype(np.float32)
    nblk = -(-S // bs)
    kbar = ops.kbar_pool_contig(torch.from_numpy(ik).cuda(), None, bs)
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    dom = MD.page_domain_from_ids(torch.from_numpy(ids).cuda(), image_token_id=IMG,
                                  page_token_id=PG, per_page=100, block_size=bs, nblk=nblk)
    scores = torch.empty(B * S, nblk, dtype=torch.float32, device="cuda")
    idx, bias = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                          prior_floor=1e-4, sigma=1.0, topm=topm, K=K,
                          idx_q=torch.from_numpy(iq).cuda().view(B * S, 128), kbar=kbar,
                          scores_out=scores, page=dom)
    cand = P.dash_block_cand(ids, IMG, PG, 100, S, np.broadcast_to(np.arange(S), (B, S)), nblk,
                             bs, True)
    assert cand is not None
    oi, ob, _ = O.route_select(scores.cpu().numpy(), cand.reshape(B * S, nblk), IDX_SCALE, topm,
                               K, 1e-4, 1.0)
    assert np.array_equal(idx.cpu().numpy(), oi)
    # log() of the device and of the host C library may differ by an ulp
    np.testing.assert_allclose(bias.cpu().numpy(), ob, atol=1e-4)
    # the dense path of the same domain gives the same lists
    idx2, bias2 = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                            prior_floor=1e-4, sigma=1.0, topm=topm, K=K,
                            idx_q=torch.from_numpy(iq).cuda().view(B * S, 128), kbar=kbar,
                            cand=torch.from_numpy(cand.reshape(B * S, nblk)).cuda())
    assert torch.equal(idx, idx2) and torch.equal(bias, bias2)
    # page restriction changes the routes of image-page queries
    idx3, _ = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                        prior_floor=1e-4, sigma=1.0, topm=topm, K=K,
                        idx_q=torch.from_numpy(iq).cuda().view(B * S, 128), kbar=kbar)
    assert not torch.equal(idx, idx3)


def test_route_page_mode_paged_bitexact():
    """Serving path: page bounds of physical blocks through the block table,
    one prefill step then decode steps, routes == dense image_allow routes."""
    rng = np.random.default_rng(8)
    bs, lb, K, per, Pn, R, W = 16, 2, 8, 24, 160, 3, 48
    cfg = {"image_token_id": IMG, "page_token_id": PG, "per_page_image_tokens": per}
    pst = PS.PageIsolationState(cfg, bs)
    bt_np = rng.permutation(Pn)[: R * W].reshape(R, W).astype(np.int64)
    bt = torch.from_numpy(bt_np).cuda()
    lens = [600, 450, 700]
    doc = [P.make_document_ids(rng, n, n_pages=n // 60, page_tokens=40, text_in_page=2,
                               response_pages=0) for n in lens]
    toks = np.concatenate(doc)
    qs = np.concatenate([[0], np.cumsum(lens)])
    T = int(qs[-1])
    slots = np.concatenate([[bt_np[r, p // bs] * bs + p % bs for p in range(lens[r])]
                            for r in range(R)])
    q_start = torch.from_numpy(qs).cuda()
    layout = PS.BatchLayout(num_tokens=T, num_reqs=R, q_start=q_start,
                            start_pos=torch.zeros(R, dtype=torch.int64, device="cuda"),
                            block_table=bt, req_of_token=PS._req_of_token(q_start, T))
    q_page = pst.step(torch.from_numpy(toks).cuda(), layout, torch.from_numpy(slots).cuda(),
                      Pn * bs)
    kbar = (torch.randn(Pn, 128, device="cuda") * 0.5).contiguous()
    iq = (torch.randn(T, 128, device="cuda") * 0.5).contiguous()
    seqs = ops.Seqs(n_seq=R, q_start=q_start.to(torch.int32),
                    pos0=torch.zeros(R, dtype=torch.int32, device="cuda"),
                    kv_len_t=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                    total_rows=T, max_q_len=max(lens))
    bt32 = bt.to(torch.int32)
    kw = dict(width=W, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE, prior_floor=1e-4,
              sigma=1.0, topm=K, K=K, idx_q=iq, kbar=kbar, block_table=bt32)
    i1, b1 = ops.route(seqs, page=pst.candidate_domain(q_page), **kw)
    allow = pst.build_query_allow(layout, q_page, W, Pn)
    i2, b2 = ops.route(seqs, cand=allow, **kw)
    assert torch.equal(i1, i2) and torch.equal(b1, b2)
    i3, _ = ops.route(seqs, **kw)
    assert not torch.equal(i1, i3)
    # decode steps
    for step in range(3):
        tok = rng.choice([PG, 5, 77], size=R, p=[.4, .3, .3])
        pos = np.array(lens)
        sl = np.array([bt_np[r, pos[r] // bs] * bs + pos[r] % bs for r in range(R)])
        lens = [n + 1 for n in lens]
        seq_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
        qd, _ = DM.decode_meta_fused(input_ids=torch.from_numpy(tok).cuda(), block_table=bt,
                                     seq_lens=seq_lens, slot_mapping=torch.from_numpy(sl).cuda(),
                                     page_state=pst, num_slots=Pn * bs, block_size=bs)
        da = DM.decode_allow_fused(block_table=bt, page_state=pst, q_page=qd, seq_lens=seq_lens,
                                   max_block=W, num_blocks=Pn, block_size=bs)
        iqd = (torch.randn(R, 128, device="cuda") * 0.5).contiguous()
        sd = ops.Seqs(n_seq=R, q_len=1, kv_len=0, kv_len_t=seq_lens, max_q_len=1)
        kw.update(idx_q=iqd)
        j1, c1 = ops.route(sd, page=pst.candidate_domain(qd), **kw)
        j2, c2 = ops.route(sd, cand=da, **kw)
        assert torch.equal(j1, j2) and torch.equal(c1, c2)


def test_cpu_tensors_raise():
    with pytest.raises(RuntimeError):
        pages.page_ids(torch.zeros(1, 10, dtype=torch.int64), image_token_id=IMG,
                       page_token_id=PG, per_page=1, key_length=10)


def test_serving_plans_match_reference_golden_and_oracle():
    """The serving-plan kernel behind kbar_all_plan / kbar_tail_plan /
    prefill_row2req against the sglang wheel's outputs, plus a larger random
    case against the oracle; the caller's out buffers are filled in place."""
    from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
    g = np.load(os.path.join(GOLD, "serving_plan.npz"))
    dev = torch.device("cuda")
    for bs in (16, 32, 64):
        seq, ctx, bt, cu = g[f"seq_{bs}"], g[f"ctx_{bs}"], g[f"bt_{bs}"], g[f"cu_{bs}"]
        tbt, tsl, tctx = (torch.from_numpy(x).to(dev) for x in (bt, seq, ctx))
        W = bt.shape[1]
        for full, mb in ((True, W), (False, W - 3)):
            p, t = RT.kbar_all_plan(block_table=tbt, seq_lens=tsl, context_lens=tctx, block_size=bs,
                                    max_block=mb, max_query_len=int((seq - ctx).max()), device=dev)
            np.testing.assert_array_equal(p.cpu().numpy(), g[f"all_{bs}_{full}_pages"])
            np.testing.assert_array_equal(t.cpu().numpy(), g[f"all_{bs}_{full}_ntok"])
        for tp in (1, 3):
            buf = (torch.full((64,), -7, dtype=torch.int64, device=dev),
                   torch.full((64,), -7, dtype=torch.int32, device=dev))
            p, t = RT.kbar_tail_plan(block_table=tbt, seq_lens=tsl, block_size=bs, tail_pages=tp,
                                     device=dev, out=buf)
            assert p.data_ptr() == buf[0].data_ptr()
            np.testing.assert_array_equal(p.cpu().numpy(), g[f"tail_{bs}_{tp}_pages"])
            np.testing.assert_array_equal(t.cpu().numpy(), g[f"tail_{bs}_{tp}_ntok"])
        r2r = RT.prefill_row2req(cu_seqlens_q=torch.from_numpy(cu).to(dev), device=dev,
                                 total_q=int(cu[-1]))
        np.testing.assert_array_equal(r2r.cpu().numpy(), g[f"row2req_{bs}"])
    rng = np.random.default_rng(3)
    R, bs = 300, 32
    seq = rng.integers(0, 30000, R)
    ctx = np.minimum(seq, rng.integers(0, 30000, R))
    bt = rng.integers(0, 1 << 20, (R, 1000)).astype(np.int32)
    cu = np.concatenate([[0], np.cumsum(seq - ctx)]).astype(np.int32)
    p, t = RT.kbar_all_plan(block_table=torch.from_numpy(bt).to(dev),
                            seq_lens=torch.from_numpy(seq).to(dev),
                            context_lens=torch.from_numpy(ctx).to(dev), block_size=bs,
                            max_block=1000, max_query_len=int((seq - ctx).max()), device=dev)
    rp, rt_ = P.plan_prefill_pages(bt, seq, ctx, bs, 1000, int((seq - ctx).max()))
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(t.cpu().numpy(), rt_)
    r2r = RT.prefill_row2req(cu_seqlens_q=torch.from_numpy(cu).to(dev), device=dev)
    np.testing.assert_array_equal(r2r.cpu().numpy(), P.rows_to_requests(cu))


def test_page2d_coordinates_match_reference_golden():
    """Page2D coordinates over a serving trace (chunked prefills, decode
    steps, a state row reused by a new request) against the wheel's
    PageCoordState.step / decode_meta_fused, and the cos/sin tables against
    PageRope2D.cos_sin (fp32) and cos_sin_2d_fused (bf16)."""
    from ananta_ocr_b200.unlimited_dash_ops import page2d_rope as PR
    from ananta_ocr_b200.unlimited_dash_ops import decode_meta_triton as DMT
    from ananta_ocr_b200.unlimited_dash_ops import page_state as PSM
    g = np.load(os.path.join(GOLD, "page_coords.npz"))
    dev = torch.device("cuda")
    IMG, PG = 128815, 128827
    cfg = {"image_token_id": IMG, "page_token_id": PG, "per_page_image_tokens": 24}
    sbs, P = int(g["sbs"]), int(g["P"])
    coord = PR.PageCoordState(cfg, max_reqs=int(g["max_reqs"]), max_pages=int(g["max_pages"]))
    pst = PSM.PageIsolationState(cfg, sbs)
    rope = PR.PageRope2D(128, 10000.0, 256.0, 1, "resample", page_mod=int(g["page_mod"]))
    np.testing.assert_array_equal(rope.inv_tok.numpy(), g["inv_tok"])
    np.testing.assert_array_equal(rope.inv_page.numpy(), g["inv_page"])
    bt = torch.from_numpy(g["bt"]).to(dev)
    for i in range(int(g["steps"])):
        rows = g[f"s{i}_rows"]
        ids = torch.from_numpy(g[f"s{i}_ids"]).to(dev)
        btab = bt[torch.from_numpy(rows).to(dev)]
        if int(g[f"s{i}_decode"]):
            seq = torch.from_numpy(g[f"s{i}_start_pos"] + 1).to(dev, torch.int32)
            q_page, (tok, page) = DMT.decode_meta_fused(
                input_ids=ids, block_table=btab, seq_lens=seq,
                slot_mapping=torch.from_numpy(g[f"s{i}_slots"]).to(dev), page_state=pst,
                coord_state=coord, num_slots=P * sbs, block_size=sbs)
            np.testing.assert_array_equal(q_page.cpu().numpy(), g[f"s{i}_q_page"])
            T = tok.shape[0]
            cos = torch.zeros(T, 128, dtype=torch.bfloat16, device=dev)
            sin = torch.zeros_like(cos)
            DMT.cos_sin_2d_fused(rope=rope, tok_pos=tok, page_pos=page, dtype=torch.bfloat16,
                                 out_cos=cos, out_sin=sin)
            # the interpreted Triton golden truncates to bf16 (the CPU
            # interpreter's conversion); the GPU kernel and torch round to
            # nearest: compare with the torch fp32 table rounded to nearest
            for got, key, k32 in ((cos, "cos_fused", "cos32"), (sin, "sin_fused", "sin32")):
                a = got.view(torch.int16).cpu().numpy().astype(np.int32)
                rn = torch.from_numpy(g[f"s{i}_{k32}"]).bfloat16().view(torch.int16).numpy()
                assert np.abs(a - rn.astype(np.int32)).max() <= 1
                assert (a == rn).mean() >= 0.99
                assert np.abs(a - g[f"s{i}_{key}"].astype(np.int32)).max() <= 1
        else:
            layout = types.SimpleNamespace(
                num_tokens=int(ids.shape[0]), q_start=torch.from_numpy(g[f"s{i}_q_start"]).to(dev),
                start_pos=torch.from_numpy(g[f"s{i}_start_pos"]).to(dev), block_table=btab,
                num_decode_tokens=0, gen_start=None)
            tok, page = coord.step(ids, layout)
        np.testing.assert_array_equal(tok.cpu().numpy(), g[f"s{i}_tok"])
        np.testing.assert_array_equal(page.cpu().numpy(), g[f"s{i}_page"])
        c32, s32 = rope.cos_sin(tok, page, torch.float32)
        np.testing.assert_allclose(c32.cpu().numpy(), g[f"s{i}_cos32"], atol=2e-6, rtol=0)
        np.testing.assert_allclose(s32.cpu().numpy(), g[f"s{i}_sin32"], atol=2e-6, rtol=0)
