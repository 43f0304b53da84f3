"""Pin the page-aware oracle (oracle/page_oracle.py) to the reference's outputs.

tests/golden/page_aware.npz holds what the reference's own functions returned
(tests/golden/make_golden.py, ``page_aware_case``): the indexer's page-id and
candidate-mask builders, ``_dash_block_cand``, ``_uocr_dash_decode_allow`` and the
sglang ``PageIsolationState`` / ``decode_allow_fused`` / ``local_union_fused``
over a short serving trace.  CPU only.
"""
import os

import numpy as np

from oracle import page_oracle as P

GOLD = os.path.join(os.path.dirname(__file__), "golden")
G = np.load(os.path.join(GOLD, "page_aware.npz"))
IMG, PG = P.IMAGE_TOKEN_ID, P.PAGE_TOKEN_ID


def unpack(a, n):
    return np.unpackbits(a, axis=-1)[..., :n].astype(bool)


def test_page_aware_ids_match_reference():
    ids, S = G["ids"], int(G["S"])
    for scope in (0, 1):
        itm, ipi, qpi, _, _ = P.page_aware_ids(ids, IMG, PG, int(G["per_page"]), S, bool(scope))
        np.testing.assert_array_equal(itm, G[f"itm_{scope}"])
        np.testing.assert_array_equal(ipi, G[f"ipi_{scope}"])
        np.testing.assert_array_equal(qpi, G[f"qpi_{scope}"])
    for kl in (1000, 1700):
        _, ipi, qpi, _, _ = P.page_aware_ids(ids, IMG, PG, int(G["per_page"]), kl)
        np.testing.assert_array_equal(ipi, G[f"ipi_kl{kl}"])
        np.testing.assert_array_equal(qpi, G[f"qpi_kl{kl}"])


def test_candidate_masks_match_reference():
    ids, S, bs, nblk = G["ids"], int(G["S"]), int(G["bs"]), int(G["nblk"])
    per = int(G["per_page"])
    B = ids.shape[0]
    pos = np.broadcast_to(np.arange(S), (B, S))
    for scope in (0, 1):
        itm, ipi, qpi, _, _ = P.page_aware_ids(ids, IMG, PG, per, S, bool(scope))
        cm = P.kl_candidate_mask(pos, nblk, itm, bs, True, ipi, qpi)
        np.testing.assert_array_equal(cm, unpack(G[f"cand_page_{scope}"], nblk))
    flat = P.flat_image_token_mask(ids, IMG, S)
    np.testing.assert_array_equal(P.image_block_allow_mask(flat, nblk, bs), G["img_blk"])
    np.testing.assert_array_equal(P.image_block_allow_mask(flat, nblk - 5, bs), G["img_blk_short"])
    cm = P.kl_candidate_mask(pos[:, :300], nblk, flat, bs, False)
    np.testing.assert_array_equal(cm, unpack(G["cand_flat"], nblk))
    bc = P.dash_block_cand(ids, IMG, PG, per, S, pos, nblk, bs, True)
    np.testing.assert_array_equal(bc, unpack(G["block_cand"], nblk))
    itm, ipi, qpi, _, _ = P.page_aware_ids(ids, IMG, PG, per, S)
    pos2 = np.minimum(pos + 37, S + 20)
    cm = P.kl_candidate_mask(pos2, nblk, itm, bs, True, ipi, qpi)
    np.testing.assert_array_equal(cm, unpack(G["cand_pos_shift"], nblk))


def test_descriptors_restate_the_membership_mask():
    """The compact (lo, hi, bits) form gives exactly the reference's same-page
    block test, gap blocks (pages without image tokens in between) included."""
    ids, S, bs, nblk = G["ids"], int(G["S"]), int(G["bs"]), int(G["nblk"])
    _, ipi, qpi, _, _ = P.page_aware_ids(ids, IMG, PG, int(G["per_page"]), S, True)
    lo, hi, bits = P.page_descriptors(ipi, nblk, bs)
    kp = P.page_blocks(ipi, nblk, bs)
    for q in range(-1, int(ipi.max()) + 2):
        ref = (kp == q).any(-1) & (q >= 0)
        k = q - lo
        inr = (lo >= 0) & (q >= lo) & (q <= hi) & (q >= 0)
        kk = np.clip(k, 0, 32 * bits.shape[-1] - 1)
        bit = (np.take_along_axis(bits, (kk >> 5)[..., None], -1)[..., 0] >> (kk & 31)) & 1
        np.testing.assert_array_equal(inr & (bit == 1), ref)
    gap = (hi - lo + 1 > np.array([[len(set(b[b >= 0].tolist())) for b in row] for row in kp]))
    assert gap.any(), "fixture has no block with a page gap"


def test_decode_allow_matches_reference():
    ids, bs = G["ids"], int(G["bs"])
    st = P.decode_allow_prefill(ids[:, :1300], IMG, PG, int(G["per_page"]), bs)
    for k in ("bmin", "bmax", "pp", "mcum"):
        np.testing.assert_array_equal(st[k], G[f"dec_{k}"])
    total = 1300
    for k, last in enumerate(G["dec_ids"]):
        allow = P.decode_allow_step(st, last, total + 1, PG, bs)
        np.testing.assert_array_equal(allow, unpack(G["dec_allow"][k], allow.shape[1]))
        total += 1


def test_serving_trace_matches_reference():
    bs, per, Pn, W = int(G["sg_bs"]), int(G["sg_per"]), int(G["sg_P"]), int(G["sg_W"])
    bt = G["sg_bt"]
    st = P.new_slot_state(Pn * bs)
    lens = {}
    for i in range(int(G["sg_steps"])):
        g = {k[len(f"sg{i}_"):]: G[k] for k in G.files if k.startswith(f"sg{i}_")}
        rows = g["rows"]
        q_page = P.page_state_step(st, g["ids"], g["q_start"], g["start_pos"], bt[rows],
                                   g["slots"], Pn * bs, bs, per, IMG, PG,
                                   num_decode_tokens=int(g["n_dec"]))
        np.testing.assert_array_equal(q_page, g["q_page"])
        for name, key in (("img_page", "slot_img_page"), ("marker_cum", "slot_marker_cum"),
                          ("img_run", "slot_img_run"), ("prompt_pages", "slot_prompt_pages")):
            np.testing.assert_array_equal(st[name], g[key])
        allow = P.build_query_allow(st["img_page"], bt[rows], g["q_start"], q_page, W, Pn, bs)
        np.testing.assert_array_equal(allow, g["allow"])
        if "decode_allow" in g:
            da = P.decode_allow(st["img_page"], bt[rows], q_page, g["seq_lens"], W, Pn, bs)
            np.testing.assert_array_equal(da, g["decode_allow"] != 0)
            lu = P.local_union(da, g["seq_lens"], W, bs, 2)
            np.testing.assert_array_equal(lu, g["local_union"] != 0)
        for j, r in enumerate(rows):
            lens[r] = int(g["start_pos"][j]) + int(g["q_start"][j + 1] - g["q_start"][j])


def test_serving_plans_match_reference_golden():
    """kbar_all_plan / kbar_tail_plan / prefill_row2req restated in the oracle
    against the sglang wheel's own outputs."""
    g = np.load(os.path.join(GOLD, "serving_plan.npz"))
    for bs in (16, 32, 64):
        seq, ctx, bt, cu = g[f"seq_{bs}"], g[f"ctx_{bs}"], g[f"bt_{bs}"], g[f"cu_{bs}"]
        W = bt.shape[1]
        for full, mb in ((True, W), (False, W - 3)):
            p, t = P.plan_prefill_pages(bt, seq, ctx, bs, mb, int((seq - ctx).max()))
            np.testing.assert_array_equal(p, g[f"all_{bs}_{full}_pages"])
            np.testing.assert_array_equal(t, g[f"all_{bs}_{full}_ntok"])
        for tp in (1, 3):
            p, t = P.plan_tail_pages(bt, seq, bs, tp)
            np.testing.assert_array_equal(p, g[f"tail_{bs}_{tp}_pages"])
            np.testing.assert_array_equal(t, g[f"tail_{bs}_{tp}_ntok"])
        np.testing.assert_array_equal(P.rows_to_requests(cu), g[f"row2req_{bs}"])
