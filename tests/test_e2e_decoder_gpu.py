"""The end-to-end decoder (ananta_ocr_b200/e2e_decoder.py) on a small
configuration: a paged prefill of S tokens followed by one decode step gives
the last-token logits of a prefill of S + 1 tokens (KV cache, index cache,
k-bar refresh, decode routing and decode attention consistent with the
prefill path), and the decode step replayed from a CUDA graph equals the
eager step bit for bit.  The two paths sum in different orders (prefill vs
decode attention kernels, grouped vs dense MoE GEMMs), so the logits agree to
2% of their largest magnitude.  One layer of the model is also checked
against the CPU oracle in prefill and in the decode step: its k-bar rows
(bitwise), routed lists (bit-exact) and attention output (bf16 tolerance)."""
import pytest
import torch

from ananta_ocr_b200.e2e_decoder import DashDecoder, DecoderConfig

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=256, heads=2, kv_heads=2, layers=3, vocab=1000, dense_ffn=512, moe_ffn=128,
             experts=8, topk=2, shared=1)
CFGS = {
    # 64-token blocks, 2-block window, 4 routed blocks
    "bs64": DecoderConfig(**SMALL, block_size=64, local_blocks=2, K=4, topm=4, slots=4),
    # the checkpoint's DASH settings: 32-token blocks (one page each), 4-block
    # window, 12 routed blocks out of an entmax window of 16, 16 output slots
    "bs32": DecoderConfig(**SMALL),
}
CFG = CFGS["bs64"]


@pytest.fixture(params=sorted(CFGS))
def cfg(request):
    global CFG
    CFG = CFGS[request.param]
    yield CFG
    CFG = CFGS["bs64"]


def make(seed=3):
    return DashDecoder(CFG, batch=2, max_len=420, device=torch.device("cuda"), seed=seed)


def test_prefill_plus_decode_equals_longer_prefill(cfg):
    S = 333
    ids = torch.randint(0, CFG.vocab, (2, S + 1), generator=torch.Generator().manual_seed(0)).cuda()
    full = make()
    ref = full.prefill(full.embed[ids])
    part = make()
    part.prefill(part.embed[ids[:, :S]])
    part.tok.copy_(ids[:, S])
    got = part.decode_step()
    assert torch.isfinite(got).all() and torch.isfinite(ref).all()
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 0.02 * ref.float().abs().max().item(), err
    assert torch.equal(part.seq_lens, torch.full_like(part.seq_lens, S + 1))


def test_graph_decode_equals_eager(cfg):
    S = 200
    ids = torch.randint(0, CFG.vocab, (2, S), generator=torch.Generator().manual_seed(1)).cuda()
    a, b = make(5), make(5)
    a.prefill(a.embed[ids])
    b.prefill(b.embed[ids])
    a.tok.fill_(7)
    b.tok.fill_(7)
    eager = [a.decode_step().clone() for _ in range(3)]
    b.decode_step()                       # warm-up (eager), then rewind one step
    b.seq_lens.sub_(1)
    b.tok.fill_(7)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            out = b.decode_step()
    torch.cuda.current_stream().wait_stream(s)
    replay = []
    for _ in range(3):
        g.replay()
        replay.append(out.clone())
    for e, r in zip(eager, replay):
        assert torch.equal(e, r)
    assert torch.equal(a.tok, b.tok) and torch.equal(a.seq_lens, b.seq_lens)


# ---------------------------------------------------------------------------
# page-aware candidates (the model's image_bucket_constraint): token ids lay
# out pages of [marker] + image tokens followed by text
# ---------------------------------------------------------------------------
IMG, PG, PER = 900, 901, 41
PAGE_CFG = dict(image_token_id=IMG, page_token_id=PG, per_page_image_tokens=PER)


def doc_ids(S, n_pages, seed, per=PER):
    """n_pages pages of ``per`` tokens (marker + image tokens), text after,
    with one response-page marker 20 tokens into the text."""
    ids = torch.randint(0, 800, (2, S), generator=torch.Generator().manual_seed(seed))
    for p in range(n_pages):
        ids[:, p * per] = PG
        ids[:, p * per + 1:(p + 1) * per] = IMG
    ids[:, n_pages * per + 20] = PG
    return ids.cuda()


def make_paged(seed=3, max_len=420):
    return DashDecoder(CFG, batch=2, max_len=max_len, device=torch.device("cuda"), seed=seed,
                       page_cfg=PAGE_CFG)


def test_page_aware_prefill_plus_decode_equals_longer_prefill(cfg):
    S = 333
    ids = doc_ids(S + 1, 6, 4)
    full = make_paged()
    # the decode step numbers its text page as a response page: the longer
    # prefill marks its last token as generated to match
    ref = full.prefill(full.embed[ids], token_ids=ids,
                       gen_start=torch.full((2,), S, dtype=torch.int64, device="cuda"))
    part = make_paged()
    part.prefill(part.embed[ids[:, :S]], token_ids=ids[:, :S])
    part.tok.copy_(ids[:, S])
    got = part.decode_step()
    assert torch.isfinite(got).all() and torch.isfinite(ref).all()
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 0.02 * ref.float().abs().max().item(), err
    # the page state after prefill + decode equals the state of the longer prefill
    for a, b in zip(part.pst._slots, full.pst._slots):
        assert torch.equal(a, b)
    assert torch.equal(part.pst._blk_lo, full.pst._blk_lo)
    assert torch.equal(part.pst._blk_hi, full.pst._blk_hi)


def test_page_domain_equals_reference_allow_mask(cfg):
    """The compact page domain routes exactly as the reference's dense allow
    masks (``build_query_allow`` in prefill, ``decode_allow_fused`` in decode)
    through the whole model: equal routes, equal logits; and the page-aware
    routes differ from the unconstrained ones.  Pages of 200 tokens span
    blocks outside the 2-block local window, and a query has more remote
    blocks than K, so the page restriction changes what is routed."""
    S = 1000
    ids = doc_ids(S, 4, 5, per=200)
    dom, ref = make_paged(max_len=1100), make_paged(max_len=1100)
    dense = DashDecoder(CFG, batch=2, max_len=1100, device=torch.device("cuda"), seed=3)
    dom.page_mask, ref.page_mask = False, True
    a = dom.prefill(dom.embed[ids], token_ids=ids)
    b = ref.prefill(ref.embed[ids], token_ids=ids)
    dense.prefill(dense.embed[ids])
    assert torch.equal(dom.last_route[0], ref.last_route[0])
    assert torch.equal(dom.last_route[1], ref.last_route[1])
    assert torch.equal(a, b)
    assert not torch.equal(dom.last_route[0], dense.last_route[0])
    for d in (dom, ref):
        d.tok.fill_(IMG)
    for _ in range(3):
        assert torch.equal(dom.decode_step(), ref.decode_step())
        assert torch.equal(dom.oi, ref.oi) and torch.equal(dom.ob, ref.ob)


# ---------------------------------------------------------------------------
# one layer of the decoder against the CPU oracle: the k-bar rows of the page
# cache, the routed lists (bit-exact) and the attention output, in prefill and
# in the decode step that follows
# ---------------------------------------------------------------------------
def _capture(monkeypatch):
    """Record the last call's inputs / outputs of the routing and attention
    functions the decoder calls (module attributes, restored after the test)."""
    import ananta_ocr_b200.e2e_decoder as E
    rec = {}

    def wrap(mod, name, keys):
        orig = getattr(mod, name)

        def f(*args, **kw):
            r = orig(*args, **kw)
            rec[name] = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in kw.items() if k in keys}
            rec[name]["args"] = [a.clone() if torch.is_tensor(a) else a for a in args]
            return r
        monkeypatch.setattr(mod, name, f)

    wrap(E.RT, "route_prefill_triton", ("idx_q", "out_idx", "out_bias"))
    wrap(E.RT, "route_decode_triton", ("idx_q", "out_idx", "out_bias", "seq_lens"))
    wrap(E.AT, "dash_sparse_attn", ())
    wrap(E.AT, "dash_sparse_attn_decode", ())
    return rec


def _oracle_layer(d, li, idx_q, pos, req, seq_lens):
    """k-bar rows of every page in use, routes and bias of the given rows."""
    import numpy as np
    from oracle import dash_oracle as O
    c = d.cfg
    bs = c.block_size
    bt = d.block_table.cpu().numpy()
    sl = seq_lens.cpu().numpy()
    pages, ntok = [], []
    for r in range(bt.shape[0]):
        for b in range(-(-int(sl[r]) // bs)):
            pages.append(bt[r, b])
            ntok.append(min(bs, int(sl[r]) - b * bs))
    kbar = np.zeros((d.num_pages, c.index_dim), np.float32)
    O.kbar_paged(d.ic[li].cpu().numpy(), np.array(pages), np.array(ntok),
                 d.layers[li]["head_cls"].cpu().numpy(), kbar)
    sc = O.scores_paged(idx_q.cpu().numpy(), pos, req, sl, kbar, bt, bs, c.local_blocks, d.pps)
    oi, ob, _ = O.route_select(sc, None, d.idx_scale, c.topm, c.K, c.prior_floor, c.sigma)
    return np.array(pages), kbar, oi, ob


def test_layer_vs_oracle_prefill_and_decode(cfg, monkeypatch):
    import numpy as np
    from oracle import dash_oracle as O
    from dash_testutil import assert_close_bf16
    rec = _capture(monkeypatch)
    S, B = 301, 2
    c = CFG
    d = make(11)
    ids = torch.randint(0, c.vocab, (B, S + 1), generator=torch.Generator().manual_seed(2)).cuda()
    d.prefill(d.embed[ids[:, :S]])
    li = c.layers - 1                       # every cache below is this layer's, after its call
    K, bs = c.K, c.block_size
    scale = 1.0 / np.sqrt(c.head_dim)
    # ---- prefill ----
    rp = rec["route_prefill_triton"]
    pos = np.tile(np.arange(S), B)
    req = np.repeat(np.arange(B), S)
    pages, kbar, oi, ob = _oracle_layer(d, li, rp["idx_q"], pos, req, d.seq_lens)
    assert np.array_equal(d.kbar[li].cpu().numpy()[pages], kbar[pages]), "prefill k-bar rows"
    gi, gb = rp["out_idx"].cpu().numpy(), rp["out_bias"].cpu().numpy()
    np.testing.assert_array_equal(gi[:, :K], oi)
    assert (gi[:, K:] == -1).all()
    np.testing.assert_allclose(gb[:, :K], ob, atol=1e-4, rtol=0)
    q = rec["dash_sparse_attn"]["args"][0].float().cpu().numpy()
    out = rec["dash_sparse_attn"]["args"][12].float().cpu().numpy()
    kc, vc = d.kc[li].float().cpu().numpy(), d.vc[li].float().cpu().numpy()
    bt = d.block_table.cpu().numpy()
    ref = O.attend_paged(q, kc, vc, oi, ob, bt, req, pos, bs, c.local_blocks * bs, scale)
    assert_close_bf16(out, ref)
    # ---- the decode step that follows ----
    d.tok.copy_(ids[:, S])
    d.decode_step()
    rd = rec["route_decode_triton"]
    dpos = np.full(B, S)
    _, kbar2, oi2, ob2 = _oracle_layer(d, li, rd["idx_q"], dpos, np.arange(B), rd["seq_lens"])
    pages2 = bt[:, :-(-(S + 1) // bs)].reshape(-1)
    assert np.array_equal(d.kbar[li].cpu().numpy()[pages2], kbar2[pages2]), "decode k-bar rows"
    gi2, gb2 = rd["out_idx"].cpu().numpy(), rd["out_bias"].cpu().numpy()
    np.testing.assert_array_equal(gi2[:, :K], oi2)
    np.testing.assert_allclose(gb2[:, :K], ob2, atol=1e-4, rtol=0)
    qd = rec["dash_sparse_attn_decode"]["args"][0].float().cpu().numpy()
    outd = rec["dash_sparse_attn_decode"]["args"][9].float().cpu().numpy()
    refd = O.attend_paged(qd, d.kc[li].float().cpu().numpy(), d.vc[li].float().cpu().numpy(), oi2, ob2,
                          bt, np.arange(B), dpos, bs, c.local_blocks * bs, scale)
    assert_close_bf16(outd, refd)
