"""Pin the CPU oracle to the reference's own outputs (CPU only).

The golden files were produced by tests/golden/make_golden.py, which ran the
reference's PyTorch functions (and, on tiny shapes, its Triton kernels under
the Triton interpreter) on the same seeded inputs regenerated here.
"""
import hashlib
import math
import os

import numpy as np
import pytest

from oracle import dash_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def canon(topi, bias, valid):
    """Reference (descending-score, valid mask) -> ascending ids with -1 tail."""
    big = 1 << 30
    ti = np.where(valid, topi, big)
    o = np.argsort(ti, -1, kind="stable")
    ii = np.take_along_axis(ti, o, -1)
    bb = np.take_along_axis(np.where(valid, bias, 0.0), o, -1)
    return np.where(ii == big, -1, ii).astype(np.int32), bb.astype(np.float32)


def near_tie_rows(scores, K):
    """Rows whose K-th and (K+1)-th best remote scores are within 4 ulp."""
    s = np.sort(np.where(scores > -5e8, scores, -np.inf), -1)[..., ::-1]
    if s.shape[-1] <= K:
        return np.zeros(s.shape[:-1], bool)
    a, b = s[..., K - 1], s[..., K]
    with np.errstate(invalid="ignore"):
        gap = np.abs(a - b)
    return np.isfinite(b) & (gap <= 4 * np.spacing(np.abs(a).astype(np.float32)))


PREFILL = ["c1_headcls", "c1_bs32", "small_headcls", "small_indexer"]


def regen_prefill(g):
    q, k, v, iq, ik = O.make_prefill_inputs(
        int(g["seed"]), int(g["B"]), int(g["H"]), int(g["S"]), 128, int(g["n_pages"]),
        int(g["page_tokens"]), float(g["off_std"]))
    assert sha(q, k, v, iq, ik) == str(g["input_sha"]), "input generator drifted"
    return q, k, v, iq, ik


@pytest.mark.parametrize("name", PREFILL)
def test_prefill_scores_match_reference(name):
    g = load(name)
    q, k, v, iq, ik = regen_prefill(g)
    S, bs, lb = int(g["S"]), int(g["bs"]), int(g["lb"])
    pos = np.arange(S)[None]
    if str(g["stage0"]) == "head_cls":
        sc = O.block_scores_headcls(iq, ik, pos, bs, lb, g["head_cls"])
    else:
        sc = O.block_scores_indexer(iq, ik, pos, bs, lb * bs)
    ref = g["scores"]
    assert sc.shape == ref.shape
    masked_o, masked_r = sc < -5e8, ref < -5e8
    np.testing.assert_array_equal(masked_o, masked_r)
    np.testing.assert_allclose(sc[~masked_o], ref[~masked_r], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("name", PREFILL)
def test_select_bit_exact_on_reference_scores(name):
    g = load(name)
    ri, rb = canon(g["topi"], g["bias"], g["valid"])
    K, topm = int(g["K"]), int(g["topm"])
    oi, ob, cnt = O.route_select(g["scores"], None, float(g["idx_scale"]), topm, K,
                                 float(g["floor"]), float(g["sigma"]))
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_allclose(ob, rb, atol=1e-4, rtol=0)
    np.testing.assert_array_equal(cnt, (ri >= 0).sum(-1))


@pytest.mark.parametrize("name", PREFILL)
def test_end_to_end_route_indices(name):
    """Oracle scores -> oracle selection equals the reference except at near-ties."""
    g = load(name)
    q, k, v, iq, ik = regen_prefill(g)
    S, bs, lb, K = int(g["S"]), int(g["bs"]), int(g["lb"]), int(g["K"])
    pos = np.arange(S)[None]
    if str(g["stage0"]) == "head_cls":
        sc = O.block_scores_headcls(iq, ik, pos, bs, lb, g["head_cls"])
    else:
        sc = O.block_scores_indexer(iq, ik, pos, bs, lb * bs)
    oi, _, _ = O.route_select(sc, None, float(g["idx_scale"]), int(g["topm"]), K,
                              float(g["floor"]), float(g["sigma"]))
    ri, _ = canon(g["topi"], g["bias"], g["valid"])
    bad = (oi != ri).any(-1)
    tie = near_tie_rows(g["scores"], K)
    assert not (bad & ~tie).any(), f"{int((bad & ~tie).sum())} non-tie rows differ"


@pytest.mark.parametrize("name", PREFILL)
def test_prefill_attend_matches_reference(name):
    g = load(name)
    q, k, v, iq, ik = regen_prefill(g)
    ri, rb = canon(g["topi"], g["bias"], g["valid"])
    bs, lb = int(g["bs"]), int(g["lb"])
    out = O.attend_contig(q, k, v, ri, rb, bs, lb * bs, 1.0 / math.sqrt(128), rows=g["rows"])
    np.testing.assert_allclose(out, g["out_rows"], atol=2e-5, rtol=0)


def test_decode_route_and_attend():
    g = load("decode_small")
    B, H, S, bs, lb, K = (int(g[x]) for x in ("B", "H", "S", "bs", "lb", "K"))
    q, k, v, iq, ik = O.make_prefill_inputs(int(g["seed"]), B, H, S, 128, 0, 273, 0.0)
    assert sha(q, k, v, iq, ik, g["qd"], g["iqd"]) == str(g["input_sha"])
    pos = np.full((B, 1), S - 1)
    sc = O.block_scores_headcls(g["iqd"], ik, pos, bs, lb, np.zeros(128, np.float32))
    np.testing.assert_allclose(sc, g["scores"], rtol=2e-5, atol=2e-5)
    oi, ob, _ = O.route_select(g["scores"], None, float(g["idx_scale"]), int(g["topm"]), K,
                               float(g["floor"]), float(g["sigma"]))
    ri, rb = canon(g["topi"], g["bias"], g["valid"])
    np.testing.assert_array_equal(oi, ri)
    np.testing.assert_allclose(ob, rb, atol=1e-4)
    # decode attend: the query sits at position S-1 of a contiguous cache
    out = O.attend_contig(np.broadcast_to(g["qd"], (B, H, S, 128)), k, v,
                          np.broadcast_to(ri[:, :1], (B, S, K)),
                          np.broadcast_to(rb[:, :1], (B, S, K)), bs, lb * bs,
                          1.0 / math.sqrt(128), rows=[S - 1])
    np.testing.assert_allclose(out, g["out"], atol=2e-5)


def test_paged_router_matches_sglang_torch_path():
    g = load("paged_router")
    d, bs, lb = int(g["d"]), int(g["bs"]), int(g["lb"])
    seq_lens, ctx, cu = g["seq_lens"], g["ctx_lens"], g["cu"]
    bt = g["block_table"]
    R, W = bt.shape
    kbar = np.zeros_like(g["kbar"])
    pages, ntok = [], []
    for r in range(R):
        nb = -(-int(seq_lens[r]) // bs)
        for b in range(nb):
            pages.append(bt[r, b])
            ntok.append(min(bs, int(seq_lens[r]) - b * bs))
    O.kbar_paged(g["cache"], np.array(pages), np.array(ntok), g["head_cls"], kbar)
    np.testing.assert_allclose(kbar, g["kbar"], rtol=1e-5, atol=1e-6)
    # prefill rows
    row_req = np.repeat(np.arange(R), np.diff(cu))
    row_pos = np.concatenate([np.arange(ctx[r], seq_lens[r]) for r in range(R)])
    sc = O.scores_paged(g["idx_q"], row_pos, row_req, seq_lens, kbar, bt, bs, lb, W)
    np.testing.assert_allclose(sc, g["scores_prefill"], rtol=2e-5, atol=2e-5)
    budget, topm, slots = int(g["budget"]), int(g["topm"]), int(g["out_slots"])
    oi, ob, _ = O.route_select(g["scores_prefill"], None, float(g["idx_scale"]), topm, budget,
                               1e-4, 1.0)
    ref_i = g["idx_prefill"][:, :slots]
    ri, rb = canon(ref_i, g["bias_prefill"][:, :slots], ref_i >= 0)
    np.testing.assert_array_equal(oi, ri[:, :budget])
    np.testing.assert_allclose(ob, rb[:, :budget], atol=1e-4)
    # decode rows (query at seq_len - 1)
    scd = O.scores_paged(g["iq_dec"], seq_lens - 1, np.arange(R), seq_lens, kbar, bt, bs, lb, W)
    np.testing.assert_allclose(scd, g["scores_decode"], rtol=2e-5, atol=2e-5)
    oi, ob, _ = O.route_select(g["scores_decode"], None, float(g["idx_scale"]), topm, budget,
                               1e-4, 1.0)
    ref_i = g["idx_decode"][:, :slots]
    ri, rb = canon(ref_i, g["bias_decode"][:, :slots], ref_i >= 0)
    np.testing.assert_array_equal(oi, ri[:, :budget])
    np.testing.assert_allclose(ob, rb[:, :budget], atol=1e-4)


@pytest.mark.parametrize("name", ["triton_interp", "triton_interp_bs32"])
def test_triton_kernels_semantics(name):
    """The reference Triton kernels (interpreted) and the oracle agree."""
    g = load(name)
    q, k, v, idx, bias = g["q"], g["k"], g["v"], g["idx"], g["bias"]
    bs, lb = int(g["bs"]), int(g["lb"])
    scale = 1.0 / math.sqrt(128)
    out = O.attend_contig(q, k, v, idx, bias, bs, lb * bs, scale)
    np.testing.assert_allclose(out, g["out_e2e"], atol=1e-4)
    T, H = q.shape[2], q.shape[1]
    qp = q[0].transpose(1, 0, 2)
    kc = np.zeros((g["block_table"].max() + 1, bs, H, 128), np.float32)
    vc = np.zeros_like(kc)
    for b, p in enumerate(g["block_table"][0]):
        kc[p] = k[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
        vc[p] = v[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
    outp = O.attend_paged(qp, kc, vc, idx[0], bias[0], g["block_table"], np.zeros(T, np.int64),
                          np.arange(T), bs, lb * bs, scale)
    np.testing.assert_allclose(outp, g["out_paged"], atol=1e-4)
    np.testing.assert_allclose(outp[-1:], g["out_decode"], atol=1e-4)


def test_det_expf_accuracy():
    xs = np.linspace(-80, 0, 20001).astype(np.float32)
    got = np.array([O.det_expf(float(x)) for x in xs[::50]], np.float64)
    ref = np.exp(xs[::50].astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 3e-7
