"""The DashAttention drop-in (ananta_ocr_b200/dash_attention.py) against the
reference's own DashAttention.forward and its autograd backward (run on the
CPU by tests/golden/make_golden.py), on the checkpoint's block size 32, a
4-block window and K = 12, stage 0 head_cls and indexer, with and without a
per-query candidate domain.

Rows are compared where the selected set is defined: the reference takes
``topk`` of the masked entmax prior, so when a row has more zero-prior
candidates than slots left after its non-zero-prior blocks, which zero-prior
blocks it reads is torch.topk's tie order; the library ranks by score.  The
module-default scale (2.0) gives smooth priors and every row defined for the
head_cls variants, whose gradients are compared too."""
import os
import sys
import types

import numpy as np
import pytest
import torch


sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from golden_inputs import dash_attention_inputs, sha  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
VARIANTS = ["head_cls_0_2", "head_cls_1_2", "indexer_0_2", "head_cls_0_128"]


def _setup(tag, monkeypatch):
    from ananta_ocr_b200.dash_attention import DashAttention
    g = np.load(os.path.join(GOLD, "dash_attention.npz"))
    B, S, hidden, H, D = 1, 600, 256, 2, 128
    w, x = dash_attention_inputs(12, B, S, hidden, H, D, n_pages=3, page_tokens=150)
    assert sha(*w.values(), *x.values()) == str(g["input_sha"])
    stage0, use_cand, scale = tag.rsplit("_", 2)
    monkeypatch.setenv("DASH_STAGE0", stage0)
    sp = dict(sparse_block_size=32, sparse_local_block=4, dash_scaling_factor=float(scale),
              dash_prior_floor=1e-2, sparse_topk_blocks=16, sparse_index_dim=128, dash_sigma=1.0)
    cfg = types.SimpleNamespace(num_attention_heads=H, hidden_size=hidden, rms_norm_eps=1e-6,
                                sparse_attention_config=sp)
    m = DashAttention(cfg).cuda()
    m.k = 12
    with torch.no_grad():
        for n, t in w.items():
            (m.head_cls if n == "head_cls" else getattr(m, n).weight).copy_(torch.from_numpy(t))
    nblk = -(-S // 32)
    cand = np.unpackbits(g["cand"], axis=-1)[..., :nblk].astype(bool) if use_cand == "1" else None
    t = {k: torch.from_numpy(v).cuda() for k, v in x.items()}
    return g, m, t, None if cand is None else torch.from_numpy(cand).cuda(), nblk


def _defined_rows(g, tag, nblk):
    """Rows whose selected set does not depend on the order of equal priors."""
    pr, ti, v = g["prior_" + tag][0], g["topi_" + tag][0].astype(np.int64), g["valid_" + tag][0]
    cand = np.unpackbits(g["candm_" + tag][0], axis=-1)[:, :nblk].astype(bool)
    picked0 = ((np.take_along_axis(pr, ti, -1) == 0) & v).sum(-1)
    zero_cand = (cand & (pr == 0)).sum(-1)
    return np.nonzero((picked0 == 0) | (picked0 == zero_cand))[0]


@pytest.mark.parametrize("tag", VARIANTS)
def test_forward_matches_reference(tag, monkeypatch):
    g, m, t, cand, nblk = _setup(tag, monkeypatch)
    with torch.no_grad():
        out = m(t["hidden"], t["q"], t["k"], t["v"], position_embeddings=(t["cos"], t["sin"]),
                block_cand=cand)
    rows = g["rows"]
    ok = np.isin(rows, _defined_rows(g, tag, nblk))
    assert ok.sum() >= 16
    # fp32 inputs: the router and the attention compute in fp32
    assert out.dtype == torch.float32
    np.testing.assert_allclose(out.cpu().numpy()[:, :, rows[ok]], g["out_" + tag][:, :, ok],
                               atol=2e-4, rtol=0)


@pytest.mark.parametrize("tag", ["head_cls_0_2", "head_cls_1_2"])
def test_training_forward_backward_matches_reference(tag, monkeypatch):
    g, m, t, cand, nblk = _setup(tag, monkeypatch)
    assert len(_defined_rows(g, tag, nblk)) == 600
    q, k, v = (t[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    hs = t["hidden"].clone().requires_grad_(True)
    out = m(hs, q, k, v, position_embeddings=(t["cos"], t["sin"]), block_cand=cand)
    (out.float() * t["dout"]).sum().backward()
    rows = g["rows"]
    np.testing.assert_allclose(out.detach().cpu().numpy()[:, :, rows], g["out_" + tag],
                               atol=2e-4, rtol=0)

    def rel(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
    # fp32 end to end: gradients within 2e-3 (relative Frobenius) of the
    # reference's fp32 autograd (summation orders differ)
    errs = dict(dq=rel(q.grad.cpu().numpy()[:, :, rows], g["dq_" + tag]),
                dv=rel(v.grad.cpu().numpy()[:, :, rows], g["dv_" + tag]),
                dqproj=rel(m.q_proj.weight.grad.cpu().numpy(), g["dqproj_" + tag]),
                dheadcls=rel(m.head_cls.grad.cpu().numpy(), g["dheadcls_" + tag]))
    assert max(errs.values()) < 2e-3, errs
