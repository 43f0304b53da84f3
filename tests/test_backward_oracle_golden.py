"""Pin the backward oracle (oracle/backward_oracle.py) to the reference.

tests/golden/backward.npz holds the reference's own training backward
(_E2EGatherAttnFn.backward of sparse_gather_e2e_triton.py, its Triton dq /
d_bias / dk / dv kernels interpreted on the CPU in fp32) and its entmax
Jacobian (dash_attention.py:_Entmax15), made by tests/golden/make_golden.py
(``backward_case``).  CPU only."""
import math
import os

import numpy as np
import torch

from oracle import backward_oracle as BO

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "backward.npz"))


def t(name):
    a = G[name]
    if a.dtype == np.uint16:           # bf16 bit patterns of the inputs
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).float()
    return torch.from_numpy(a)


def test_attention_grads_match_reference():
    for c in (0, 1):
        B, HQ, H, T, bs, LW, K = (int(x) for x in G[f"c{c}_cfg"])
        o, lse, dq, dk, dv, db = BO.gather_attention_grads(
            t(f"c{c}_q"), t(f"c{c}_k"), t(f"c{c}_v"), t(f"c{c}_idx"), t(f"c{c}_bias"),
            t(f"c{c}_do"), bs, LW, 1.0 / math.sqrt(128))
        for got, key in ((o, "o"), (lse, "lse"), (dq, "dq"), (dk, "dk"), (dv, "dv"),
                         (db, "dbias")):
            ref = G[f"c{c}_{key}"]
            np.testing.assert_allclose(got.numpy(), ref, rtol=1e-4, atol=2e-5, err_msg=f"c{c} {key}")


def test_kept_slots_drop_window_and_empty_ids():
    """Slots routed to a block with no key below the window carry no gradient."""
    B, HQ, H, T, bs, LW, K = (int(x) for x in G["c0_cfg"])
    idx = t("c0_idx")
    keep = BO.kept_slots(idx, (T + bs - 1) // bs, bs, LW)
    db = G["c0_dbias"]
    assert np.all(db[~keep.numpy()] == 0)
    assert (~keep & (idx >= 0)).any(), "fixture has no window-block slot"


def test_entmax_matches_reference():
    y = BO.entmax15(t("ent_x"))
    np.testing.assert_allclose(y.numpy(), G["ent_y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(y.sum(-1).numpy(), 1.0, rtol=1e-5)
    dx = BO.entmax15_backward(t("ent_y"), t("ent_dy"))
    np.testing.assert_allclose(dx.numpy(), G["ent_dx"], rtol=1e-5, atol=1e-6)


def test_multi_index_head_restatement_reduces_to_the_pinned_one():
    """gather_attention_heads (several index heads, packed sequences, no bias)
    with one index head and no packing equals gather_attention with zero
    biases, which the reference's e2e goldens pin; with two index heads each
    query head follows its own index head's routes."""
    g = torch.Generator().manual_seed(4)
    B, HQ, H, T, bs, LW, K = 1, 4, 2, 200, 64, 64, 3
    q = torch.randn(B, T, HQ, 128, generator=g) * 0.5
    k = torch.randn(B, T, H, 128, generator=g) * 0.5
    v = torch.randn(B, T, H, 128, generator=g) * 0.5
    idx = torch.randint(-1, 4, (B, 2, T, K), generator=g, dtype=torch.int32)
    seg = torch.zeros(B, T, dtype=torch.int32)
    o1, l1 = BO.gather_attention_heads(q, k, v, idx[:, :1], seg, bs, LW, 1.0 / math.sqrt(128))
    o2, l2 = BO.gather_attention(q, k, v, idx[:, 0], torch.zeros(B, T, K), bs, LW, 1.0 / math.sqrt(128))
    torch.testing.assert_close(o1, o2, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(l1, l2, rtol=1e-5, atol=1e-5)
    oh, _ = BO.gather_attention_heads(q, k, v, idx, seg, bs, LW, 1.0 / math.sqrt(128))
    ob, _ = BO.gather_attention(q[:, :, 2:], k[:, :, 1:], v[:, :, 1:], idx[:, 1], torch.zeros(B, T, K),
                                bs, LW, 1.0 / math.sqrt(128))
    torch.testing.assert_close(oh[:, :, 2:], ob, rtol=1e-5, atol=1e-5)
