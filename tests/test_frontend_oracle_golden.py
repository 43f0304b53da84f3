"""Pin the router front-end restatement (oracle/frontend_oracle.py) to the
reference's own outputs (tests/golden/frontend.npz: the reference's
``_router_qk`` and the sglang index branch, bf16 on CPU).  CPU only."""
import os

import numpy as np
import torch

from oracle import frontend_oracle as F

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "frontend.npz"))


def bf(name):
    return torch.from_numpy(G[name]).view(torch.bfloat16)


def test_router_qk_matches_reference():
    T, Hd, d = int(G["B"]) * int(G["S"]), int(G["Hd"]), int(G["d"])
    h = bf("hidden").view(T, Hd)
    cos, sin = bf("cos").view(T, d), bf("sin").view(T, d)
    args = (h, bf("wq"), bf("wk"), bf("nq"), bf("nk"), float(G["eps"]))
    q, k = F.router_qk(*args, cos, sin)
    assert np.array_equal(q.numpy(), G["hf_q"].reshape(T, d))
    assert np.array_equal(k.numpy(), G["hf_k"].reshape(T, d))
    q0, k0 = F.router_qk(*args)
    assert np.array_equal(q0.numpy(), G["hf_q_norope"].reshape(T, d))
    assert np.array_equal(k0.numpy(), G["hf_k_norope"].reshape(T, d))


def test_index_branch_matches_reference():
    T, Hd, d = int(G["B"]) * int(G["S"]), int(G["Hd"]), int(G["d"])
    h = bf("hidden").view(T, Hd)
    q, k = F.index_qk(h, bf("wq"), bf("wk"), bf("nq"), bf("nk"), float(G["eps"]),
                      bf("cos").view(T, d), bf("sin").view(T, d))
    assert np.array_equal(q.numpy(), G["sg_q"])
    assert np.array_equal(k.numpy(), G["sg_k"])


def test_rope_rows_match_reference():
    T, d = int(G["B"]) * int(G["S"]), int(G["d"])
    cos, sin = bf("cos").view(T, d), bf("sin").view(T, d)
    for x, o in (("rope_x", "rope_ox"), ("rope_y", "rope_oy")):
        got = F.rope_rows(bf(x), cos, sin, d)
        assert torch.equal(got, bf(o))
