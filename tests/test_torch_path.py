"""The torch fp32 restatement of the reference's CPU path (oracle/torch_path.py,
the CPU baseline's arithmetic) against the reference's own outputs."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import dash_oracle as O
from oracle import torch_path as TP

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["c1_headcls", "c1_bs32"])
def test_torch_path_matches_reference_golden(name):
    g = np.load(os.path.join(GOLD, name + ".npz"))
    B, H, S, bs, lb, K, topm = (int(g[x]) for x in ("B", "H", "S", "bs", "lb", "K", "topm"))
    q, k, v, iq, ik = O.make_prefill_inputs(int(g["seed"]), B, H, S, 128, int(g["n_pages"]),
                                            int(g["page_tokens"]), float(g["off_std"]))
    rows = torch.from_numpy(g["rows"])
    out, ids, bias, valid = TP.prefill_rows(
        torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(iq),
        torch.from_numpy(ik), rows, block_size=bs, local_blocks=lb, K=K, topm=topm,
        idx_scale=float(g["idx_scale"]), floor=float(g["floor"]), sigma=float(g["sigma"]),
        head_cls=torch.from_numpy(g["head_cls"]))
    r = g["rows"]
    np.testing.assert_array_equal(np.where(valid.numpy(), ids.numpy(), -1),
                                  np.where(g["valid"][:, r], g["topi"][:, r], -1))
    np.testing.assert_allclose(bias.numpy(), g["bias"][:, r], atol=1e-4)
    np.testing.assert_allclose(out.numpy(), g["out_rows"], atol=2e-5)
