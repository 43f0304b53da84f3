"""Out-of-range block and page ids: the kernels record the first one in the
device error word, skip that block, and finish the rest of the work.  Each
case is checked against a clean call with the offending slot removed."""
import math

import numpy as np
import pytest
import torch

from ananta_ocr_b200 import _lib as L
from ananta_ocr_b200 import ops
from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn_decode
from dash_testutil import random_routes

pytestmark = pytest.mark.gpu


def test_prefill_out_of_range_block_is_reported_and_dropped():
    rng = np.random.default_rng(11)
    B, H, T, D, bs, lb, K = 1, 2, 700, 128, 64, 4, 4
    q, k, v = ((torch.randn(B, H, T, D, device="cuda") * 0.5).bfloat16() for _ in range(3))
    idx_np, bias_np = random_routes(rng, B, T, K, bs, lb * bs, messy=False)
    nblk = (T + bs - 1) // bs
    t = 650
    clean = torch.from_numpy(idx_np[:, 0]).cuda()
    bias = torch.from_numpy(bias_np[:, 0]).cuda()
    clean[0, t, 0] = -1
    bad = clean.clone()
    bad[0, t, 0] = nblk + 3
    err = ops.DeviceErrorWord("cuda")
    kw = dict(block_size=bs, local_window=lb * bs, scale=1.0 / math.sqrt(D))
    out_bad = ops.gather_attention(q, k, v, bad, bias, device_error=err, **kw)
    out_clean = ops.gather_attention(q, k, v, clean, bias, **kw)
    torch.cuda.synchronize()
    code, _, info = err.read()
    assert code == L.DASH_DEV_BAD_BLOCK and info == nblk + 3
    assert torch.equal(out_bad, out_clean)


def test_router_out_of_range_kbar_page_is_reported_and_skipped():
    torch.manual_seed(3)
    R, W, bs, d, P = 6, 40, 64, 128, 300
    seqs = ops.Seqs(n_seq=R, q_len=1, kv_len=W * bs, max_q_len=1)
    kbar = torch.randn(P, d, device="cuda") * 0.5
    iq = torch.randn(R, d, device="cuda") * 0.5
    bt = torch.randperm(P, device="cuda")[:R * W].view(R, W).to(torch.int32).contiguous()
    kw = dict(width=W, block_size=bs, local_blocks=4, idx_scale=128.0 / math.sqrt(128),
              prior_floor=1e-4, sigma=1.0, topm=8, K=8, idx_q=iq, kbar=kbar)
    ref_idx, ref_bias = ops.route(seqs, block_table=bt, **kw)
    bad_bt = bt.clone()
    victim = int(ref_idx[2, 0])                  # a block row 2 selected
    bad_bt[2, victim] = P + 17
    err = ops.DeviceErrorWord("cuda")
    idx, _ = ops.route(seqs, block_table=bad_bt, device_error=err, **kw)
    torch.cuda.synchronize()
    code, _, info = err.read()
    assert code == L.DASH_DEV_BAD_PAGE and info == P + 17
    assert victim not in idx[2].tolist()
    keep = [r for r in range(R) if r != 2]
    assert torch.equal(idx[keep], ref_idx[keep])


def test_decode_out_of_range_page_is_reported_and_skipped():
    torch.manual_seed(4)
    R, H, D, bs, S, K = 3, 2, 128, 64, 64 * 20, 4
    nb = S // bs
    P = R * nb + 5
    kc = (torch.randn(P, bs, H, D, device="cuda") * 0.5).bfloat16()
    vc = (torch.randn(P, bs, H, D, device="cuda") * 0.5).bfloat16()
    q = torch.randn(R, H, D, device="cuda").bfloat16()
    bt = torch.randperm(P, device="cuda")[:R * nb].view(R, nb).to(torch.int32).contiguous()
    sl = torch.full((R,), S, dtype=torch.int32, device="cuda")
    idx = torch.tensor([[1, 5, 9, 12]] * R, dtype=torch.int32, device="cuda")
    bias = torch.randn(R, K, device="cuda")
    bad_bt = bt.clone()
    bad_bt[1, 5] = P + 40                        # routed block 5 of row 1
    clean_idx = idx.clone()
    clean_idx[1, 1] = -1

    def run(bt_, idx_, err=None):
        out = torch.empty(R, H, D, dtype=torch.bfloat16, device="cuda")
        dash_sparse_attn_decode(q, kc, vc, idx_[None].expand(H, -1, -1), bias[None].expand(H, -1, -1),
                                bt_, sl, H, 1.0 / math.sqrt(D), out, 1, local_blocks=4,
                                sparse_block_size=bs, num_splits=1, device_error=err)
        return out

    err = ops.DeviceErrorWord("cuda")
    out_bad = run(bad_bt, idx, err)
    out_clean = run(bt, clean_idx)
    torch.cuda.synchronize()
    code, _, info = err.read()
    assert code == L.DASH_DEV_BAD_PAGE and info == P + 40
    diff = (out_bad.float() - out_clean.float()).abs()
    assert float(diff.max()) <= 2e-2 and float(diff.mean()) <= 2e-3


def test_bounded_wait_gives_up_and_reports():
    """A kernel waiting on a barrier phase that never completes gives up after
    its limit, records DASH_DEV_TIMEOUT, and the context stays usable."""
    import time
    err = ops.DeviceErrorWord("cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ops.selftest_bounded_wait(err, limit_ms=50.0)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    code, where, _ = err.read()
    assert code == L.DASH_DEV_TIMEOUT and where == 90
    assert 0.04 <= elapsed < 5.0
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 28.0
