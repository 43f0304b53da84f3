"""Training backward on the GPU (``dash_attn_bwd``, ``dash_entmax15_fwd/bwd``).

Pinned to the reference's own backward (tests/golden/backward.npz: the Triton
dq / d_bias / dk / dv kernels interpreted in fp32, and ``_Entmax15``) and, on
larger ragged shapes, to the torch fp32 autograd restatement
(oracle/backward_oracle.py, itself pinned to the same goldens).

Tolerances: fp32 kernel vs fp32 reference: 1e-4 of the tensor's largest
magnitude (summation order only).  bf16 kernel (bf16 inputs and outputs,
fp32 arithmetic; lse and o from the tcgen05 forward) vs fp32 reference:
every element within 2% of the tensor's largest magnitude and a relative
Frobenius error below 1.5%.  Entmax: 1e-5 relative, 1e-6 absolute."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import backward_oracle as BO
from ananta_ocr_b200 import ops
from ananta_ocr_b200 import sparse_gather_e2e_triton as E2E
from ananta_ocr_b200.dash_attention import entmax15

pytestmark = pytest.mark.gpu
G = None


def gold():
    global G
    if G is None:
        G = np.load(os.path.join(os.path.dirname(__file__), "golden", "backward.npz"))
    return G


def gt(name, dtype=torch.float32):
    a = gold()[name]
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dtype).cuda()
    return torch.from_numpy(a).to(dtype).cuda()


def close(got, ref, frac, fro=None):
    got, ref = got.float().cpu(), ref.float().cpu()
    m = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= frac * m + 1e-6, f"max err {err} vs {frac} x {m}"
    if fro is not None:
        r = ((got - ref).norm() / ref.norm().clamp_min(1e-12)).item()
        assert r <= fro, f"relative error {r}"


@pytest.mark.parametrize("c", [0, 1])
def test_fp32_backward_matches_reference_golden(c):
    B, HQ, H, T, bs, LW, K = (int(x) for x in gold()[f"c{c}_cfg"])
    dq, dk, dv, db = ops.gather_attention_bwd(
        gt(f"c{c}_q"), gt(f"c{c}_k"), gt(f"c{c}_v"), gt(f"c{c}_o"), gt(f"c{c}_do"),
        gt(f"c{c}_lse"), gt(f"c{c}_idx", torch.int32), gt(f"c{c}_bias"), block_size=bs,
        local_window=LW, scale=1.0 / math.sqrt(128))
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv"), (db, "dbias")):
        close(got, gt(f"c{c}_{key}"), 1e-4)


@pytest.mark.parametrize("c", [0, 1])
def test_bf16_backward_matches_reference_golden(c):
    B, HQ, H, T, bs, LW, K = (int(x) for x in gold()[f"c{c}_cfg"])
    bf = torch.bfloat16
    dq, dk, dv, db = ops.gather_attention_bwd(
        gt(f"c{c}_q", bf), gt(f"c{c}_k", bf), gt(f"c{c}_v", bf), gt(f"c{c}_o", bf),
        gt(f"c{c}_do", bf), gt(f"c{c}_lse"), gt(f"c{c}_idx", torch.int32), gt(f"c{c}_bias"),
        block_size=bs, local_window=LW, scale=1.0 / math.sqrt(128))
    assert dq.dtype == bf and dk.dtype == bf and db.dtype == torch.float32
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv"), (db, "dbias")):
        close(got, gt(f"c{c}_{key}"), 0.02, 0.015)


def routes(B, T, K, bs, LW, seed, dup=True):
    g = torch.Generator().manual_seed(seed)
    nblk = (T + bs - 1) // bs
    idx = torch.full((B, T, K), -1, dtype=torch.int32)
    for t in range(T):
        hi = t // bs + 1
        n = int(torch.randint(0, K + 1, (1,), generator=g))
        if n:
            idx[:, t, :n] = torch.randint(0, hi, (B, n), generator=g, dtype=torch.int32)
    if dup:
        idx[:, -7:, 1] = idx[:, -7:, 0]          # duplicate ids: the later slot is ignored
    idx[0, 5, 0] = nblk + 3                       # out of range: ignored
    bias = torch.randn(B, T, K, generator=g) * 0.5
    return idx.cuda(), bias.cuda()


@pytest.mark.parametrize("B,HQ,H,T,bs,LW,K", [(2, 8, 2, 1000, 128, 256, 6),
                                               (1, 2, 2, 777, 64, 256, 16),
                                               (1, 8, 1, 300, 64, 64, 3),
                                               # 32-token blocks: four per 128-key tile
                                               (1, 2, 2, 700, 32, 128, 12),
                                               # a window that ends inside a block
                                               (2, 4, 2, 500, 32, 96, 8),
                                               (1, 2, 2, 600, 64, 96, 5)])
def test_bf16_forward_backward_matches_oracle(B, HQ, H, T, bs, LW, K):
    """Our tcgen05 forward (o, lse) + the backward vs fp32 autograd."""
    g = torch.Generator().manual_seed(T + HQ)
    q = (torch.randn(B, T, HQ, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    k = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    v = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    do = torch.randn(B, T, HQ, 128, generator=g).to(torch.bfloat16).cuda()
    idx, bias = routes(B, T, K, bs, LW, T)
    scale = 1.0 / math.sqrt(128)
    lse = torch.empty(B, HQ, T, device="cuda")
    o = ops.gather_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), idx[:, None],
                             bias[:, None], block_size=bs, local_window=LW, scale=scale, lse=lse)
    o = o.transpose(1, 2).contiguous()
    dq, dk, dv, db = ops.gather_attention_bwd(q, k, v, o, do, lse.transpose(1, 2), idx, bias,
                                              block_size=bs, local_window=LW, scale=scale)
    ro, rlse, rdq, rdk, rdv, rdb = BO.gather_attention_grads(q, k, v, idx, bias, do, bs, LW, scale)
    close(lse.transpose(1, 2), rlse, 1e-3)
    for got, ref in ((dq, rdq), (dk, rdk), (dv, rdv), (db, rdb)):
        close(got, ref, 0.02, 0.015)
    keep = BO.kept_slots(idx, (T + bs - 1) // bs, bs, LW)
    assert torch.all(db[~keep] == 0)


@pytest.mark.parametrize("dt,B,HQ,H,T,bs,LW,K", [
    (torch.float16, 1, 4, 2, 700, 64, 128, 5),     # fp16 tensor-core path
    (torch.bfloat16, 2, 2, 2, 100, 64, 64, 3),     # shorter than one 128-key tile
    (torch.bfloat16, 1, 2, 1, 333, 64, 128, 0),    # no routed slots: local window only
    (torch.bfloat16, 1, 2, 2, 520, 192, 192, 4),   # blocks straddling the 128-key tiles
    (torch.float32, 1, 2, 2, 600, 32, 128, 12),    # fp32 (CUDA cores), 32-token blocks
    (torch.float32, 1, 4, 2, 400, 96, 100, 3),     # fp32, two blocks in a 64-key tile
])
def test_backward_edge_cases_match_oracle(dt, B, HQ, H, T, bs, LW, K):
    g = torch.Generator().manual_seed(T * 7 + K)
    q = (torch.randn(B, T, HQ, 128, generator=g) * 0.5).to(dt).cuda()
    k = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(dt).cuda()
    v = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(dt).cuda()
    do = torch.randn(B, T, HQ, 128, generator=g).to(dt).cuda()
    if K > 0:
        idx, bias = routes(B, T, K, bs, LW, T + 1, dup=False)
    else:
        idx = torch.zeros(B, T, 0, dtype=torch.int32, device="cuda")
        bias = torch.zeros(B, T, 0, device="cuda")
    scale = 1.0 / math.sqrt(128)
    lse = torch.empty(B, HQ, T, device="cuda")
    o = ops.gather_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), idx[:, None],
                             bias[:, None], block_size=bs, local_window=LW, scale=scale, lse=lse)
    o = o.transpose(1, 2).contiguous()
    dq, dk, dv, db = ops.gather_attention_bwd(q, k, v, o, do, lse.transpose(1, 2), idx, bias,
                                              block_size=bs, local_window=LW, scale=scale)
    _, _, rdq, rdk, rdv, rdb = BO.gather_attention_grads(q, k, v, idx, bias, do, bs, LW, scale)
    tol = (1e-4, None) if dt == torch.float32 else (0.02, 0.015)
    for got, ref in ((dq, rdq), (dk, rdk), (dv, rdv)):
        assert got.dtype == dt
        close(got, ref, *tol)
    if K > 0:
        close(db, rdb, *tol)


def test_autograd_mirror_matches_oracle():
    """triton_gather_attention_e2e with requires_grad: gradients of q, k, v and
    the slot biases through the reference-named autograd Function."""
    B, HQ, H, T, bs, LW, K = 1, 4, 2, 640, 64, 128, 5
    g = torch.Generator().manual_seed(3)
    q = (torch.randn(B, HQ, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    k = (torch.randn(B, H, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    v = (torch.randn(B, H, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    idx, bias = routes(B, T, K, bs, LW, 9, dup=False)
    bias.requires_grad_()
    do = torch.randn(B, HQ, T, 128, generator=g).to(torch.bfloat16).cuda()
    pos = torch.arange(T, device="cuda")[None]
    o = E2E.triton_gather_attention_e2e(q, k, v, idx[:, None], bias, pos, None, bs,
                                        1.0 / math.sqrt(128), LW)
    o.backward(do)
    tr = lambda t: t.detach().transpose(1, 2)     # noqa: E731
    ro, _, rdq, rdk, rdv, rdb = BO.gather_attention_grads(tr(q), tr(k), tr(v), idx, bias.detach(),
                                                          tr(do), bs, LW, 1.0 / math.sqrt(128))
    close(o.detach().transpose(1, 2), ro, 0.02, 0.01)
    for got, ref in ((q.grad, rdq), (k.grad, rdk), (v.grad, rdv)):
        close(got.transpose(1, 2), ref, 0.02, 0.015)
    close(bias.grad, rdb, 0.02, 0.015)


def test_entmax_matches_reference_golden():
    x, y_ref = gt("ent_x"), gt("ent_y")
    y = ops.entmax15(x)
    torch.testing.assert_close(y, y_ref, rtol=1e-5, atol=1e-6)
    dx = ops.entmax15_backward(y_ref, gt("ent_dy"))
    torch.testing.assert_close(dx, gt("ent_dx"), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,n", [(513, 1024), (7, 1), (100, 431)])
def test_entmax_autograd_matches_oracle(rows, n):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(rows, n, generator=g) * 4
    x[torch.rand(rows, n, generator=g) < 0.4] = -1e4
    x = x.cuda().requires_grad_()
    dy = torch.randn(rows, n, generator=g).cuda()
    y = entmax15(x, -1)
    y.backward(dy)
    xr = x.detach().clone().requires_grad_()
    yr = BO.entmax15(xr)
    torch.testing.assert_close(y, yr, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(y.sum(-1), torch.ones(rows, device="cuda"), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(x.grad, BO.entmax15_backward(yr.detach(), dy), rtol=1e-5, atol=1e-5)
    # another dim than the last
    y2 = entmax15(x.detach().t().contiguous(), 0)
    torch.testing.assert_close(y2.t(), yr.detach(), rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------------------
# several index heads + packed sequences (sparse_gather_triton's path, no bias)
# ---------------------------------------------------------------------------
from ananta_ocr_b200 import sparse_gather_triton as SG  # noqa: E402
from ananta_ocr_b200 import _lib as L  # noqa: E402


def packed(B, T, seed):
    """position_ids of packed sequences (random segment lengths) and the
    matching segment starts arange(T) - position_ids."""
    g = torch.Generator().manual_seed(seed)
    pos = torch.empty(B, T, dtype=torch.int64)
    for b in range(B):
        t = 0
        while t < T:
            n = int(torch.randint(40, 300, (1,), generator=g))
            pos[b, t:t + n] = torch.arange(min(n, T - t))
            t += n
    return pos.cuda(), (torch.arange(T)[None] - pos.cpu()).to(torch.int32).cuda()


def heads_routes(B, HI, T, K, bs, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.full((B, HI, T, K), -1, dtype=torch.int32)
    for t in range(T):
        n = int(torch.randint(0, K + 1, (1,), generator=g))
        if n:
            idx[:, :, t, :n] = torch.randint(0, t // bs + 1, (B, HI, n), generator=g, dtype=torch.int32)
    return idx.cuda()


@pytest.mark.parametrize("B,HQ,H,HI,T,bs,LW,K", [(2, 8, 4, 2, 600, 64, 128, 5),
                                                  (1, 4, 2, 1, 450, 128, 128, 3),
                                                  # one index head per kv head, a window
                                                  # ending inside a block
                                                  (1, 4, 4, 4, 500, 64, 96, 4),
                                                  (1, 4, 2, 2, 520, 32, 112, 6)])
def test_multi_index_head_packed_backward_matches_oracle(B, HQ, H, HI, T, bs, LW, K):
    g = torch.Generator().manual_seed(T + HI)
    q = (torch.randn(B, T, HQ, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    k = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    v = (torch.randn(B, T, H, 128, generator=g) * 0.5).to(torch.bfloat16).cuda()
    do = torch.randn(B, T, HQ, 128, generator=g).to(torch.bfloat16).cuda()
    _, seg = packed(B, T, T)
    idx = heads_routes(B, HI, T, K, bs, T + 1)
    scale = 1.0 / math.sqrt(128)
    lse = torch.empty(B, HQ, T, device="cuda")
    o = ops.gather_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), idx, None,
                             block_size=bs, local_window=LW, scale=scale, seg_start=seg,
                             n_index_heads=HI, lse=lse)
    o = o.transpose(1, 2).contiguous()
    dq, dk, dv, _ = ops.gather_attention_bwd(q, k, v, o, do, lse.transpose(1, 2), idx, None,
                                             block_size=bs, local_window=LW, scale=scale,
                                             want_d_bias=False, seg_start=seg)
    ro, rlse, rdq, rdk, rdv = BO.gather_attention_heads_grads(q, k, v, idx, seg, do, bs, LW, scale)
    close(o, ro, 0.02, 0.01)
    close(lse.transpose(1, 2), rlse, 1e-3)
    for got, ref in ((dq, rdq), (dk, rdk), (dv, rdv)):
        close(got, ref, 0.02, 0.015)


def test_gather_attention_mirror_gradients_match_oracle():
    """sparse_gather_triton.triton_gather_attention with requires_grad (two
    index heads, packed sequences) through the reference-named autograd
    Function."""
    B, HQ, H, HI, T, bs, LW, K = 1, 4, 2, 2, 520, 64, 128, 4
    g = torch.Generator().manual_seed(11)
    q = (torch.randn(B, HQ, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    k = (torch.randn(B, H, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    v = (torch.randn(B, H, T, 128, generator=g) * 0.5).to(torch.bfloat16).cuda().requires_grad_()
    do = torch.randn(B, HQ, T, 128, generator=g).to(torch.bfloat16).cuda()
    pos, seg = packed(B, T, 5)
    idx = heads_routes(B, HI, T, K, bs, 6)
    o = SG.triton_gather_attention(q, k, v, idx, pos, None, bs, 1.0 / math.sqrt(128), LW)
    o.backward(do)
    tr = lambda t: t.detach().transpose(1, 2)     # noqa: E731
    ro, _, rdq, rdk, rdv = BO.gather_attention_heads_grads(tr(q), tr(k), tr(v), idx, seg, tr(do), bs, LW,
                                                           1.0 / math.sqrt(128))
    close(o.detach().transpose(1, 2), ro, 0.02, 0.01)
    for got, ref in ((q.grad, rdq), (k.grad, rdk), (v.grad, rdv)):
        close(got.transpose(1, 2), ref, 0.02, 0.015)


def test_fp32_with_segments_is_rejected():
    T = 128
    x = torch.zeros(1, T, 2, 128, device="cuda")
    idx = torch.full((1, T, 2), -1, dtype=torch.int32, device="cuda")
    seg = torch.zeros(1, T, dtype=torch.int32, device="cuda")
    with pytest.raises(L.DashError):
        ops.gather_attention_bwd(x, x, x, x, x, torch.zeros(1, T, 2, device="cuda"), idx, None,
                                 block_size=64, local_window=64, scale=0.1, seg_start=seg)


def test_autograd_mirror_fp32_matches_oracle():
    """fp32 inputs through triton_gather_attention_e2e with requires_grad: the
    fp32 forward (CUDA cores) and the fp32 backward keep fp32 precision
    (1e-4 of each tensor's largest magnitude against the fp32 autograd of the
    dense restatement), like the reference's fp32 kernels."""
    B, HQ, H, T, bs, LW, K = 1, 4, 2, 640, 64, 128, 5
    g = torch.Generator().manual_seed(4)
    q = (torch.randn(B, HQ, T, 128, generator=g) * 0.5).cuda().requires_grad_()
    k = (torch.randn(B, H, T, 128, generator=g) * 0.5).cuda().requires_grad_()
    v = (torch.randn(B, H, T, 128, generator=g) * 0.5).cuda().requires_grad_()
    idx, bias = routes(B, T, K, bs, LW, 11, dup=False)
    bias.requires_grad_()
    do = torch.randn(B, HQ, T, 128, generator=g).cuda()
    pos = torch.arange(T, device="cuda")[None]
    o = E2E.triton_gather_attention_e2e(q, k, v, idx[:, None], bias, pos, None, bs,
                                        1.0 / math.sqrt(128), LW)
    assert o.dtype == torch.float32
    o.backward(do)
    tr = lambda t: t.detach().transpose(1, 2)     # noqa: E731
    ro, _, rdq, rdk, rdv, rdb = BO.gather_attention_grads(tr(q), tr(k), tr(v), idx, bias.detach(),
                                                          tr(do), bs, LW, 1.0 / math.sqrt(128))
    close(o.detach().transpose(1, 2), ro, 1e-4)
    for got, ref in ((q.grad, rdq), (k.grad, rdk), (v.grad, rdv)):
        close(got.transpose(1, 2), ref, 1e-4)
    close(bias.grad, rdb, 1e-4)
