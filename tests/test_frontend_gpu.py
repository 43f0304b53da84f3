"""Router front end on the GPU (``dash_index_proj``: tcgen05 GEMM + RMSNorm +
RoPE epilogue) against the reference's outputs (tests/golden/frontend.npz) and
against the torch restatement (oracle/frontend_oracle.py, pinned to the same
goldens) on larger shapes.

Tolerance: the kernel and the reference both round the projection to bf16, but
the fp32 accumulation order of the GEMM differs (tcgen05 vs the reference's
GEMM), so an element's bf16 rounding can land one bf16 ulp apart and the norm
and the RoPE carry that through; where the RoPE sum cancels, one ulp of an
operand is many ulps of the small result.  Bar: every output within
max(3 ulp(|ref|), 2 ulp(max |ref| of its row)) of the reference (bf16 ulp =
2^(floor(log2 x) - 7)), at least 90% of them bitwise equal, and equal mean
absolute value to 1e-3 relative."""
import math
import os
import types

import numpy as np
import pytest
import torch

from oracle import frontend_oracle as F
from ananta_ocr_b200 import ops
from ananta_ocr_b200 import modeling_deepseekv2 as MD
from ananta_ocr_b200.unlimited_dash_ops.index_frontend import index_qk_fused

pytestmark = pytest.mark.gpu
G = None


def golden():
    global G
    if G is None:
        G = np.load(os.path.join(os.path.dirname(__file__), "golden", "frontend.npz"))
    return G


def bf(name):
    return torch.from_numpy(golden()[name]).view(torch.bfloat16).cuda()


def ulp_bf16(x):
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(x), 1e-3))) - 7)


def check(got, ref):
    d = np.asarray(ref).shape[-1]
    got = np.asarray(got, np.float64).reshape(-1, d)
    ref = np.asarray(ref, np.float64).reshape(-1, d)
    tol = np.maximum(3 * ulp_bf16(ref), 2 * ulp_bf16(np.abs(ref).max(-1, keepdims=True)))
    err = np.abs(got - ref)
    assert np.all(err <= tol + 1e-7), f"max err {err.max()} (vs tol {np.max(err / tol):.2f}x)"
    eq = np.mean(got == ref)
    assert eq >= 0.90, f"only {eq:.3f} bitwise equal"
    assert abs(np.mean(np.abs(got)) - np.mean(np.abs(ref))) <= 1e-3 * np.mean(np.abs(ref))


def rand_inputs(seed, T, Hd, d=128, rope=True, dev="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    h = torch.randn(T, Hd, generator=g).to(torch.bfloat16)
    wq = (torch.randn(d, Hd, generator=g) / math.sqrt(Hd)).to(torch.bfloat16)
    wk = (torch.randn(d, Hd, generator=g) / math.sqrt(Hd)).to(torch.bfloat16)
    nq = (torch.randn(d, generator=g) * 0.1).to(torch.bfloat16)
    nk = (torch.randn(d, generator=g) * 0.1).to(torch.bfloat16)
    cos = sin = None
    if rope:
        pos = torch.randint(0, 30000, (T, 1), generator=g).float()
        inv = 1.0 / (10000.0 ** (torch.arange(0, d // 2).float() / (d // 2)))
        emb = torch.cat([pos * inv, pos * inv], -1)
        cos, sin = emb.cos().to(torch.bfloat16).to(dev), emb.sin().to(torch.bfloat16).to(dev)
    return [t.to(dev) for t in (h, wq, wk, nq, nk)] + [cos, sin]


@pytest.mark.parametrize("rope", [True, False])
def test_router_qk_matches_reference_golden(rope):
    g = golden()
    B, S, Hd, d = int(g["B"]), int(g["S"]), int(g["Hd"]), int(g["d"])
    router = types.SimpleNamespace(
        index_dim=d, q_proj=types.SimpleNamespace(weight=bf("wq")),
        k_proj=types.SimpleNamespace(weight=bf("wk")),
        q_norm=types.SimpleNamespace(weight=bf("nq"), eps=float(g["eps"])),
        k_norm=types.SimpleNamespace(weight=bf("nk"), eps=float(g["eps"])))
    pe = (bf("cos"), bf("sin")) if rope else None
    q, k = MD._router_qk(router, bf("hidden"), pe)
    assert q.shape == (B, S, d) and q.dtype == torch.float32
    check(q.cpu().numpy(), g["hf_q"] if rope else g["hf_q_norope"])
    check(k.cpu().numpy(), g["hf_k"] if rope else g["hf_k_norope"])


def test_index_branch_matches_reference_golden():
    g = golden()
    T, Hd, d = int(g["B"]) * int(g["S"]), int(g["Hd"]), int(g["d"])
    q, k = index_qk_fused(bf("hidden").view(T, Hd), bf("wq"), bf("wk"), bf("nq"), bf("nk"),
                          float(g["eps"]), bf("cos").view(T, d), bf("sin").view(T, d))
    check(q.cpu().numpy(), g["sg_q"])
    check(k.cpu().numpy(), g["sg_k"])


@pytest.mark.parametrize("T,Hd", [(1, 64), (128, 1280), (1000, 1280), (4099, 640)])
@pytest.mark.parametrize("clamp", [True, False])
def test_index_proj_matches_torch_restatement(T, Hd, clamp):
    h, wq, wk, nq, nk, cos, sin = rand_inputs(T + Hd, T, Hd)
    q, k = ops.index_proj(h, wq, wk, nq, nk, 1e-6, cos=cos, sin=sin, norm_clamp=clamp)
    ref = (F.router_qk if clamp else F.index_qk)(h, wq, wk, nq, nk, 1e-6, cos, sin)
    check(q.cpu().numpy(), ref[0].cpu().numpy())
    check(k.cpu().numpy(), ref[1].cpu().numpy())


@pytest.mark.parametrize("kdtype", [torch.float32, torch.bfloat16])
def test_index_k_written_into_paged_cache(kdtype):
    T, Hd, P, bs = 700, 1280, 64, 16
    h, wq, wk, nq, nk, cos, sin = rand_inputs(5, T, Hd)
    cache = torch.full((P, bs, 128), 7.0, dtype=kdtype, device="cuda")
    slots = torch.randperm(P * bs, device="cuda")[:T]
    q, c = index_qk_fused(h, wq, wk, nq, nk, 1e-6, cos, sin, index_cache=cache, slot_mapping=slots)
    assert c is cache
    rq, rk = F.index_qk(h, wq, wk, nq, nk, 1e-6, cos, sin)
    rows = cache.view(-1, 128)
    check(rows[slots].float().cpu().numpy(), rk.to(kdtype).float().cpu().numpy())
    check(q.cpu().numpy(), rq.cpu().numpy())
    untouched = torch.ones(P * bs, dtype=torch.bool, device="cuda")
    untouched[slots] = False
    assert torch.all(rows[untouched] == 7.0)


def test_bad_slot_is_recorded_and_skipped():
    T, Hd, P, bs = 300, 256, 32, 16
    h, wq, wk, nq, nk, cos, sin = rand_inputs(6, T, Hd)
    cache = torch.zeros(P * bs, 128, device="cuda")
    slots = torch.arange(T, device="cuda")
    slots[17] = P * bs + 5
    err = ops.DeviceErrorWord("cuda")
    q, _ = ops.index_proj(h, wq, wk, nq, nk, 1e-6, cos=cos, sin=sin, idx_k=cache,
                          slot_mapping=slots, device_error=err)
    code, where, info = err.read()
    assert code == 3 and where == 74 and info == P * bs + 5
    rq, rk = F.index_qk(h, wq, wk, nq, nk, 1e-6, cos, sin)
    keep = torch.ones(T, dtype=torch.bool, device="cuda")
    keep[17] = False
    check(cache[slots[keep]].cpu().numpy(), rk[keep].cpu().numpy())
    check(q.cpu().numpy(), rq.cpu().numpy())


# ---------------------------------------------------------------------------
# main-branch RoPE + paged K/V store: bf16 products and sums, bit-exact
# ---------------------------------------------------------------------------
from ananta_ocr_b200.unlimited_dash_ops import index_frontend as IF  # noqa: E402


def test_rope_pair_matches_reference_golden_bitwise():
    g = golden()
    T, d = int(g["B"]) * int(g["S"]), int(g["d"])
    cos, sin = bf("cos").view(T, d), bf("sin").view(T, d)
    ox, oy = IF.apply_page2d_rope_pair(bf("rope_x"), bf("rope_y"), cos, sin, d)
    assert torch.equal(ox, bf("rope_ox")) and torch.equal(oy, bf("rope_oy"))
    assert torch.equal(IF.apply_page2d_rope(bf("rope_x"), cos, sin, d), bf("rope_ox"))


@pytest.mark.parametrize("Hq,Hkv", [(10, 10), (16, 2)])
def test_rope_and_store_kv_bitwise(Hq, Hkv):
    T, D, P, bs = 777, 128, 128, 16
    gen = torch.Generator(device="cpu").manual_seed(Hq * 31 + Hkv)
    q = torch.randn(T, Hq * D, generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn(T, Hkv * D, generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn(T, Hkv * D, generator=gen).to(torch.bfloat16).cuda()
    pos = torch.randint(0, 20000, (T, 1), generator=gen).float()
    inv = 1.0 / (10000.0 ** (torch.arange(0, D // 2).float() / (D // 2)))
    emb = torch.cat([pos * inv, pos * inv], -1)
    cos, sin = emb.cos().to(torch.bfloat16).cuda(), emb.sin().to(torch.bfloat16).cuda()
    k_cache = torch.full((P, bs, Hkv, D), 3.0, dtype=torch.bfloat16, device="cuda")
    v_cache = torch.full_like(k_cache, 5.0)
    slots = torch.randperm(P * bs, device="cuda")[:T]
    rq = F.rope_rows(q, cos, sin, D)
    rk = F.rope_rows(k, cos, sin, D)
    q2 = q.clone()
    IF.rope_and_store_kv(q2, k, v, cos, sin, k_cache, v_cache, slots, D)
    assert torch.equal(q2, rq)
    kc = k_cache.view(P * bs, Hkv * D)
    vc = v_cache.view(P * bs, Hkv * D)
    assert torch.equal(kc[slots], rk) and torch.equal(vc[slots], v)
    untouched = torch.ones(P * bs, dtype=torch.bool, device="cuda")
    untouched[slots] = False
    assert torch.all(kc[untouched] == 3.0) and torch.all(vc[untouched] == 5.0)


@pytest.mark.parametrize("kdtype,bs,R", [(torch.float32, 32, 300), (torch.bfloat16, 64, 40)])
def test_fused_kbar_refresh_equals_separate_refresh(kdtype, bs, R):
    """A decode step's index-K write with the k-bar refresh of each token's
    tail page in the same kernel gives k-bar rows bitwise equal to the separate
    dash_kbar_pool launch (and to the oracle)."""
    from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
    from oracle import dash_oracle as O
    Hd, W = 1280, 40
    P = R * W
    h, wq, wk, nq, nk, cos, sin = rand_inputs(9, R, Hd)
    g = torch.Generator(device="cuda").manual_seed(2)
    cache = (torch.randn(P, bs, 128, generator=g, device="cuda") * 0.5).to(kdtype)
    bt = torch.randperm(P, generator=g, device="cuda").to(torch.int32).view(R, W)
    seq = torch.randint(1, W * bs, (R,), generator=g, device="cuda").to(torch.int32)   # incl. this token
    pos = seq.long() - 1
    slots = bt.long().gather(1, (pos // bs)[:, None])[:, 0] * bs + pos % bs
    hc = torch.randn(128, generator=g, device="cuda") * 0.3
    plan = RT.kbar_tail_plan(block_table=bt, seq_lens=seq, block_size=bs, tail_pages=1, device="cuda")
    k_fused = torch.full((P, 128), 3.0, device="cuda")
    k_sep = k_fused.clone()
    c1 = cache.clone()
    index_qk_fused(h, wq, wk, nq, nk, 1e-6, cos, sin, index_cache=c1, slot_mapping=slots,
                   kbar_refresh=(k_fused, plan, hc, bs))
    c2 = cache.clone()
    index_qk_fused(h, wq, wk, nq, nk, 1e-6, cos, sin, index_cache=c2, slot_mapping=slots)
    RT.kbar_refresh_tail_triton(kv_cache=c2, k_bar=k_sep, block_table=bt, seq_lens=seq, head_cls=hc,
                                block_size=bs, plan=plan)
    assert torch.equal(c1, c2)
    assert torch.equal(k_fused, k_sep)
    pages, ntok = (t.cpu().numpy() for t in plan)
    ref = np.full((P, 128), 3.0, np.float32)
    O.kbar_paged(c2.float().cpu().numpy(), pages, ntok, hc.cpu().numpy(), ref)
    assert np.array_equal(k_fused.cpu().numpy(), ref)
