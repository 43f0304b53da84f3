"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout, naming it with
``DASH_REFERENCE`` (no default path); optional arguments name the cases to
regenerate (default: all):

    DASH_REFERENCE=<checkout> python tests/golden/make_golden.py [case ...]

It imports the reference's OWN PyTorch functions and runs them on seeded
inputs built by ``oracle.dash_oracle.make_prefill_inputs`` (numpy PCG64, so the
tests regenerate identical inputs anywhere):

* ``modeling_deepseekv2._block_scores_infer``   (head_cls and indexer stage-0)
* ``modeling_deepseekv2._infer_route_select``   (canonical selection + bias)
* ``dash_attention.DashAttention._forward_dense`` (prefill attend)
* ``modeling_deepseekv2._decode_attend``        (decode attend)
* the sglang wheel's ``dash_stage0.headcls_scores_prefill/decode`` and
  ``dash_router.DashRouterMath.route_and_select`` (paged router, torch path)
* the reference Triton kernels under ``TRITON_INTERPRET=1`` on tiny shapes
  (``triton_gather_attention_e2e``, sglang ``dash_sparse_attn`` and
  ``dash_sparse_attn_decode``).

Outputs are small ``.npz`` files next to this script.  Inputs are not stored;
their sha256 is, so a drifting generator is detected.
"""
from __future__ import annotations

import hashlib
import math
import os
import sys
import tempfile
import types
import zipfile
import glob

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle.dash_oracle import make_prefill_inputs  # noqa: E402
sys.path.insert(0, HERE)
from golden_inputs import dash_attention_inputs  # noqa: E402

REF = os.environ.get("DASH_REFERENCE", "")


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def import_reference():
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set DASH_REFERENCE to the reference checkout")
    import transformers.utils.import_utils as iu
    if not hasattr(iu, "is_torch_fx_available"):
        iu.is_torch_fx_available = lambda: False
    tmp = tempfile.mkdtemp()
    os.symlink(REF, os.path.join(tmp, "ananta_ref"))
    whl = glob.glob(os.path.join(REF, "wheel", "*.whl"))[0]
    z = zipfile.ZipFile(whl)
    pkg = "sglang/srt/layers/attention/unlimited_dash_ops/"
    for n in z.namelist():
        if n.startswith(pkg) and n.endswith(".py"):
            z.extract(n, tmp)
    for p in ["sglang", "sglang/srt", "sglang/srt/layers", "sglang/srt/layers/attention"]:
        open(os.path.join(tmp, p, "__init__.py"), "w").close()
    sys.path.insert(0, tmp)
    # modules the reference imports but this path never uses
    rt = types.ModuleType("sglang.srt.runtime_context")
    rt.get_buffer = lambda key, factory: factory()
    sys.modules["sglang.srt.runtime_context"] = rt

    class _AttrDict(dict):
        __getattr__ = dict.__getitem__
    for mod, attr in (("easydict", "EasyDict"), ("addict", "Dict")):
        m = types.ModuleType(mod)
        setattr(m, attr, _AttrDict)
        sys.modules.setdefault(mod, m)
    import ananta_ref.dash_attention as da
    import ananta_ref.modeling_deepseekv2 as md
    return da, md


def router_stub(stage0, bs, lb, head_cls, q_chunk=2048):
    return types.SimpleNamespace(stage0=stage0, block_size=bs, local_blocks=lb,
                                 local_window=lb * bs, head_cls=torch.tensor(head_cls),
                                 q_chunk=q_chunk)


def prefill_case(da, md, name, seed, B, H, S, bs, lb, K, topm, stage0, hc_std,
                 n_pages, page_tokens, off_std, sample_rows=None):
    D = 128
    q, k, v, iq, ik = make_prefill_inputs(seed, B, H, S, D, n_pages, page_tokens, off_std)
    rng = np.random.default_rng(seed + 1000)
    head_cls = (rng.standard_normal(D) * hc_std).astype(np.float32)
    nblk = (S + bs - 1) // bs
    r = router_stub(stage0, bs, lb, head_cls)
    pos = torch.arange(S)[None].expand(B, -1)
    sc = md._block_scores_infer(r, torch.tensor(iq), torch.tensor(ik), pos, nblk)
    idx_scale = 128.0 / math.sqrt(128)
    p = dict(idx_scale=idx_scale, floor=1e-4, sigma=1.0, K=K, topm=topm)
    topi, bias, valid = md._infer_route_select(sc, None, p)
    stub = types.SimpleNamespace(block_size=bs, q_chunk=512, local_window=lb * bs,
                                 _scale=1.0 / math.sqrt(D))
    out = da.DashAttention._forward_dense(stub, torch.tensor(q), torch.tensor(k),
                                          torch.tensor(v), topi, bias, valid, S, nblk, None)
    out = out.numpy()
    rows = np.arange(S) if sample_rows is None else np.asarray(sample_rows)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        seed=seed, B=B, H=H, S=S, bs=bs, lb=lb, K=K, topm=topm, stage0=stage0,
        hc_std=hc_std, n_pages=n_pages, page_tokens=page_tokens, off_std=off_std,
        head_cls=head_cls, idx_scale=idx_scale, floor=1e-4, sigma=1.0,
        input_sha=sha(q, k, v, iq, ik),
        scores=sc.numpy(), topi=topi.numpy().astype(np.int32), bias=bias.numpy(),
        valid=valid.numpy(), rows=rows, out_rows=out[:, :, rows])
    print(name, "saved", sc.shape, out.shape)


def decode_case(da, md, name, seed, B, H, S, bs, lb, K, topm):
    D = 128
    q, k, v, iq, ik = make_prefill_inputs(seed, B, H, S, D, 0, 273, 0.0)
    rng = np.random.default_rng(seed + 7)
    qd = (rng.standard_normal((B, H, 1, D))).astype(np.float32)
    iqd = (rng.standard_normal((B, 1, 128)) * 0.5).astype(np.float32)
    head_cls = np.zeros(128, np.float32)
    nblk = (S + bs - 1) // bs
    r = router_stub("head_cls", bs, lb, head_cls)
    pos = torch.full((B, 1), S - 1)
    sc = md._block_scores_infer(r, torch.tensor(iqd), torch.tensor(ik), pos, nblk)
    idx_scale = 128.0 / math.sqrt(128)
    p = dict(idx_scale=idx_scale, floor=1e-4, sigma=1.0, K=K, topm=topm)
    topi, bias, valid = md._infer_route_select(sc, None, p)
    out = md._decode_attend(torch.tensor(qd), torch.tensor(k), torch.tensor(v), topi, bias,
                            valid, pos, bs, lb * bs, 1.0 / math.sqrt(D))
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), seed=seed, B=B, H=H, S=S, bs=bs, lb=lb, K=K,
        topm=topm, idx_scale=idx_scale, floor=1e-4, sigma=1.0,
        input_sha=sha(q, k, v, iq, ik, qd, iqd), qd=qd, iqd=iqd, scores=sc.numpy(),
        topi=topi.numpy().astype(np.int32), bias=bias.numpy(), valid=valid.numpy(),
        out=out.numpy())
    print(name, "saved", out.shape)


def paged_router_case(name, seed):
    """sglang torch reference of the paged head_cls router (prefill + decode)."""
    from sglang.srt.layers.attention.unlimited_dash_ops import dash_stage0 as st0
    from sglang.srt.layers.attention.unlimited_dash_ops.dash_router import DashRouterMath
    rng = np.random.default_rng(seed)
    d, bs, lb, R = 128, 16, 2, 3
    seq_lens = np.array([150, 97, 230], np.int64)
    ctx_lens = np.array([40, 0, 100], np.int64)         # prefix already cached
    q_lens = seq_lens - ctx_lens
    W = int(math.ceil(seq_lens.max() / bs))
    P = 64
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((R, W), np.int32)
    n = 0
    for r in range(R):
        nb = int(math.ceil(seq_lens[r] / bs))
        bt[r, :nb] = perm[n:n + nb]
        n += nb
    cache = (rng.standard_normal((P, bs, d)) * 0.5).astype(np.float32)
    head_cls = (rng.standard_normal(d) * 0.7).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int64)
    total_q = int(cu[-1])
    idx_q = (rng.standard_normal((total_q, d)) * 0.5).astype(np.float32)
    kc = st0.KBarCache(P, d, "cpu")
    sc = st0.headcls_scores_prefill(
        idx_q=torch.tensor(idx_q), kv_cache=torch.tensor(cache), block_table=torch.tensor(bt),
        cu_seqlens_q=torch.tensor(cu), seq_lens=torch.tensor(seq_lens),
        context_lens=torch.tensor(ctx_lens), head_cls=torch.tensor(head_cls), max_block=W,
        block_size=bs, local_blocks=lb, cache=kc)
    router = DashRouterMath(index_dim=d, block_size=bs, local_blocks=lb, topk_blocks=8,
                            scaling_factor=128.0, sigma=1.0, prior_floor=1e-4,
                            budget_remote=4, topm=8)
    idx_p, bias_p = router.route_and_select(sc, W)
    # one decode step per request
    iq_dec = (rng.standard_normal((R, d)) * 0.5).astype(np.float32)
    sc_d = st0.headcls_scores_decode(
        idx_q=torch.tensor(iq_dec), cache=kc, block_table=torch.tensor(bt),
        seq_lens=torch.tensor(seq_lens), max_block=W, block_size=bs, local_blocks=lb,
        decode_query_len=1)
    idx_d, bias_d = router.route_and_select(sc_d, W)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), seed=seed, d=d, bs=bs, lb=lb, seq_lens=seq_lens,
        ctx_lens=ctx_lens, cu=cu, block_table=bt, cache=cache, head_cls=head_cls,
        idx_q=idx_q, iq_dec=iq_dec, kbar=kc.k_bar.numpy(), scores_prefill=sc.numpy()[0],
        idx_prefill=idx_p.numpy()[0], bias_prefill=bias_p.numpy()[0],
        scores_decode=sc_d.numpy()[0], idx_decode=idx_d.numpy()[0],
        bias_decode=bias_d.numpy()[0], idx_scale=router.idx_scale, out_slots=router.out_slots,
        budget=router.budget_remote, topm=router.topm)
    print(name, "saved")


def triton_interp_case(da, md, name, seed, T=96, bs=16, lb=2, K=3):
    """Reference Triton kernels, interpreted on CPU, on tiny shapes."""
    import ananta_ref.sparse_gather_e2e_triton as e2e
    from sglang.srt.layers.attention.unlimited_dash_ops import attend_triton as at
    # the decode wrapper asks torch whether a CUDA graph is being captured; on a
    # CPU-only interpreter run nothing is
    torch.cuda.is_current_stream_capturing = lambda: False
    rng = np.random.default_rng(seed)
    B, H, D = 1, 2, 128
    q = (rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32)
    v = (rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32)
    nblk = T // bs
    idx = np.full((B, T, K), -1, np.int32)
    bias = np.zeros((B, T, K), np.float32)
    for t in range(T):
        rem = [b for b in range(nblk) if b <= t // bs - lb]
        if rem:
            ch = rng.choice(rem, size=min(K, len(rem)), replace=False)
            idx[0, t, :len(ch)] = np.sort(ch)
            bias[0, t, :len(ch)] = rng.standard_normal(len(ch)).astype(np.float32)
    out_e2e = e2e.triton_gather_attention_e2e(
        torch.tensor(q), torch.tensor(k), torch.tensor(v), torch.tensor(idx)[:, None],
        torch.tensor(bias), torch.arange(T)[None], None, bs, 1.0 / math.sqrt(D), lb * bs)
    # paged prefill + decode of the same sequence through a shuffled block table
    P = nblk + 3
    perm = rng.permutation(P)[:nblk].astype(np.int32)
    kc = np.zeros((P, bs, H, D), np.float32)
    vc = np.zeros((P, bs, H, D), np.float32)
    for b in range(nblk):
        kc[perm[b]] = k[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
        vc[perm[b]] = v[0, :, b * bs:(b + 1) * bs].transpose(1, 0, 2)
    bt = perm[None].copy()
    qp = np.ascontiguousarray(q[0].transpose(1, 0, 2))           # [T,H,D]
    out_p = torch.zeros(T, H, D)
    ti = torch.tensor(idx[0])[None].expand(H, -1, -1)
    tb = torch.tensor(bias[0])[None].expand(H, -1, -1)
    at.dash_sparse_attn(torch.tensor(qp), torch.tensor(kc), torch.tensor(vc), ti, tb,
                        torch.tensor(bt), torch.tensor([0, T], dtype=torch.int32),
                        torch.tensor([T], dtype=torch.int32),
                        torch.tensor([0], dtype=torch.int32), T, H, 1.0 / math.sqrt(D), out_p,
                        local_blocks=lb, sparse_block_size=bs)
    out_d = torch.zeros(1, H, D)
    at.dash_sparse_attn_decode(torch.tensor(qp[-1:]), torch.tensor(kc), torch.tensor(vc),
                               ti[:, -1:], tb[:, -1:], torch.tensor(bt),
                               torch.tensor([T], dtype=torch.int32), H, 1.0 / math.sqrt(D),
                               out_d, 1, local_blocks=lb, sparse_block_size=bs)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), seed=seed, q=q, k=k, v=v, idx=idx, bias=bias,
        bs=bs, lb=lb, block_table=bt, out_e2e=out_e2e.numpy(), out_paged=out_p.numpy(),
        out_decode=out_d.numpy())
    print(name, "saved")


def serving_plan_case(name, seed):
    """The serving step's planning helpers of the sglang wheel (route_triton.py:
    kbar_all_plan, prefill_row2req, kbar_tail_plan) on seeded block tables,
    including empty requests, prefixes not on a block boundary and blocks past
    the table width."""
    from sglang.srt.layers.attention.unlimited_dash_ops import route_triton as rt
    rng = np.random.default_rng(seed)
    res = {}
    for bs in (16, 32, 64):
        R = 7
        seq = rng.integers(0, 700, R)
        seq[2] = 0
        ctx = np.minimum(seq, rng.integers(0, 400, R))
        ctx[3] = seq[3]
        W = int(-(-seq.max() // bs)) + 2
        bt = rng.integers(0, 5000, (R, W)).astype(np.int32)
        q_lens = seq - ctx
        cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
        for mb in (W, W - 3):
            p, t = rt.kbar_all_plan(block_table=torch.tensor(bt), seq_lens=torch.tensor(seq),
                                    context_lens=torch.tensor(ctx), block_size=bs, max_block=mb,
                                    max_query_len=int(q_lens.max()), device="cpu")
            res[f"all_{bs}_{mb == W}_pages"], res[f"all_{bs}_{mb == W}_ntok"] = p.numpy(), t.numpy()
        for tp in (1, 3):
            p, t = rt.kbar_tail_plan(block_table=torch.tensor(bt), seq_lens=torch.tensor(seq),
                                     block_size=bs, tail_pages=tp, device="cpu")
            res[f"tail_{bs}_{tp}_pages"], res[f"tail_{bs}_{tp}_ntok"] = p.numpy(), t.numpy()
        res[f"row2req_{bs}"] = rt.prefill_row2req(cu_seqlens_q=torch.tensor(cu),
                                                  device="cpu").numpy()
        res[f"seq_{bs}"], res[f"ctx_{bs}"], res[f"bt_{bs}"], res[f"cu_{bs}"] = seq, ctx, bt, cu
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **res)
    print(name, "saved")


def dash_attention_case(da, name, seed):
    """The reference's own DashAttention.forward (CPU: its dense path) and its
    autograd backward, stage 0 head_cls and indexer, the checkpoint's block
    size 32 with a 4-block window, K = 12, with and without a per-query
    candidate domain."""
    B, S, hidden, H, D = 1, 600, 256, 2, 128
    w, x = dash_attention_inputs(seed, B, S, hidden, H, D, n_pages=3, page_tokens=150)
    da._KS._k = 12                       # the schedule's hard top-k (eval: no anneal)
    res = {"input_sha": sha(*w.values(), *x.values())}
    nblk = -(-S // 32)
    rng = np.random.default_rng(seed + 1)
    cand = rng.random((B, S, nblk)) < 0.4
    # scale 2.0 (the module default): smooth priors, every pick has prior > 0;
    # scale 128 (the checkpoint's): narrow support, zero-prior picks whose
    # order among equal priors is torch.topk's
    for stage0, use_cand, scale in (("head_cls", False, 2.0), ("head_cls", True, 2.0),
                                    ("indexer", False, 2.0), ("head_cls", False, 128.0)):
        sp = dict(sparse_block_size=32, sparse_local_block=4, dash_scaling_factor=scale,
                  dash_prior_floor=1e-2, sparse_topk_blocks=16, sparse_index_dim=128,
                  dash_sigma=1.0)
        cfg = types.SimpleNamespace(num_attention_heads=H, hidden_size=hidden, rms_norm_eps=1e-6,
                                    sparse_attention_config=sp)
        if True:
            os.environ["DASH_STAGE0"] = stage0
            m = da.DashAttention(cfg)
            with torch.no_grad():
                for n_, t in w.items():
                    getattr(m, n_).copy_(torch.tensor(t)) if n_ == "head_cls" else \
                        getattr(m, n_).weight.copy_(torch.tensor(t))
            m.eval()
            rec = {}
            sel = m._select_and_bias

            def hook(prior, cnd, nb, _sel=sel, _rec=rec):
                out = _sel(prior, cnd, nb)
                _rec["prior"], _rec["cand"] = prior.detach().clone(), cnd.clone()
                _rec["topi"], _rec["bias"], _rec["valid"] = (t.detach().clone() for t in out)
                return out
            m._select_and_bias = hook
            q, k, v = (torch.tensor(x[n_]).requires_grad_(True) for n_ in ("q", "k", "v"))
            hs = torch.tensor(x["hidden"]).requires_grad_(True)
            out = m(hs, q, k, v, position_embeddings=(torch.tensor(x["cos"]), torch.tensor(x["sin"])),
                    block_cand=torch.tensor(cand) if use_cand else None)
            (out * torch.tensor(x["dout"])).sum().backward()
            tag = f"{stage0}_{int(use_cand)}_{int(scale)}"
            rows = np.linspace(0, S - 1, 64).astype(np.int64)
            res["rows"] = rows
            res[f"out_{tag}"] = out.detach().numpy()[:, :, rows]
            res[f"topi_{tag}"] = rec["topi"].numpy().astype(np.int32)
            res[f"valid_{tag}"] = rec["valid"].numpy()
            res[f"bias_{tag}"] = rec["bias"].numpy()
            res[f"prior_{tag}"] = rec["prior"].numpy()
            res[f"candm_{tag}"] = np.packbits(rec["cand"].numpy(), axis=-1)
            res[f"dq_{tag}"] = q.grad.numpy()[:, :, rows]
            res[f"dv_{tag}"] = v.grad.numpy()[:, :, rows]
            res[f"dqproj_{tag}"] = m.q_proj.weight.grad.numpy()
            res[f"dheadcls_{tag}"] = (m.head_cls.grad.numpy() if m.head_cls.grad is not None
                                      else np.zeros(128, np.float32))
    res["cand"] = np.packbits(cand, axis=-1)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **res)
    print(name, "saved")


def page_aware_case(name, seed):
    """Page-aware candidate domain: the indexer's id builders and candidate mask
    (_sparse_base_impl.py), _dash_block_cand (modeling_deepseekv2.py), the
    contiguous decoder's decode allow (modeling_anantaocr.py) and the sglang
    PageIsolationState / decode_allow_fused / local_union_fused (Triton
    interpreted) over a short serving trace."""
    import ananta_ref._sparse_base_impl as sb
    import ananta_ref.modeling_deepseekv2 as mdl
    import ananta_ref.modeling_anantaocr as ma
    from sglang.srt.layers.attention.unlimited_dash_ops import page_state as ps
    from sglang.srt.layers.attention.unlimited_dash_ops import decode_meta_triton as dm
    from oracle.page_oracle import (make_document_ids, IMAGE_TOKEN_ID as IMG,
                                    PAGE_TOKEN_ID as PG, MM_PAD_SHIFT)
    torch.cuda.is_current_stream_capturing = lambda: False
    rng = np.random.default_rng(seed)
    res = {}

    # ---- contiguous documents ----
    S, bs = 1500, 64
    docs = [
        make_document_ids(rng, S, n_pages=4, page_tokens=273, text_in_page=3, empty_pages=1,
                          response_pages=2),
        make_document_ids(rng, S, n_pages=5, page_tokens=200, markers=False),
        make_document_ids(rng, S, n_pages=30, page_tokens=20, empty_pages=6, lead_images=10,
                          response_pages=3),
    ]
    ids = np.stack(docs)
    B = ids.shape[0]
    nblk = -(-S // bs)
    dev = torch.device("cpu")
    idx = types.SimpleNamespace(q_proj=types.SimpleNamespace(weight=torch.zeros(1, device=dev)),
                                per_page_image_tokens=100, block_size=bs, layer_idx=0,
                                _page_aware_diag_logged=True, image_bucket_constraint=True,
                                image_token_id=IMG, page_token_id=PG)
    for m in ("_build_page_aware_image_block_mask", "_build_image_block_allow_mask",
              "_build_page_aware_ids", "_build_flat_image_token_mask",
              "_build_kl_candidate_mask", "_log_image_mask"):
        setattr(idx, m, types.MethodType(getattr(sb.DeepseekV2Indexer, m), idx))
    idx._diag_due = lambda key: False                       # no diagnostic prints
    tid = torch.tensor(ids)
    pos = torch.arange(S)[None].expand(B, -1)
    for scope in (False, True):
        sb._PAGE_SCOPE_PREFILL = scope
        itm, ipi, qpi = sb.DeepseekV2Indexer._build_page_aware_ids(idx, tid, IMG, PG, S)
        res[f"itm_{int(scope)}"] = itm.numpy()
        res[f"ipi_{int(scope)}"] = ipi.numpy()
        res[f"qpi_{int(scope)}"] = qpi.numpy()
        cm = sb.DeepseekV2Indexer._build_kl_candidate_mask(idx, pos, nblk, itm, B, S, ipi, qpi)
        res[f"cand_page_{int(scope)}"] = np.packbits(cm[:, 0].numpy(), axis=-1)
    sb._PAGE_SCOPE_PREFILL = False
    # a truncated key length (ids longer than the keys) and a padded one
    for kl in (1000, 1700):
        itm, ipi, qpi = sb.DeepseekV2Indexer._build_page_aware_ids(idx, tid, IMG, PG, kl)
        res[f"ipi_kl{kl}"] = ipi.numpy()
        res[f"qpi_kl{kl}"] = qpi.numpy()
    flat = sb.DeepseekV2Indexer._build_flat_image_token_mask(idx, tid, IMG, S)
    res["img_blk"] = sb.DeepseekV2Indexer._build_image_block_allow_mask(idx, flat, nblk).numpy()
    res["img_blk_short"] = sb.DeepseekV2Indexer._build_image_block_allow_mask(
        idx, flat, nblk - 5).numpy()
    idx.image_bucket_constraint = False
    cm = sb.DeepseekV2Indexer._build_kl_candidate_mask(idx, pos[:, :300], nblk, flat, B, 300)
    res["cand_flat"] = np.packbits(cm[:, 0].numpy(), axis=-1)
    idx.image_bucket_constraint = True
    router = types.SimpleNamespace(q_chunk=512)
    itm, ipi, qpi = mdl._dash_page_ids(None, idx, tid, S)
    bc = mdl._dash_block_cand(None, idx, router, pos, itm, ipi, qpi, nblk, B, S)
    res["block_cand"] = np.packbits(bc.numpy(), axis=-1)
    # positions that differ from the token index (a shifted window of queries)
    pos2 = torch.clamp(torch.arange(S)[None].expand(B, -1) + 37, max=S + 20)
    cm = sb.DeepseekV2Indexer._build_kl_candidate_mask(idx, pos2, nblk, itm, B, S, ipi, qpi)
    res["cand_pos_shift"] = np.packbits(cm[:, 0].numpy(), axis=-1)

    # ---- contiguous decoder: decode allow over a few decode steps ----
    class _Cache:
        def __init__(self):
            self.n = 0

        def get_seq_length(self):
            return self.n
    cache = _Cache()
    L0 = 1300
    ma._uocr_dash_decode_allow(idx, tid[:, :L0], cache)
    st = cache._uocr_pg
    res["dec_bmin"], res["dec_bmax"] = st["bmin"].numpy(), st["bmax"].numpy()
    res["dec_pp"], res["dec_mcum"] = st["pp"].numpy(), st["mcum"].numpy()
    cache.n = L0
    steps = []
    dec_ids = rng.integers(0, 1000, size=(6, B))
    dec_ids[1, 0] = PG
    dec_ids[3, :] = PG
    dec_ids[4, 2] = PG
    for k in range(dec_ids.shape[0]):
        allow = ma._uocr_dash_decode_allow(idx, torch.tensor(dec_ids[k][:, None]), cache)
        steps.append(np.packbits(allow.numpy(), axis=-1))
        cache.n += 1
    res["dec_ids"] = dec_ids
    assert len({a.shape for a in steps}) == 1
    res["dec_allow"] = np.stack(steps)

    # ---- sglang serving trace ----
    sbs, per = 16, 24
    cfg = {"image_token_id": IMG, "page_token_id": PG, "per_page_image_tokens": per}
    pst = ps.PageIsolationState(cfg, sbs)
    P = 96
    num_slots = P * sbs
    perm = rng.permutation(P)
    W = 24
    R = 3
    bt = np.zeros((R, W), np.int64)
    for r in range(R):
        bt[r] = perm[r * W:(r + 1) * W]
    doc = [make_document_ids(rng, 200, n_pages=4, page_tokens=30, text_in_page=2,
                             response_pages=0),
           make_document_ids(rng, 170, n_pages=3, page_tokens=40, markers=False),
           make_document_ids(rng, 190, n_pages=5, page_tokens=25, empty_pages=1,
                             lead_images=7, response_pages=0)]
    seg = doc[1][5:60]                                      # multimodal pad ids
    seg[seg == IMG] = MM_PAD_SHIFT + 5
    # steps: (per request: (start, n_tokens, ids)); extend steps first, then decodes
    trace = []
    lens = [0, 0, 0]
    plan = [[120, 170, 150], [80, 0, 40], [1, 1, 1], [1, 1, 1], [1, 1, 1], [1, 1, 1]]
    gen_ids = rng.integers(0, 1000, size=(4, R))
    gen_ids[0, 0] = PG
    gen_ids[1, 2] = PG
    gen_ids[2, 1] = IMG
    gen_ids[3, 0] = PG
    for si, q_lens in enumerate(plan):
        toks, starts, qs, rows = [], [], [0], []
        n_dec = 0
        for r in range(R):
            n = q_lens[r]
            if n == 0:
                continue
            if si >= 2:
                t = [int(gen_ids[si - 2, r])]
            else:
                t = doc[r][lens[r]:lens[r] + n].tolist()
            toks += t
            starts.append(lens[r])
            rows.append(r)
            qs.append(qs[-1] + n)
        nr = len(rows)
        q_start = torch.tensor(qs, dtype=torch.int64)
        start_pos = torch.tensor(starts, dtype=torch.int64)
        btab = torch.tensor(bt[rows])
        T = qs[-1]
        gen_start = None
        if si >= 2:
            n_dec = T
        layout = ps.BatchLayout(num_tokens=T, num_reqs=nr, q_start=q_start, start_pos=start_pos,
                                block_table=btab, req_of_token=ps._req_of_token(q_start, T),
                                num_decode_tokens=n_dec, gen_start=gen_start)
        slots = []
        for j, r in enumerate(rows):
            for i in range(qs[j + 1] - qs[j]):
                p = starts[j] + i
                slots.append(int(bt[r, p // sbs]) * sbs + p % sbs)
        slot_mapping = torch.tensor(slots, dtype=torch.int64)
        ids_t = torch.tensor(toks, dtype=torch.int64)
        q_page = pst.step(ids_t, layout, slot_mapping, num_slots).clone()
        allow = pst.build_query_allow(layout, q_page, W, P).clone()
        rec = {"rows": np.array(rows), "q_start": np.array(qs), "start_pos": np.array(starts),
               "ids": np.array(toks), "slots": np.array(slots), "n_dec": n_dec,
               "q_page": q_page.numpy(), "allow": allow.numpy(),
               "slot_img_page": pst._slot_img_page.numpy().copy(),
               "slot_marker_cum": pst._slot_marker_cum.numpy().copy(),
               "slot_img_run": pst._slot_img_run.numpy().copy(),
               "slot_prompt_pages": pst._slot_prompt_pages.numpy().copy()}
        for j, r in enumerate(rows):
            lens[r] += qs[j + 1] - qs[j]
        if si >= 2:
            seq_lens = torch.tensor([lens[r] for r in rows], dtype=torch.int32)
            da_ = dm.decode_allow_fused(block_table=btab, page_state=pst, q_page=q_page,
                                        seq_lens=seq_lens, max_block=W, num_blocks=P,
                                        block_size=sbs)
            rec["decode_allow"] = da_.numpy().copy()
            lu = dm.local_union_fused(allow=da_, seq_lens=seq_lens,
                                      out=torch.zeros(nr, W, dtype=torch.int8), max_block=W,
                                      block_size=sbs, local_blocks=2)
            rec["local_union"] = lu.numpy().copy()
            rec["seq_lens"] = seq_lens.numpy()
        trace.append(rec)
    for i, rec in enumerate(trace):
        for k, v in rec.items():
            res[f"sg{i}_{k}"] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), seed=seed, ids=ids, S=S, bs=bs,
                        nblk=nblk, per_page=100, sg_bs=sbs, sg_per=per, sg_P=P, sg_W=W,
                        sg_bt=bt, sg_steps=len(trace), **res)
    print(name, "saved")


def page_coords_case(name, seed):
    """Page2D coordinates of the sglang wheel over a serving trace: the torch
    PageCoordState.step for prefill chunks, the fused one-token decode
    (decode_meta_fused, Triton interpreted) for decode steps, a finished
    request whose state row is reused by a new one, and the cos/sin tables
    (PageRope2D.cos_sin in torch and cos_sin_2d_fused interpreted)."""
    from sglang.srt.layers.attention.unlimited_dash_ops import page_state as ps
    from sglang.srt.layers.attention.unlimited_dash_ops import decode_meta_triton as dm
    from sglang.srt.layers.attention.unlimited_dash_ops import page2d_rope as pr
    from oracle.page_oracle import make_document_ids, IMAGE_TOKEN_ID as IMG, PAGE_TOKEN_ID as PG
    torch.cuda.is_current_stream_capturing = lambda: False
    rng = np.random.default_rng(seed)
    sbs, per, P, W = 16, 24, 128, 24
    cfg = {"image_token_id": IMG, "page_token_id": PG, "per_page_image_tokens": per}
    pst = ps.PageIsolationState(cfg, sbs)
    coord = pr.PageCoordState(cfg, max_reqs=3, max_pages=6)
    rope = pr.PageRope2D(128, 10000.0, 256.0, 1, "resample", page_mod=2)
    num_slots = P * sbs
    perm = rng.permutation(P)
    bt = np.stack([perm[i * W:(i + 1) * W] for i in range(4)]).astype(np.int64)
    docs = [make_document_ids(rng, 200, n_pages=4, page_tokens=30, text_in_page=2, response_pages=0),
            make_document_ids(rng, 170, n_pages=3, page_tokens=40, markers=False),
            make_document_ids(rng, 190, n_pages=5, page_tokens=25, empty_pages=1, lead_images=7,
                              response_pages=0),
            make_document_ids(rng, 120, n_pages=2, page_tokens=30, response_pages=0)]
    lens = [0, 0, 0, 0]
    # per step: (request, n_tokens) pairs; n == 1 after the prompt is a decode token
    plan = [[(0, 120), (1, 170), (2, 150)], [(0, 80), (2, 40)],
            [(0, 1), (1, 1), (2, 1)], [(0, 1), (1, 1), (2, 1)],
            [(3, 90)],                                   # request 3 takes request 1's row
            [(0, 1), (2, 1), (3, 1)], [(0, 1), (2, 1), (3, 1)]]
    gen = rng.integers(0, 1000, size=(len(plan), 4))
    gen[2, 0] = PG
    gen[3, 2] = PG
    gen[5, 3] = IMG
    gen[6, 0] = PG
    res = {"bt": bt}
    prompt_len = [200, 170, 190, 90]
    for si, st in enumerate(plan):
        rows = [r for r, _ in st]
        ns = [n for _, n in st]
        toks, qs, starts = [], [0], []
        for r, n in st:
            if lens[r] >= prompt_len[r]:
                toks.append(int(gen[si, r]))
            else:
                toks += docs[r][lens[r]:lens[r] + n].tolist()
            starts.append(lens[r])
            qs.append(qs[-1] + n)
        T = qs[-1]
        decode = all(lens[r] >= prompt_len[r] for r in rows)
        q_start = torch.tensor(qs, dtype=torch.int64)
        btab = torch.tensor(bt[rows])
        slots = [int(bt[r, (starts[j] + i) // sbs]) * sbs + (starts[j] + i) % sbs
                 for j, (r, n) in enumerate(st) for i in range(n)]
        ids_t = torch.tensor(toks, dtype=torch.int64)
        rec = {"rows": np.array(rows), "q_start": np.array(qs), "start_pos": np.array(starts),
               "ids": np.array(toks), "slots": np.array(slots), "decode": int(decode)}
        if decode:
            seq = torch.tensor([lens[r] + 1 for r in rows], dtype=torch.int32)
            q_page, (tok, page) = dm.decode_meta_fused(
                input_ids=ids_t, block_table=btab, seq_lens=seq,
                slot_mapping=torch.tensor(slots, dtype=torch.int64), page_state=pst,
                coord_state=coord, num_slots=num_slots, block_size=sbs)
            cos = torch.zeros(T, 128, dtype=torch.bfloat16)
            sin = torch.zeros(T, 128, dtype=torch.bfloat16)
            dm.cos_sin_2d_fused(rope=rope, tok_pos=tok, page_pos=page, dtype=torch.bfloat16,
                                out_cos=cos, out_sin=sin)
            rec["cos_fused"] = cos.view(torch.int16).numpy()
            rec["sin_fused"] = sin.view(torch.int16).numpy()
            rec["q_page"] = q_page.numpy().copy()
        else:
            layout = ps.BatchLayout(num_tokens=T, num_reqs=len(rows), q_start=q_start,
                                    start_pos=torch.tensor(starts, dtype=torch.int64),
                                    block_table=btab, req_of_token=ps._req_of_token(q_start, T),
                                    num_decode_tokens=0, gen_start=None)
            tok, page = coord.step(ids_t, layout)
        c32, s32 = rope.cos_sin(tok, page, torch.float32)
        rec["tok"], rec["page"] = tok.numpy().copy(), page.numpy().copy()
        rec["cos32"], rec["sin32"] = c32.numpy(), s32.numpy()
        for r, n in st:
            lens[r] += n
        for k, v in rec.items():
            res[f"s{si}_{k}"] = np.asarray(v)
    res["inv_tok"], res["inv_page"] = rope.inv_tok.numpy(), rope.inv_page.numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), steps=len(plan), sbs=sbs, P=P, W=W,
                        max_reqs=3, max_pages=6, page_mod=2, n_tok=rope.n_tok, **res)
    print(name, "saved")


def _gemma_forward_native():
    """GemmaRMSNorm.forward_native of the sglang wheel (WHL layernorm.py:1113-1131),
    compiled from the wheel's own source (the module's imports need a full
    sglang runtime)."""
    import ast
    whl = glob.glob(os.path.join(REF, "wheel", "*.whl"))[0]
    src = zipfile.ZipFile(whl).read("sglang/srt/layers/layernorm.py").decode()
    tree = ast.parse(src)
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "GemmaRMSNorm")
    fn = next(n for n in cls.body if isinstance(n, ast.FunctionDef) and n.name == "forward_native")
    mod = ast.Module(body=[fn], type_ignores=[])
    import typing
    ns = {"torch": torch, "Optional": typing.Optional, "Union": typing.Union,
          "Tuple": typing.Tuple}
    exec(compile(mod, "layernorm.py", "exec"), ns)
    return ns["forward_native"]


def frontend_case(name, seed):
    """Router front end: the reference's _router_qk (index projections +
    _RMSNorm + RoPE, modeling_deepseekv2.py:336-348) and the sglang index branch
    (Linear + GemmaRMSNorm.forward_native + _rope2d_torch), bf16 on CPU."""
    import ananta_ref.dash_attention as da
    import ananta_ref.modeling_deepseekv2 as mdl
    from sglang.srt.layers.attention.unlimited_dash_ops import page2d_rope as pr
    gemma = _gemma_forward_native()
    rng = np.random.default_rng(seed)
    B, S, Hd, d, eps = 2, 83, 192, 128, 1e-6
    bf = torch.bfloat16
    hidden = torch.tensor(rng.standard_normal((B, S, Hd)), dtype=torch.float32).to(bf)
    wq = torch.tensor(rng.standard_normal((d, Hd)) / math.sqrt(Hd), dtype=torch.float32).to(bf)
    wk = torch.tensor(rng.standard_normal((d, Hd)) / math.sqrt(Hd), dtype=torch.float32).to(bf)
    nq = torch.tensor(rng.standard_normal(d) * 0.1, dtype=torch.float32).to(bf)
    nk = torch.tensor(rng.standard_normal(d) * 0.1, dtype=torch.float32).to(bf)
    pos = torch.tensor(rng.integers(0, 5000, size=(B, S)), dtype=torch.float32)
    inv = 1.0 / (10000.0 ** (torch.arange(0, d // 2, dtype=torch.float32) / (d // 2)))
    ang = pos[..., None] * inv
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(bf), emb.sin().to(bf)

    def lin(w):
        m = torch.nn.Linear(Hd, d, bias=False, dtype=bf)
        m.weight.data.copy_(w)
        return m

    def hf_norm(w):
        m = da._RMSNorm(d, eps=eps).to(bf)
        m.weight.data.copy_(w)
        return m
    router = types.SimpleNamespace(index_dim=d, q_proj=lin(wq), k_proj=lin(wk),
                                   q_norm=hf_norm(nq), k_norm=hf_norm(nk))
    with torch.no_grad():
        hq, hk = mdl._router_qk(router, hidden, (cos, sin))
        hq0, hk0 = mdl._router_qk(router, hidden, None)
        T = B * S
        x = hidden.view(T, Hd)
        out = {}
        for tag, w, nw in (("q", wq, nq), ("k", wk, nk)):
            y = torch.nn.functional.linear(x, w)
            stub = types.SimpleNamespace(weight=nw, variance_epsilon=eps)
            y = gemma(stub, y.view(-1, 1, d)).view(T, d)
            out[tag] = pr._rope2d_torch(y, cos.view(T, d), sin.view(T, d), d).float()
    # main-branch RoPE of a 2-head q and a 1-head k (apply_page2d_rope's torch path)
    T = B * S
    rx = torch.tensor(rng.standard_normal((T, 2 * d)), dtype=torch.float32).to(bf)
    ry = torch.tensor(rng.standard_normal((T, d)), dtype=torch.float32).to(bf)
    with torch.no_grad():
        ox = pr._rope2d_torch(rx, cos.view(T, d), sin.view(T, d), d)
        oy = pr._rope2d_torch(ry, cos.view(T, d), sin.view(T, d), d)
    u16 = lambda t: t.contiguous().view(torch.int16).numpy()
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), seed=seed, B=B, S=S, Hd=Hd, d=d, eps=eps,
        rope_x=u16(rx), rope_y=u16(ry), rope_ox=u16(ox), rope_oy=u16(oy),
        hidden=u16(hidden), wq=u16(wq), wk=u16(wk), nq=u16(nq), nk=u16(nk), cos=u16(cos),
        sin=u16(sin), hf_q=hq.numpy(), hf_k=hk.numpy(), hf_q_norope=hq0.numpy(),
        hf_k_norope=hk0.numpy(), sg_q=out["q"].numpy(), sg_k=out["k"].numpy())
    print(name, "saved")


def backward_case(name, seed):
    """The reference's training backward (_E2EGatherAttnFn.backward: the Triton
    dq/d_bias and dk/dv kernels, interpreted on the CPU, fp32) and its entmax
    Jacobian (_Entmax15) on small shapes.  Routed lists hold -1 slots and ids
    of blocks inside the local window; no duplicate ids (the reference's
    dedup keeps an unspecified one of equal ids)."""
    import ananta_ref.sparse_gather_e2e_triton as e2e
    import ananta_ref.dash_attention as da
    rng = np.random.default_rng(seed)
    out = {}

    def bf16_exact(a):
        # inputs representable in bf16 (stored as uint16): the same values drive
        # the fp32 and the bf16 kernels
        return torch.tensor(a).to(torch.bfloat16).float().numpy()

    def as_u16(a):
        return torch.tensor(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    for c, (B, HQ, H, T, bs, LW, K) in enumerate([(1, 1, 1, 128, 64, 64, 2),
                                                   (1, 2, 1, 192, 64, 64, 2)]):
        D = 128
        q = bf16_exact(rng.standard_normal((B, HQ, T, D)) * 0.5)
        k = bf16_exact(rng.standard_normal((B, H, T, D)) * 0.5)
        v = bf16_exact(rng.standard_normal((B, H, T, D)) * 0.5)
        do = bf16_exact(rng.standard_normal((B, HQ, T, D)))
        nblk = (T + bs - 1) // bs
        idx = np.full((B, T, K), -1, np.int32)
        for b in range(B):
            for t in range(T):
                pool = list(range(0, t // bs + 1))        # remote and window blocks
                n = min(K, len(pool), int(rng.integers(0, K + 1)))
                if n:
                    idx[b, t, :n] = rng.choice(pool, size=n, replace=False)
        bias = (rng.standard_normal((B, T, K)) * 0.5).astype(np.float32)
        tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
        tb = torch.tensor(bias, requires_grad=True)
        o = e2e.triton_gather_attention_e2e(tq, tk, tv, torch.tensor(idx)[:, None], tb,
                                            torch.arange(T)[None].expand(B, T), None, bs,
                                            1.0 / math.sqrt(D), LW)
        node = o.grad_fn.next_functions[0][0]
        lse = node.saved_tensors[-1].detach().numpy()              # [B, T, HQ]
        o.backward(torch.tensor(do))
        tr = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3))   # -> [B, T, heads, D]
        out.update({f"c{c}_q": as_u16(tr(q)), f"c{c}_k": as_u16(tr(k)), f"c{c}_v": as_u16(tr(v)),
                    f"c{c}_do": as_u16(tr(do)),
                    f"c{c}_idx": idx, f"c{c}_bias": bias, f"c{c}_o": tr(o.detach().numpy()),
                    f"c{c}_lse": lse, f"c{c}_dq": tr(tq.grad.numpy()), f"c{c}_dk": tr(tk.grad.numpy()),
                    f"c{c}_dv": tr(tv.grad.numpy()), f"c{c}_dbias": tb.grad.numpy(),
                    f"c{c}_cfg": np.array([B, HQ, H, T, bs, LW, K])})
    # entmax: rows like _route's input (masked entries at -1e4, scaled scores)
    x = (rng.standard_normal((40, 37)) * 3).astype(np.float32)
    x[rng.random(x.shape) < 0.3] = -1e4
    x[:, 0] = rng.standard_normal(40) * 3
    tx = torch.tensor(x, requires_grad=True)
    y = da.entmax15(tx, -1)
    dy = rng.standard_normal(x.shape).astype(np.float32)
    y.backward(torch.tensor(dy))
    out.update(ent_x=x, ent_y=y.detach().numpy(), ent_dy=dy, ent_dx=tx.grad.numpy())
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
    print(name, "saved")


def main(names=None):
    da, md = import_reference()
    torch.set_num_threads(os.cpu_count())
    cases = {
        # C1: BASELINE config 1 (fp32, B=1, 10 heads, S=1348, bs=64, window 4 blocks, k=8)
        "c1_headcls": lambda: prefill_case(
            da, md, "c1_headcls", seed=0, B=1, H=10, S=1348, bs=64, lb=4, K=8, topm=8,
            stage0="head_cls", hc_std=0.0, n_pages=0, page_tokens=273, off_std=0.0,
            sample_rows=np.linspace(0, 1347, 48).astype(np.int64)),
        # the checkpoint's own DASH settings (config.json: sparse_block_size 32,
        # sparse_local_block 4, dash_topk_blocks 12) on the config-1 shape with
        # page offsets
        "c1_bs32": lambda: prefill_case(
            da, md, "c1_bs32", seed=10, B=1, H=10, S=1348, bs=32, lb=4, K=12, topm=12,
            stage0="head_cls", hc_std=0.0, n_pages=4, page_tokens=273, off_std=0.2,
            sample_rows=np.linspace(0, 1347, 64).astype(np.int64)),
        # small cases: learned head_cls, topm > K, page offsets; indexer stage-0
        "small_headcls": lambda: prefill_case(
            da, md, "small_headcls", seed=1, B=2, H=2, S=300, bs=16, lb=2, K=4, topm=6,
            stage0="head_cls", hc_std=1.0, n_pages=5, page_tokens=50, off_std=0.3),
        "small_indexer": lambda: prefill_case(
            da, md, "small_indexer", seed=2, B=1, H=2, S=400, bs=32, lb=2, K=5, topm=5,
            stage0="indexer", hc_std=0.0, n_pages=6, page_tokens=60, off_std=0.3),
        "decode_small": lambda: decode_case(da, md, "decode_small", seed=3, B=4, H=2, S=1000,
                                            bs=64, lb=4, K=8, topm=8),
        "paged_router": lambda: paged_router_case("paged_router", seed=4),
        "triton_interp": lambda: triton_interp_case(da, md, "triton_interp", seed=5),
        # 32-token blocks (one page per block) with a 4-block window
        "triton_interp_bs32": lambda: triton_interp_case(da, md, "triton_interp_bs32", seed=9,
                                                         T=256, bs=32, lb=4, K=3),
        "page_aware": lambda: page_aware_case("page_aware", seed=6),
        "serving_plan": lambda: serving_plan_case("serving_plan", seed=11),
        "page_coords": lambda: page_coords_case("page_coords", seed=13),
        "dash_attention": lambda: dash_attention_case(da, "dash_attention", seed=12),
        "frontend": lambda: frontend_case("frontend", seed=7),
        "backward": lambda: backward_case("backward", seed=8),
    }
    for n in (names or list(cases)):
        cases[n]()


if __name__ == "__main__":
    main(sys.argv[1:])
