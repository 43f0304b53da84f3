"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (default ``/root/reference``,
override with ``DASH_REFERENCE``):

    python tests/golden/make_golden.py

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

REF = os.environ.get("DASH_REFERENCE", "/root/reference")


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def import_reference():
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


def triton_interp_case(da, md, name, seed):
    """Reference Triton kernels, interpreted on CPU, on tiny shapes."""
    import ananta_ref.sparse_gather_e2e_triton as e2e
    from sglang.srt.layers.attention.unlimited_dash_ops import attend_triton as at
    # the decode wrapper asks torch whether a CUDA graph is being captured; on a
    # CPU-only interpreter run nothing is
    torch.cuda.is_current_stream_capturing = lambda: False
    rng = np.random.default_rng(seed)
    B, H, T, D, bs, lb, K = 1, 2, 96, 128, 16, 2, 3
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


def main():
    da, md = import_reference()
    torch.set_num_threads(os.cpu_count())
    # C1: BASELINE config 1 (fp32, B=1, 10 heads, S=1348, bs=64, window 4 blocks, k=8)
    prefill_case(da, md, "c1_headcls", seed=0, B=1, H=10, S=1348, bs=64, lb=4, K=8, topm=8,
                 stage0="head_cls", hc_std=0.0, n_pages=0, page_tokens=273, off_std=0.0,
                 sample_rows=np.linspace(0, 1347, 48).astype(np.int64))
    # small cases: learned head_cls, topm > K, page offsets; indexer stage-0
    prefill_case(da, md, "small_headcls", seed=1, B=2, H=2, S=300, bs=16, lb=2, K=4, topm=6,
                 stage0="head_cls", hc_std=1.0, n_pages=5, page_tokens=50, off_std=0.3)
    prefill_case(da, md, "small_indexer", seed=2, B=1, H=2, S=400, bs=32, lb=2, K=5, topm=5,
                 stage0="indexer", hc_std=0.0, n_pages=6, page_tokens=60, off_std=0.3)
    decode_case(da, md, "decode_small", seed=3, B=4, H=2, S=1000, bs=64, lb=4, K=8, topm=8)
    paged_router_case("paged_router", seed=4)
    triton_interp_case(da, md, "triton_interp", seed=5)


if __name__ == "__main__":
    main()
