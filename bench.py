"""DASH block-sparse attention benchmark (router + gather attention) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c4] [--no-decode] [--no-e2e] [--no-cpu]

Workload ("c2"): bf16 prefill, B=4 sequences per GPU,
10 heads, head_dim 128, S=9,248 (32 pages x 273 + 512 text tokens), block 64,
local window 4 blocks, routed cap k=16, q/k/v ~ N(0,1)*0.5 with per-page mean
offsets ~ N(0,0.2); router queries/keys drawn the same way.  One step = k-bar
pooling + routing (scores, 1.5-entmax, top-k, bias) + tcgen05 gather attention
for all B*S tokens and all heads.  Inputs are created on the device and exceed
L2 (126 MB), so no flush is needed between steps.  `decode` adds BASELINE
configs[2] (batch 64 decode over a 27,556-token paged cache, k=32) measured in
the same run.  With N GPUs every rank runs its own shard of sequences (weak
scaling, no collective inside the step); value = tokens of all ranks / max
rank time.

`--impl reference` times the reference's own CPU inference path on the host:
the reference is Python/PyTorch+Triton and cannot travel to the GPU box, so
the arm runs a torch fp32 restatement of it (oracle/torch_path.py: head_cls
k-bar, scores, canonical selection and the dense masked attention of
dash_attention.py:980-1006, checked against the reference's own outputs by
tests/test_torch_path.py) with every host thread, on a bounded sample of the
same workload (query tokens of one sequence; every token of the dense form
costs the same).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

C2 = dict(name="config2_prefill_bf16", B=4, H=10, S=9248, D=128, bs=64, lb=4, K=16,
          n_pages=32, page_tokens=273, off_std=0.2)
C4 = dict(name="config4_longdoc_prefill_bf16", B=8, H=16, S=131072, D=128, bs=128, lb=8, K=64,
          n_pages=480, page_tokens=273, off_std=0.2)
C3 = dict(name="config3_decode_bf16", R=64, H=10, S=27556, D=128, bs=64, lb=4, K=32)
# the config-2 inputs under the checkpoint's own DASH settings (config.json:
# sparse_block_size 32, sparse_local_block 4, dash_topk_blocks 12; the serving
# router's entmax window of 16, WHL dash_router.py:16)
C2_BS32 = dict(C2, name="config2_prefill_bf16_block32", bs=32, lb=4, K=12, topm=16)
IDX_SCALE = 128.0 / math.sqrt(128)
IMAGE_TOKEN_ID, PAGE_TOKEN_ID = 128815, 128827   # config.json:156,160


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(prefix=f"dash_clocks_gpu{self.gpu}_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f.read().splitlines()[1:]:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1].split()[0]))
                    mx = float(parts[2].split()[0])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def page_cpu_baseline(cfg, threads=None):
    """Reference candidate-domain path (page ids + per-query same-page block
    mask, the numpy restatement in oracle/page_oracle.py) for one sequence."""
    import numpy as np
    from oracle import page_oracle as PO
    ids = document_ids_np(cfg, 0)[:1]
    S, bs = cfg["S"], cfg["bs"]
    nblk = -(-S // bs)
    t0 = time.perf_counter()
    itm, ipi, qpi, _, _ = PO.page_aware_ids(ids, IMAGE_TOKEN_ID, PAGE_TOKEN_ID,
                                            cfg["page_tokens"], S, True)
    PO.kl_candidate_mask(np.arange(S)[None], nblk, itm, bs, True, ipi, qpi)
    dt = time.perf_counter() - t0
    return dict(value=S / dt, unit="tokens/s", cores=1, kind="port",
                sample=f"1 sequence x {S} query tokens of {cfg['name']} (page ids + same-page "
                       f"candidate mask), oracle/page_oracle.py", seconds=dt)


def run_c5(dev, decode_steps, warmup):
    """the 12-layer decoder of ananta_ocr_b200/e2e_decoder.py
    (random init, bf16), a prefill of 8 x 27,556 tokens of visual embeddings
    ~N(0, 0.02) whose token ids lay out a 100-page document (page marker + 272
    image tokens per page, then 256 text tokens), routed with page-aware
    candidates as the model's ``image_bucket_constraint`` asks, then
    ``decode_steps`` greedy decode steps replayed from a CUDA graph.  Device
    time with CUDA events."""
    import torch
    from ananta_ocr_b200.e2e_decoder import DashDecoder, DecoderConfig
    cfg = DecoderConfig()
    B, S = 8, 27556
    doc = dict(B=B, S=S, n_pages=100, page_tokens=273)
    page_cfg = dict(image_token_id=IMAGE_TOKEN_ID, page_token_id=PAGE_TOKEN_ID,
                    per_page_image_tokens=doc["page_tokens"])
    dec = DashDecoder(cfg, B, S + decode_steps + warmup + 4, dev, seed=0, page_cfg=page_cfg)
    g = torch.Generator(device=dev).manual_seed(1)
    emb = (torch.randn(B, S, cfg.hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    ids = document_ids(doc, dev, 2)
    dec.prefill(emb, token_ids=ids)        # warm-up (the timed prefill rewrites the caches)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(cfg.layers)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    logits = dec.prefill(emb, attn_events=ev, token_ids=ids)
    e1.record()
    torch.cuda.synchronize()
    t_prefill = e0.elapsed_time(e1)
    t_attn = sum(a.elapsed_time(b) for a, b in ev)
    dec.tok.copy_(logits.argmax(-1))
    for _ in range(warmup):
        dec.decode_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            dec.decode_step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(decode_steps):
        graph.replay()
    d1.record()
    torch.cuda.synchronize()
    t_dec = d0.elapsed_time(d1) / decode_steps
    ok = bool(torch.isfinite(logits).all())
    del graph
    return dict(B=B, S=S, prefill_ms=t_prefill, attn_ms=t_attn, decode_ms=t_dec,
                decode_steps=decode_steps, finite=ok)


def c5_summary(r):
    """The config-5 figures of ``run_c5`` as a JSON object."""
    from ananta_ocr_b200.e2e_decoder import DecoderConfig
    c = DecoderConfig()
    return {
        "config": {"workload": "config5_e2e_decoder", "layers": c.layers, "hidden": c.hidden,
                   "heads": c.heads, "experts": "64 routed top-6 + 2 shared", "batch": r["B"],
                   "prompt_tokens": r["S"], "decode_steps": r["decode_steps"],
                   "block_size": c.block_size, "local_blocks": c.local_blocks, "routed_k": c.K,
                   "entmax_window": c.topm,
                   "document": "100 pages x (marker + 272 image tokens) + 256 text",
                   "candidates": "page-aware (PageIsolationState, once per forward)",
                   "weights": "random init (the checkpoint is absent)"},
        "prefill": {"ms": r["prefill_ms"], "tokens_per_s": r["B"] * r["S"] / (r["prefill_ms"] / 1e3),
                    "attention_ms": r["attn_ms"],
                    "attention_fraction": r["attn_ms"] / r["prefill_ms"],
                    "attention_scope": "per layer: RoPE + K/V store, index front end, "
                                       "k-bar, routing, paged attention; page state "
                                       "once per forward outside the layer events"},
        "decode": {"ms_per_step": r["decode_ms"], "tokens_per_s": r["B"] / (r["decode_ms"] / 1e3),
                   "graph": f"one CUDA graph per step, {r['decode_steps']} replays"},
        "finite_logits": r["finite"]}


# ---------------------------------------------------------------------------
# synthetic OCR documents: pages of [<PAGE>] + image tokens, then a text tail
# carrying two response-page markers
# ---------------------------------------------------------------------------
def _doc_layout(cfg):
    P, pt, S = cfg["n_pages"], cfg["page_tokens"], cfg["S"]
    tail = P * pt
    return P, pt, S, [tail + o for o in (64, 256) if tail + o < S]


def document_ids(cfg, dev, seed):
    import torch
    P, pt, S, marks = _doc_layout(cfg)
    g = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(0, 100_000, (cfg["B"], S), generator=g, device=dev)
    for p in range(P):
        a = p * pt
        if a >= S:
            break
        ids[:, a] = PAGE_TOKEN_ID
        ids[:, a + 1:min(S, a + pt)] = IMAGE_TOKEN_ID
    for m in marks:
        ids[:, m] = PAGE_TOKEN_ID
    return ids


def document_ids_np(cfg, seed):
    import numpy as np
    P, pt, S, marks = _doc_layout(cfg)
    ids = np.random.default_rng(seed).integers(0, 100_000, (cfg["B"], S))
    for p in range(P):
        a = p * pt
        if a >= S:
            break
        ids[:, a] = PAGE_TOKEN_ID
        ids[:, a + 1:min(S, a + pt)] = IMAGE_TOKEN_ID
    for m in marks:
        ids[:, m] = PAGE_TOKEN_ID
    return ids


def run_page_aware(cfg, st, dev, steps, warmup):
    """Page-aware routing of the prefill workload (every query on its own
    page): the page-id pass, the router with the compact domain, the router
    without candidates, and the dense-mask alternative, each timed alone."""
    import torch
    from ananta_ocr_b200 import ops, pages
    from ananta_ocr_b200 import modeling_deepseekv2 as MD
    B, S, bs, lb, K = (cfg[x] for x in ("B", "S", "bs", "lb", "K"))
    nblk = -(-S // bs)
    ids = document_ids(cfg, dev, 99)
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    oi = torch.empty(B * S, K, dtype=torch.int32, device=dev)
    ob = torch.empty(B * S, K, dtype=torch.float32, device=dev)
    kw = dict(width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE, prior_floor=1e-4,
              sigma=1.0, topm=K, K=K, idx_q=st["iq"].view(B * S, 128), kbar=st["ws"]["kbar"],
              out_idx=oi, out_bias=ob)

    def ids_fn():
        return MD.page_domain_from_ids(ids, image_token_id=IMAGE_TOKEN_ID,
                                       page_token_id=PAGE_TOKEN_ID, per_page=cfg["page_tokens"],
                                       block_size=bs, nblk=nblk, page_scope_prefill=True)
    dom = ids_fn()
    cand = pages.page_allow(dom.q_page, dom.lo, dom.hi, bits=dom.bits, width=nblk, rows=B * S,
                            rows_per_seq=S, fallback=True)
    fns = {
        "page_ids": ids_fn,
        "route_page": lambda: ops.route(seqs, page=dom, **kw),
        "route_plain": lambda: ops.route(seqs, **kw),
        "dense_mask": lambda: pages.page_allow(dom.q_page, dom.lo, dom.hi, bits=dom.bits,
                                               width=nblk, rows=B * S, rows_per_seq=S,
                                               fallback=True, out=cand),
        "route_dense": lambda: ops.route(seqs, cand=cand, **kw),
    }
    res = {}
    for name, fn in fns.items():
        # replayed from a CUDA graph so the figure is device time, not the
        # host's launch cost
        for _ in range(max(3, warmup)):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / steps
        del graph
    # the routes the page domain gives are those of the dense mask
    ops.route(seqs, page=dom, **kw)
    i1, b1 = oi.clone(), ob.clone()
    ops.route(seqs, cand=cand, **kw)
    same = bool(torch.equal(i1, oi) and torch.equal(b1, ob))
    constrained = int((dom.q_page >= 0).sum())
    words = dom.bits.shape[-1]
    ids_bytes = B * S * (8 + 4) + B * nblk * (8 + 4 * words) + 16 * B
    return dict(ms=res, equal_to_dense=same, rows=B * S, rows_with_page=constrained,
                page_ids_bytes=ids_bytes)


def run_backward(cfg, dev, steps, warmup):
    """Training backward of the prefill workload's attention (``dash_attn_bwd``:
    dq + slot-bias gradient, dk/dv) on config-2 shapes: bf16 q, k, v ~N(0,1)*0.5,
    dout ~N(0,1), o and lse from the tcgen05 forward, K distinct remote blocks
    per row drawn uniformly (noise-driven routes).  Inputs (q, k, v, o, dout:
    ~470 MB) exceed L2.  Algorithmic FLOPs: 10 * D per kept (row, head, key):
    the five products s, dp, dq, dk, dv."""
    import torch
    from ananta_ocr_b200 import ops
    B, S, H, D, bs, LW, K = cfg["B"], cfg["S"], cfg["H"], 128, cfg["bs"], cfg["lb"] * cfg["bs"], cfg["K"]
    g = torch.Generator(device=dev).manual_seed(321)
    q = (torch.randn(B, S, H, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, S, H, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, S, H, D, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    do = torch.randn(B, S, H, D, generator=g, device=dev).to(torch.bfloat16)
    t = torch.arange(S, device=dev)
    nrem = torch.clamp((t - LW + 1 + bs - 1) // bs, min=0)            # blocks with a remote key
    r = torch.rand(B, S, (S + bs - 1) // bs, generator=g, device=dev)
    r = r.masked_fill(torch.arange(r.shape[-1], device=dev)[None, None] >= nrem[None, :, None], 2.0)
    idx = r.argsort(-1)[..., :K].to(torch.int32)
    idx = torch.where(torch.arange(K, device=dev)[None, None] < nrem[None, :, None], idx,
                      torch.full_like(idx, -1)).sort(-1).values
    bias = torch.randn(B, S, K, generator=g, device=dev) * 0.5
    lse = torch.empty(B, H, S, device=dev)
    o = ops.gather_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), idx[:, None],
                             bias[:, None], block_size=bs, local_window=LW, scale=1 / math.sqrt(D),
                             lse=lse).transpose(1, 2).contiguous()
    lse_t = lse.transpose(1, 2).contiguous()

    def step():
        return ops.gather_attention_bwd(q, k, v, o, do, lse_t, idx, bias, block_size=bs,
                                        local_window=LW, scale=1 / math.sqrt(D))
    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(max(1, steps)):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    # kept keys per (row, head): window min(LW, t+1) + routed blocks' keys below it
    valid = idx >= 0
    blk_keys = torch.clamp(torch.minimum((idx.long() + 1) * bs, (t - LW + 1)[None, :, None])
                           - idx.long() * bs, min=0) * valid
    keys = blk_keys.sum(-1).float() + torch.clamp(t + 1, max=LW)[None].float()
    flops = 10.0 * D * H * float(keys.sum())
    return dict(ms=statistics.median(times), flops=flops, tokens=B * S)


def run_frontend(cfg, dev, steps, warmup):
    """Router front end of the prefill workload: index projections (hidden
    1280 -> 2 x 128) + RMSNorm + RoPE for every token, one tcgen05 kernel,
    against the same computation as PyTorch ops (cuBLAS GEMMs + elementwise).
    Device time of CUDA-graph replays; L2 is flushed before every timed
    replay (the 95 MB hidden input would otherwise stay in the 126 MB L2)."""
    import torch
    from ananta_ocr_b200 import ops
    T, Hd, d = cfg["B"] * cfg["S"], 1280, 128
    g = torch.Generator(device=dev).manual_seed(123)
    h = torch.randn(T, Hd, generator=g, device=dev).to(torch.bfloat16)
    wq = (torch.randn(d, Hd, generator=g, device=dev) / math.sqrt(Hd)).to(torch.bfloat16)
    wk = (torch.randn(d, Hd, generator=g, device=dev) / math.sqrt(Hd)).to(torch.bfloat16)
    nq = torch.randn(d, generator=g, device=dev) * 0.1
    nk = torch.randn(d, generator=g, device=dev) * 0.1
    pos = torch.arange(T, device=dev, dtype=torch.float32)[:, None] % cfg["S"]
    inv = 1.0 / (10000.0 ** (torch.arange(0, d // 2, device=dev).float() / (d // 2)))
    emb = torch.cat([pos * inv, pos * inv], -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    iq = torch.empty(T, d, device=dev)
    ik = torch.empty(T, d, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def ours():
        ops.index_proj(h, wq, wk, nq, nk, 1e-6, cos=cos, sin=sin, idx_q=iq, idx_k=ik)

    def torch_path():
        hq = torch.nn.functional.linear(h, wq)
        hk = torch.nn.functional.linear(h, wk)
        outs = []
        for x, w in ((hq, nq), (hk, nk)):
            x32 = x.float()
            x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + 1e-6)
            y = (x32 * (1.0 + w)).to(torch.bfloat16)
            rot = torch.cat((-y[:, d // 2:], y[:, :d // 2]), -1)
            outs.append((y * cos + rot * sin).float())
        return outs

    res = {}
    for name, fn in (("index_proj", ours), ("torch_ops", torch_path)):
        for _ in range(max(3, warmup)):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        times = []
        for i in range(3 + steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            if i >= 3:
                times.append(e0.elapsed_time(e1))
        res[name] = statistics.median(times)
        del graph
    nbytes = T * Hd * 2 + 2 * d * Hd * 2 + 2 * T * d * 4 + 2 * T * d * 2
    flops = 2.0 * T * Hd * 2 * d
    return dict(ms=res, tokens=T, bytes=nbytes, flops=flops)


# ---------------------------------------------------------------------------
# workload construction (device-side, seeded)
# ---------------------------------------------------------------------------
def make_prefill(cfg, dev, seed):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    B, H, S, D = cfg["B"], cfg["H"], cfg["S"], cfg["D"]
    P, pt = cfg["n_pages"], cfg["page_tokens"]

    def offsets(heads, dim):
        off = torch.zeros(heads, S, dim, device=dev)
        for p in range(P):
            a, b = p * pt, min(S, (p + 1) * pt)
            if a >= S:
                break
            off[:, a:b] = torch.randn(heads, 1, dim, generator=g, device=dev) * cfg["off_std"]
        return off

    q = torch.empty(B, H, S, D, device=dev, dtype=torch.bfloat16)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    iq = torch.empty(B, S, 128, device=dev)
    ik = torch.empty(B, S, 128, device=dev)
    for b in range(B):
        off = offsets(H, D)
        q[b] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5 + off).bfloat16()
        k[b] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5 + off).bfloat16()
        v[b] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5).bfloat16()
        ioff = offsets(1, 128)[0]
        iq[b] = torch.randn(S, 128, generator=g, device=dev) * 0.5 + ioff
        ik[b] = torch.randn(S, 128, generator=g, device=dev) * 0.5 + ioff
    return q, k, v, iq, ik


def make_prefill_seqs(cfg, dev, seqs, seed):
    """Sequences ``seqs`` of a prefill workload, each from its own seeded
    generator, so a rank holding any subset draws what one GPU holding all
    would (the strong-scaling runs compare like with like)."""
    import torch
    H, S, D = cfg["H"], cfg["S"], cfg["D"]
    P, pt = cfg["n_pages"], cfg["page_tokens"]
    n = len(seqs)
    q = torch.empty(n, H, S, D, device=dev, dtype=torch.bfloat16)
    k, v = torch.empty_like(q), torch.empty_like(q)
    iq = torch.empty(n, S, 128, device=dev)
    ik = torch.empty(n, S, 128, device=dev)
    for j, b in enumerate(seqs):
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + b)
        off = torch.zeros(H, S, D, device=dev)
        ioff = torch.zeros(S, 128, device=dev)
        pages = torch.randn(P, H, 1, D, generator=g, device=dev) * cfg["off_std"]
        ipages = torch.randn(P, 128, generator=g, device=dev) * cfg["off_std"]
        for p in range(P):
            a0, a1 = p * pt, min(S, (p + 1) * pt)
            if a0 >= S:
                break
            off[:, a0:a1] = pages[p]
            ioff[a0:a1] = ipages[p]
        q[j] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5 + off).bfloat16()
        k[j] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5 + off).bfloat16()
        v[j] = (torch.randn(H, S, D, generator=g, device=dev) * 0.5).bfloat16()
        iq[j] = torch.randn(S, 128, generator=g, device=dev) * 0.5 + ioff
        ik[j] = torch.randn(S, 128, generator=g, device=dev) * 0.5 + ioff
    return q, k, v, iq, ik


def run_c4(dev, rank, world, steps, warmup, mode):
    """BASELINE config 4 (B=8 long documents of 131,072 tokens, 16 heads, block
    128, window 8 blocks, K=64) split over the ranks by sequence x kv head
    (sharding.plan_shards): every rank routes and attends its shard, and the
    step ends with the whole output on every rank (``mode`` "fused": gather in
    the attention kernel; "nccl": in-place NCCL all-gather after it).  Strong
    scaling: the total work is fixed.  Device time per step, max over ranks."""
    import torch
    import torch.distributed as dist
    from ananta_ocr_b200 import ops
    from ananta_ocr_b200.sharding import plan_shards
    cfg = C4
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    sh = plan_shards(B, H, world)[rank]
    nb = sh.b1 - sh.b0
    q, k, v, iq, ik = make_prefill_seqs(cfg, dev, list(range(sh.b0, sh.b1)), 4)
    if sh.h1 - sh.h0 < H:
        q, k, v = (t[:, sh.h0:sh.h1].contiguous() for t in (q, k, v))
    full = torch.empty(B, H, S, D, dtype=torch.bfloat16, device=dev)
    out = full[sh.b0:sh.b1, sh.h0:sh.h1]
    gather = None
    if world > 1 and mode == "fused":
        from ananta_ocr_b200.peer import PeerGather
        gather = PeerGather(full)
    peers = gather.peers_for(out) if gather is not None else None
    nblk = -(-S // bs)
    lcfg = dict(cfg, B=nb, H=sh.h1 - sh.h0)
    ws = dict(kbar=torch.empty(nb, nblk, 128, device=dev),
              idx=torch.empty(nb * S, K, dtype=torch.int32, device=dev),
              bias=torch.empty(nb * S, K, device=dev),
              attn_ws=torch.empty(_prefill_ws_bytes(lcfg), dtype=torch.uint8, device=dev))
    seqs = ops.Seqs(n_seq=nb, q_len=S, kv_len=S, max_q_len=S)

    def route_fn():
        kb = ops.kbar_pool_contig(ik, None, bs, out=ws["kbar"])
        ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                  prior_floor=1e-4, sigma=1.0, topm=K, K=K, idx_q=iq.view(nb * S, 128), kbar=kb,
                  out_idx=ws["idx"], out_bias=ws["bias"])

    def attn_fn():
        ops.gather_attention(q, k, v, ws["idx"].view(nb, S, K), ws["bias"].view(nb, S, K),
                             block_size=bs, local_window=lb * bs, scale=1.0 / math.sqrt(D),
                             out=out, workspace=ws["attn_ws"], peers=peers)

    post = None
    if gather is not None:
        post = gather.complete
    elif world > 1 and mode == "nccl":
        assert sh.h1 - sh.h0 == H, "the NCCL form gathers whole sequences"
        post = lambda: dist.all_gather_into_tensor(full.view(-1), out.reshape(-1))  # noqa: E731
    step = GraphStep(route_fn, attn_fn, True, post=post)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(ev[i])
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps,
                      statistics.mean(e[1].elapsed_time(e[2]) for e in ev)], device=dev,
                     dtype=torch.float64)
    alg, executed = prefill_flops(lcfg, ws["idx"])
    fl = torch.tensor([alg, executed], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(fl)
    if gather is not None:
        gather.close()
    del step
    return dict(ms=float(t[0]), attn_gather_ms=float(t[1]), alg=float(fl[0]),
                executed=float(fl[1]), tokens=B * S, shard=(sh.b0, sh.b1, sh.h0, sh.h1))


def c4_gathered():
    """Whether the library's automatic prefill split takes the gathered form
    at config 4 (blocks of 128 tokens with K >= 32, or ``--prefill-mode 2``)."""
    from ananta_ocr_b200 import ops as _ops
    mode = _ops.PREFILL_MODE
    return mode == 2 or (mode == 0 and C4["bs"] >= 128 and C4["K"] >= 32)


def c4_summary(r, world, gather, peaks, peak_kind):
    """The config-4 figures of ``run_c4`` as a JSON object."""
    peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    gathered = c4_gathered()
    tf = r["alg"] / (r["ms"] / 1e3) / 1e12
    return {
        "workload": C4["name"], "scaling": "strong", "n_gpus": world,
        "sequences": C4["B"], "seq_len": C4["S"], "heads": C4["H"], "block_size": C4["bs"],
        "local_blocks": C4["lb"], "routed_k": C4["K"],
        "split": "sequence x kv head (sharding.plan_shards); this run's rank-0 shard "
                 f"seqs {r['shard'][0]}:{r['shard'][1]} heads {r['shard'][2]}:{r['shard'][3]}",
        "output_gather_in_step": ("none (one GPU)" if world == 1 else
                                  "fused into the attention kernel + NCCL completion word"
                                  if gather != "nccl" else "in-place NCCL all-gather"),
        "ms_per_step": r["ms"], "tokens_per_s": r["tokens"] / (r["ms"] / 1e3),
        "attn_and_gather_ms": r["attn_gather_ms"],
        "prefill_split": ("routed keys gathered by key block (prefill_routed_kernel + "
                          "prefill_merge_kernel; window part tile-major)" if gathered else
                          "tile-major (each 128-row tile runs the union of its rows' blocks)"),
        "alg_tflops": tf,
        "executed_tflops": None if gathered else r["executed"] / (r["ms"] / 1e3) / 1e12,
        "alg_flops_per_step": r["alg"], "executed_flops_per_step": None if gathered else r["executed"],
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak * world, "unit": "TFLOP/s",
                     "frac": tf / (peak * world),
                     "kernel": "whole step (routing + prefill_kernel + gather), algorithmic FLOPs, "
                               "all GPUs", "peak_source": f"{peak_kind} bf16_tflops x {world}"},
        "steps": 3, "warmup": 3}


def prefill_step(cfg, q, k, v, iq, ik, ws, timers=None):
    """One DASH prefill step through the public API; returns (out, idx, bias)."""
    from ananta_ocr_b200 import ops
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    nblk = (S + bs - 1) // bs
    if timers:
        timers[0].record()
    kbar = ops.kbar_pool_contig(ik, None, bs, out=ws["kbar"])
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    idx, bias = ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                          prior_floor=1e-4, sigma=1.0, topm=K, K=K, idx_q=iq.view(B * S, 128),
                          kbar=kbar, out_idx=ws["idx"], out_bias=ws["bias"])
    if timers:
        timers[1].record()
    out = ops.gather_attention(q, k, v, idx.view(B, S, K), bias.view(B, S, K), block_size=bs,
                               local_window=lb * bs, scale=1.0 / math.sqrt(D), out=ws["out"],
                               workspace=ws["attn_ws"])
    if timers:
        timers[2].record()
    return out, idx, bias


def prefill_flops(cfg, idx):
    """Algorithmic FLOPs = 4*D*H*sum_t |keys(t)| from the routed lists, and the
    FLOPs the union-tile kernel executes (tiles x key tiles x 128x64x128x4)."""
    import torch
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    LW = lb * bs
    t = torch.arange(S, device=idx.device)
    local = torch.clamp(t + 1, max=LW).double()
    ids = idx.view(B, S, K).long()
    valid = ids >= 0
    lstart = (t - LW + 1)[None, :, None]
    start = ids * bs
    end = torch.minimum((ids + 1) * bs, lstart.expand_as(ids))
    rem = torch.clamp(end - start, min=0, max=bs).masked_fill(~valid, 0).double().sum(-1)
    keys = (local[None] + rem).sum()
    alg = 4.0 * D * H * float(keys)
    nblk = (S + bs - 1) // bs
    sel = torch.zeros(B, S, nblk + 1, dtype=torch.bool, device=idx.device)
    sel.scatter_(2, ids.clamp(min=0).masked_fill(~valid, nblk), True)
    sel = sel[..., :nblk]
    ntile = (S + 127) // 128
    pad = ntile * 128 - S
    if pad:
        sel = torch.cat([sel, torch.zeros(B, pad, nblk, dtype=torch.bool, device=idx.device)], 1)
    uni = sel.view(B, ntile, 128, nblk).any(2)
    tiles = torch.arange(ntile, device=idx.device)
    pmin, pmax = tiles * 128, torch.clamp(tiles * 128 + 127, max=S - 1)
    blk = torch.arange(nblk, device=idx.device)
    loc = (blk[None] >= torch.clamp((pmin[:, None] - LW + 1), min=0) // bs) & (blk[None] <= pmax[:, None] // bs)
    walked = uni | loc[None]
    if bs >= 64:
        ktiles = walked.sum() * (bs // 64)
    else:
        # 64-key tiles of two 32-token blocks: walked when either block is
        walked = torch.nn.functional.pad(walked, (0, nblk % 2))
        ktiles = walked.view(B, ntile, -1, 2).any(-1).sum()
    executed = float(ktiles) * H * 128 * 64 * D * 4
    return alg, executed


class GraphStep:
    """A step as two CUDA graphs (route part, attention part) replayed back to
    back on the current stream, with CUDA events between them."""

    def __init__(self, route_fn, attn_fn, use_graph=True, post=None):
        import torch
        self.route_fn, self.attn_fn, self.post = route_fn, attn_fn, post
        self.graphs = None
        if use_graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):          # warm the capture stream
                route_fn()
                attn_fn()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1):
                route_fn()
            with torch.cuda.graph(g2):
                attn_fn()
            self.graphs = (g1, g2)

    def __call__(self, timers=None):
        if timers:
            timers[0].record()
        self.graphs[0].replay() if self.graphs else self.route_fn()
        if timers:
            timers[1].record()
        self.graphs[1].replay() if self.graphs else self.attn_fn()
        if self.post is not None:
            self.post()          # stream-ordered, outside the graphs (an NCCL call)
        if timers:
            timers[2].record()


def run_prefill(cfg, dev, steps, warmup, rank, world, use_graph=True, gather=None):
    """The headline step on this rank's B sequences.  With ``gather`` (a
    ``peer.PeerGather`` over [world * B, H, S, D]) the attention also stores
    every output row into the other ranks' gathered tensors (the fused output
    gather) and the step ends with its stream-ordered completion."""
    import torch
    from ananta_ocr_b200 import ops
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    nblk = (S + bs - 1) // bs
    q, k, v, iq, ik = make_prefill(cfg, dev, 1234 + rank)
    out = gather.full[rank * B:(rank + 1) * B] if gather is not None else torch.empty_like(q)
    peers = gather.peers_for(out) if gather is not None else None
    ws = dict(kbar=torch.empty(B, nblk, 128, device=dev),
              idx=torch.empty(B * S, K, dtype=torch.int32, device=dev),
              bias=torch.empty(B * S, K, device=dev), out=out,
              attn_ws=torch.empty(_prefill_ws_bytes(cfg), dtype=torch.uint8, device=dev))
    out, idx, bias = prefill_step(cfg, q, k, v, iq, ik, ws)
    torch.cuda.synchronize()
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)

    def route_fn():
        kb = ops.kbar_pool_contig(ik, None, bs, out=ws["kbar"])
        ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                  prior_floor=1e-4, sigma=1.0, topm=cfg.get("topm", K), K=K,
                  idx_q=iq.view(B * S, 128), kbar=kb, out_idx=ws["idx"], out_bias=ws["bias"])

    def attn_fn():
        ops.gather_attention(q, k, v, ws["idx"].view(B, S, K), ws["bias"].view(B, S, K),
                             block_size=bs, local_window=lb * bs, scale=1.0 / math.sqrt(D),
                             out=ws["out"], workspace=ws["attn_ws"], peers=peers)

    step = GraphStep(route_fn, attn_fn, use_graph,
                     post=gather.complete if gather is not None else None)
    for _ in range(max(0, warmup - 1)):
        step()
    torch.cuda.synchronize()
    alg, executed = prefill_flops(cfg, idx)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    return dict(q=q, k=k, v=v, iq=iq, ik=ik, ws=ws, ev=ev, start=start, stop=stop, alg=alg,
                executed=executed, idx=idx, step=step)


def run_prefill_on(cfg, st, dev, steps, warmup):
    """The headline's prefill inputs (``st``) routed and attended under another
    DASH configuration ``cfg`` (block size, window, K): k-bar + routing and the
    attention replayed from CUDA graphs, device time per part with CUDA events."""
    import torch
    from ananta_ocr_b200 import ops
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    nblk = (S + bs - 1) // bs
    q, k, v, iq, ik = (st[x] for x in ("q", "k", "v", "iq", "ik"))
    ws = dict(kbar=torch.empty(B, nblk, 128, device=dev),
              idx=torch.empty(B * S, K, dtype=torch.int32, device=dev),
              bias=torch.empty(B * S, K, device=dev), out=torch.empty_like(q))
    seqs = ops.Seqs(n_seq=B, q_len=S, kv_len=S, max_q_len=S)
    # the attention scratch is sized once here, outside the graph capture
    attn_ws = torch.empty(_prefill_ws_bytes(cfg), dtype=torch.uint8, device=dev)

    def route_fn():
        kb = ops.kbar_pool_contig(ik, None, bs, out=ws["kbar"])
        ops.route(seqs, width=nblk, block_size=bs, local_blocks=lb, idx_scale=IDX_SCALE,
                  prior_floor=1e-4, sigma=1.0, topm=cfg.get("topm", K), K=K,
                  idx_q=iq.view(B * S, 128), kbar=kb, out_idx=ws["idx"], out_bias=ws["bias"])

    def attn_fn():
        ops.gather_attention(q, k, v, ws["idx"].view(B, S, K), ws["bias"].view(B, S, K),
                             block_size=bs, local_window=lb * bs, scale=1.0 / math.sqrt(D),
                             out=ws["out"], workspace=attn_ws)

    route_fn()
    step = GraphStep(route_fn, attn_fn)
    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        step(ev[i])
    torch.cuda.synchronize()
    route_ms = statistics.median(e[0].elapsed_time(e[1]) for e in ev)
    attn_ms = statistics.median(e[1].elapsed_time(e[2]) for e in ev)
    alg, executed = prefill_flops(cfg, ws["idx"])
    return dict(route_ms=route_ms, attn_ms=attn_ms, alg=alg, executed=executed, tokens=B * S)


def _prefill_ws_bytes(cfg):
    """Bytes of attention scratch for a contiguous prefill of ``cfg`` (the
    library's own sizing under the current prefill mode)."""
    from ananta_ocr_b200 import ops
    return ops.gather_attention_workspace_bytes(
        cfg["B"], cfg["H"], cfg.get("Hkv", cfg["H"]), cfg["S"], cfg["K"], block_size=cfg["bs"],
        local_window=cfg["lb"] * cfg["bs"])


def run_decode_setup(cfg, dev, seed):
    import torch
    from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
    R, H, S, D, bs, lb, K = (cfg[x] for x in ("R", "H", "S", "D", "bs", "lb", "K"))
    nb = -(-S // bs)
    P = R * nb + 28
    g = torch.Generator(device=dev).manual_seed(seed)
    kc = (torch.randn(P, bs, H, D, generator=g, device=dev) * 0.5).bfloat16()
    vc = (torch.randn(P, bs, H, D, generator=g, device=dev) * 0.5).bfloat16()
    icache = (torch.randn(P, bs, 128, generator=g, device=dev) * 0.5)
    q = torch.randn(R, H, D, generator=g, device=dev).bfloat16()
    iq = torch.randn(R, 128, generator=g, device=dev) * 0.5
    bt = torch.randperm(P, generator=g, device=dev)[:R * nb].to(torch.int32).view(R, nb).contiguous()
    sl = torch.full((R,), S, dtype=torch.int32, device=dev)
    kbar = torch.zeros(P, 128, device=dev)
    plan = RT.kbar_all_plan(block_table=bt, seq_lens=sl, context_lens=torch.zeros_like(sl),
                            block_size=bs, max_block=nb, max_query_len=S, device=dev)
    RT.kbar_refresh_tail_triton(kv_cache=icache, k_bar=kbar, block_table=bt, seq_lens=sl,
                                head_cls=None, block_size=bs, plan=plan)
    tail = RT.kbar_tail_plan(block_table=bt, seq_lens=sl, block_size=bs, tail_pages=1, device=dev)
    return dict(kc=kc, vc=vc, icache=icache, q=q, iq=iq, bt=bt, sl=sl, kbar=kbar, tail=tail,
                oi=torch.empty(R, K, dtype=torch.int32, device=dev),
                ob=torch.empty(R, K, device=dev),
                out=torch.empty(R, H, D, dtype=torch.bfloat16, device=dev), nb=nb)


def decode_route(cfg, d):
    """k-bar refresh of each sequence's tail page + decode routing, one launch
    (the refresh runs on the routing clusters' idle CTAs)."""
    from ananta_ocr_b200.unlimited_dash_ops import route_triton as RT
    bs, lb, K = cfg["bs"], cfg["lb"], cfg["K"]
    RT.route_decode_triton(idx_q=d["iq"], k_bar=d["kbar"], block_table=d["bt"], seq_lens=d["sl"],
                           image_allow=None, out_idx=d["oi"], out_bias=d["ob"], max_block=d["nb"],
                           block_size=bs, local_blocks=lb, decode_query_len=1, idx_scale=IDX_SCALE,
                           prior_floor=1e-4, sigma=1.0, topm=K, budget=K, out_slots=K,
                           refresh=(d["icache"], None, d["tail"]))


def decode_attend(cfg, d):
    from ananta_ocr_b200.unlimited_dash_ops.attend_triton import dash_sparse_attn_decode
    H, D, bs, lb = cfg["H"], cfg["D"], cfg["bs"], cfg["lb"]
    dash_sparse_attn_decode(d["q"], d["kc"], d["vc"], d["oi"][None].expand(H, -1, -1),
                            d["ob"][None].expand(H, -1, -1), d["bt"], d["sl"], H, 1.0 / math.sqrt(D),
                            d["out"], 1, local_blocks=lb, sparse_block_size=bs)


def decode_step(cfg, d, timers=None):
    if timers:
        timers[0].record()
    decode_route(cfg, d)
    if timers:
        timers[1].record()
    decode_attend(cfg, d)
    if timers:
        timers[2].record()


def decode_bytes(cfg, d):
    """Algorithmic bytes of one decode step: K+V of every attended key, k-bar
    rows scored, q and out, routed lists, block-table rows."""
    import torch
    R, H, S, D, bs, lb, K = (cfg[x] for x in ("R", "H", "S", "D", "bs", "lb", "K"))
    LW = lb * bs
    pos = S - 1
    ids = d["oi"].long()
    valid = ids >= 0
    lstart = pos - LW + 1
    rem = torch.clamp(torch.clamp((ids + 1) * bs, max=lstart) - ids * bs, min=0, max=bs)
    keys = float(rem.masked_fill(~valid, 0).sum()) + R * min(S, LW)
    kv = keys * H * D * 2 * 2
    nb_remote = max(0, pos // bs - lb + 1)
    other = R * nb_remote * 128 * 4 + R * H * D * 2 * 2 + R * K * 8 + R * d["nb"] * 4
    return kv + other, kv


# ---------------------------------------------------------------------------
# CPU baseline (oracle port) on a bounded sample
# ---------------------------------------------------------------------------
def cpu_baseline(cfg, n_tokens=1024, threads=None):
    """The reference's CPU inference path in its own arithmetic (fp32 torch:
    head_cls k-bar of every block, scores and canonical selection of the sampled
    query rows, dense masked attention of those rows over all keys, chunked by
    512 queries; oracle/torch_path.py, checked against the reference's outputs)
    on one sequence of the workload, all host threads.  Every query row of the
    dense form costs the same (all keys, masked), so the sample's tokens/s is
    the workload's."""
    import numpy as np
    import torch
    from oracle import dash_oracle as O
    from oracle import torch_path as TP
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    B, H, S, D, bs, lb, K = (cfg[x] for x in ("B", "H", "S", "D", "bs", "lb", "K"))
    q, k, v, iq, ik = (torch.from_numpy(x) for x in O.make_prefill_inputs(
        99, 1, H, S, D, cfg["n_pages"], cfg["page_tokens"], cfg["off_std"]))
    q, k, v = (t.to(torch.bfloat16).float() for t in (q, k, v))
    rows = torch.from_numpy(np.sort(np.random.default_rng(0).choice(S, size=n_tokens,
                                                                     replace=False)))
    t0 = time.perf_counter()
    with torch.no_grad():
        TP.prefill_rows(q, k, v, iq, ik, rows, block_size=bs, local_blocks=lb, K=K,
                        topm=cfg.get("topm", K), idx_scale=IDX_SCALE)
    dt = time.perf_counter() - t0
    return dict(value=n_tokens / dt, unit="tokens/s", cores=threads, kind="port",
                sample=f"{n_tokens} query tokens x {H} heads of one {S}-token sequence of "
                       f"{cfg['name']}: k-bar of all blocks, scores + selection + dense masked "
                       f"fp32 attention of the sampled tokens (the reference's torch CPU form, "
                       f"oracle/torch_path.py), {threads} threads",
                seconds=dt, dtype="fp32")


# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "c4", "c5", "bwd"],
                    help="c2 (default, the headline), c4 long-document prefill, c5 end-to-end decoder, "
                         "bwd the config-2 training backward alone")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-pages", action="store_true",
                    help="skip the page-aware routing measurement")
    ap.add_argument("--no-backward", action="store_true",
                    help="skip the training-backward measurement")
    ap.add_argument("--no-frontend", action="store_true",
                    help="skip the router front-end measurement")
    ap.add_argument("--no-c4", action="store_true",
                    help="skip the long-document (config 4) strong-scaling sub-object")
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the end-to-end decoder (config 5) sub-object")
    ap.add_argument("--no-block32", action="store_true",
                    help="skip the prefill under the checkpoint's 32-token blocks")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl", "none"],
                    help="output gather at N > 1 inside the timed step: fused into the attention "
                         "kernel (default), an NCCL all-gather after it, or none")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch eagerly instead of replaying captured CUDA graphs")
    ap.add_argument("--decode-rows", type=int, default=0,
                    help="decode batch override (small cases for profiler captures)")
    ap.add_argument("--c4-seqs", type=int, default=0,
                    help="config-4 sequence count override (small cases for profiler captures)")
    ap.add_argument("--c4-len", type=int, default=0,
                    help="config-4 sequence length override (small cases for profiler captures)")
    ap.add_argument("--prefill-mode", type=int, default=0, choices=[0, 1, 2],
                    help="prefill work split: 0 automatic, 1 tile-major, 2 routed part gathered "
                         "by key block")
    args = ap.parse_args()
    cfg = C2 if args.workload == "c2" else C4
    if args.decode_rows > 0:
        C3["R"] = args.decode_rows
    if args.c4_seqs > 0:
        C4["B"] = args.c4_seqs
    if args.c4_len > 0:
        C4["S"] = args.c4_len
        C4["n_pages"] = max(1, args.c4_len // C4["page_tokens"])
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        ms = []
        res = None
        n_tok = 1024
        for i in range(args.warmup + args.steps):
            r = cpu_baseline(cfg, n_tokens=n_tok)
            if i >= args.warmup:
                ms.append(r["seconds"])
                res = r
        val = n_tok / statistics.median(ms)
        line = {"metric": "DASH attn tokens/s", "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(ms) * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
                "data": "synthetic", "impl": "reference",
                "config": {"workload": cfg["name"], "sample_tokens": n_tok},
                "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": res["cores"],
                                 "kind": "port", "sample": res["sample"]},
                "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        # NCCL may print a banner on stdout when its communicator is created;
        # keep stdout for the one JSON line by sending it to stderr meanwhile
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_fd, 1)
            os.close(saved_fd)
    from ananta_ocr_b200 import _lib, ops as _ops
    _lib.load()
    _ops.PREFILL_MODE = args.prefill_mode

    if args.workload == "c4":
        # config 4 alone: strong scaling over the ranks, gather inside the step
        clocks = ClockSampler(local_rank)
        clocks.start()
        r = run_c4(dev, rank, world, args.steps, max(3, args.warmup),
                   args.gather if args.gather != "none" else "fused")
        clk = clocks.stop()
        if rank == 0:
            peaks, peak_kind = load_peaks()
            sub = c4_summary(r, world, args.gather, peaks, peak_kind)
            print(json.dumps({"metric": "DASH attn tokens/s", "value": sub["tokens_per_s"],
                              "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                              "warmup": max(3, args.warmup), "ms_per_step": r["ms"],
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                              "dtype": "bf16", "data": "synthetic (seeded, BASELINE distributions)",
                              "config": {"workload": C4["name"], "parallelism": f"shard{world}",
                                         "l2": "inputs exceed L2 (126 MB); no flush"},
                              "roofline": sub["roofline"], "c4": sub, "clocks": clk}))
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload == "bwd":
        # the training backward alone (one GPU; ranks other than 0 run nothing)
        if rank != 0:
            return
        r = run_backward(C2, dev, args.steps, args.warmup)
        peaks, peak_kind = load_peaks()
        peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        tf = r["flops"] / (r["ms"] / 1e3) / 1e12
        print(json.dumps({"metric": "DASH attn backward tokens/s", "value": r["tokens"] / (r["ms"] / 1e3),
                          "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": "config2_backward_bf16"},
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": peak,
                                       "unit": "TFLOP/s", "frac": tf / peak,
                                       "peak_source": f"{peak_kind} bf16_tflops"}}))
        return
    if args.workload == "c5":
        # one model per GPU: ranks other than 0 run nothing (replicas only)
        if rank != 0:
            return
        clocks = ClockSampler(local_rank)
        clocks.start()
        r = run_c5(dev, 512, max(3, args.warmup))
        clk = clocks.stop()
        sub = c5_summary(r)
        line = {"metric": "C5 e2e prefill tokens/s", "value": r["B"] * r["S"] / (r["prefill_ms"] / 1e3),
                "unit": "tokens/s", "n_gpus": 1, "steps": 1, "warmup": 1,
                "ms_per_step": r["prefill_ms"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights, visual embeddings ~N(0,0.02))",
                "config": sub["config"], "prefill": sub["prefill"], "decode": sub["decode"],
                "finite_logits": r["finite"], "clocks": clk}
        print(json.dumps(line))
        return

    # the output gather of N > 1 runs inside the timed step: fused into the
    # attention kernel (peer stores over NVLink, then one NCCL completion word),
    # or as an NCCL all-gather after it (--gather nccl)
    gather, full_out = None, None
    if world > 1 and args.gather != "none":
        full_out = torch.empty((world * cfg["B"], cfg["H"], cfg["S"], cfg["D"]),
                               dtype=torch.bfloat16, device=dev)
        if args.gather == "fused":
            from ananta_ocr_b200.peer import PeerGather
            gather = PeerGather(full_out)
    st = run_prefill(cfg, dev, args.steps, args.warmup, rank, world, not args.no_graph,
                     gather=gather)
    if world > 1 and args.gather == "nccl":
        shard = st["ws"]["out"]
        st["step"].post = lambda: dist.all_gather_into_tensor(full_out, shard)
    dec = None
    if not args.no_decode:
        dec = run_decode_setup(C3, dev, 77 + rank)
        decode_step(C3, dec)
        torch.cuda.synchronize()
        dec["step"] = GraphStep(lambda: decode_route(C3, dec), lambda: decode_attend(C3, dec),
                                not args.no_graph)
        for _ in range(args.warmup):
            dec["step"]()
    torch.cuda.synchronize()

    # ---------------- timed prefill steps ----------------
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    st["start"].record()
    for i in range(args.steps):
        st["step"](st["ev"][i])
    st["stop"].record()
    torch.cuda.synchronize()
    # library kernels per step (counted on an eager step: graph replays re-launch
    # the same captured kernels without passing through the library)
    launches0 = _lib.launches()
    st["step"].route_fn()
    st["step"].attn_fn()
    torch.cuda.synchronize()
    launches = (_lib.launches() - launches0) * args.steps
    if world > 1:
        dist.barrier()
    total_ms = st["start"].elapsed_time(st["stop"])
    route_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in st["ev"])
    attn_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in st["ev"])
    # decode steps (same run)
    dec_res = None
    if dec is not None:
        dev_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record()
        for i in range(args.steps):
            dec["step"](dev_ev[i])
        d1.record()
        torch.cuda.synchronize()
        dec_total = d0.elapsed_time(d1) / args.steps
        dec_attn = statistics.mean(e[1].elapsed_time(e[2]) for e in dev_ev)
        dec_route = statistics.mean(e[0].elapsed_time(e[1]) for e in dev_ev)
        nbytes, kv_bytes = decode_bytes(C3, dec)
        dec_res = dict(ms_per_step=dec_total, attn_ms=dec_attn, route_ms=dec_route,
                       bytes_per_step=nbytes, kv_bytes=kv_bytes)
    clk = clocks.stop()

    t_step = total_ms / args.steps
    if world > 1:
        tt = torch.tensor([t_step, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_step, attn_ms = float(tt[0]), float(tt[1])
    tokens_per_rank = cfg["B"] * cfg["S"]
    value = tokens_per_rank * world / (t_step / 1e3)

    # ---------------- reference figure: the same gather as a plain NCCL all-gather ----
    # (timed on its own, outside the step)
    nccl_gather = None
    if world > 1:
        shard = st["ws"]["out"]
        full = torch.empty((world,) + tuple(shard.shape), dtype=shard.dtype, device=dev)
        for _ in range(2):
            dist.all_gather_into_tensor(full, shard)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        dist.all_gather_into_tensor(full, shard)
        g1.record()
        torch.cuda.synchronize()
        gt = torch.tensor([g0.elapsed_time(g1)], device=dev, dtype=torch.float64)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gbytes = full.numel() * full.element_size()
        nccl_gather = {"ms": float(gt[0]), "bytes": gbytes, "bus_gbs": gbytes * (world - 1) / world / float(gt[0]) / 1e6,
                  "op": "all_gather_into_tensor (NCCL)"}
        del full

    # ---------------- e2e through the public API (pinned host buffers) -------------
    e2e = None
    if not args.no_e2e:
        from ananta_ocr_b200 import modeling_deepseekv2 as MD
        hq = st["q"].cpu().pin_memory()
        hk = st["k"].cpu().pin_memory()
        hv = st["v"].cpu().pin_memory()
        hiq = st["iq"].cpu().pin_memory()
        hik = st["ik"].cpu().pin_memory()
        hout = torch.empty(st["q"].shape, dtype=torch.bfloat16).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hiq, hik))
        d2h = hout.numel() * hout.element_size()

        # One public-API call per sequence, alternating two streams, so the
        # host->device copy of sequence b+1 and the device->host copy of b-1
        # overlap the attention of b (copy engines run both directions at once).
        # Steps follow each other on the same two streams with no barrier in
        # between (a serving loop's steady state): every step still copies all
        # of its inputs in and its whole output out; the host waits once, after
        # the last step.
        streams = [torch.cuda.Stream(dev) for _ in range(2)]
        turn = [0]

        def e2e_step():
            for b in range(cfg["B"]):
                turn[0] ^= 1
                with torch.cuda.stream(streams[turn[0]]):
                    q = hq[b:b + 1].to(dev, non_blocking=True)
                    k = hk[b:b + 1].to(dev, non_blocking=True)
                    v = hv[b:b + 1].to(dev, non_blocking=True)
                    iq = hiq[b:b + 1].to(dev, non_blocking=True)
                    ik = hik[b:b + 1].to(dev, non_blocking=True)
                    out = MD.dash_prefill_forward(q, k, v, iq, ik, block_size=cfg["bs"],
                                                  local_blocks=cfg["lb"], K=cfg["K"],
                                                  idx_scale=IDX_SCALE, prior_floor=1e-4, sigma=1.0)
                    hout[b:b + 1].copy_(out, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        main = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s_ in streams:
            s_.wait_stream(main)
        for _ in range(args.steps):
            e2e_step()
        for s_ in streams:
            main.wait_stream(s_)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            tt = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_ms = float(tt[0])
        e2e = {"value": tokens_per_rank * world / (e2e_ms / 1e3), "unit": "tokens/s",
               "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    page_res = None
    if not args.no_pages and args.workload == "c2":
        page_res = run_page_aware(cfg, st, dev, args.steps, args.warmup)
    fe_res = None
    if not args.no_frontend and args.workload == "c2":
        fe_res = run_frontend(cfg, dev, args.steps, args.warmup)
    bw_res = None
    if not args.no_backward and args.workload == "c2":
        bw_res = run_backward(cfg, dev, args.steps, args.warmup)
    b32_res = None
    if not args.no_block32 and args.workload == "c2":
        b32_res = run_prefill_on(C2_BS32, st, dev, args.steps, args.warmup)
    c4_res = None
    if not args.no_c4 and args.workload == "c2":
        # every rank takes part (strong scaling of config 4 with the gather)
        torch.cuda.empty_cache()
        c4_res = run_c4(dev, rank, world, 3, 3, args.gather if args.gather != "none" else "fused")
        torch.cuda.empty_cache()
    c5_res = None
    if not args.no_c5 and args.workload == "c2" and world == 1:
        # the whole decoder on one GPU (replicas only at N > 1, not timed there)
        c5_res = c5_summary(run_c5(dev, 64, max(3, args.warmup)))

    peaks, peak_kind = load_peaks()
    if gather is not None:
        gather.close()
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    achieved = st["alg"] / (attn_ms / 1e3) / 1e12
    peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    traffic = None
    tp = os.path.join(REPO, "profiles", "prefill_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(cfg["name"])
    line = {
        "metric": "DASH attn tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": cfg["name"], "sequences_per_gpu": cfg["B"], "heads": cfg["H"],
                   "seq_len": cfg["S"], "head_dim": cfg["D"], "block_size": cfg["bs"],
                   "local_blocks": cfg["lb"], "routed_k": cfg["K"], "parallelism": f"shard{world}",
                   "l2": "inputs exceed L2 (126 MB); no flush",
                   "output_gather_in_step": (
                       "none (one GPU)" if world == 1 else
                       {"fused": "fused into the attention kernel: every output row stored into "
                                 "every rank's gathered tensor over NVLink, then one NCCL "
                                 "completion word",
                        "nccl": "NCCL all_gather_into_tensor after the attention",
                        "none": "none (excluded)"}[args.gather])},
        "breakdown_ms": {"route": route_ms, "attention": attn_ms},
        "prefill": {"alg_tflops": achieved, "executed_tflops": st["executed"] / (attn_ms / 1e3) / 1e12,
                    "alg_flops_per_step": st["alg"], "executed_flops_per_step": st["executed"]},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "prefill_kernel (+plan_kernel), algorithmic FLOPs / CUDA-event time",
                     "peak_source": f"{peak_kind} bf16_tflops"},
        "gpu_launches": launches,
        "nccl_all_gather_alone": nccl_gather,
        "clocks": clk,
    }
    if dec_res is not None:
        hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
        gbs = dec_res["bytes_per_step"] / (dec_res["attn_ms"] + dec_res["route_ms"]) / 1e6
        attn_gbs = dec_res["kv_bytes"] / dec_res["attn_ms"] / 1e6
        line["decode"] = {"workload": C3["name"], "tokens_per_s": C3["R"] / (dec_res["ms_per_step"] / 1e3),
                          "ms_per_step": dec_res["ms_per_step"], "attn_ms": dec_res["attn_ms"],
                          "route_ms": dec_res["route_ms"], "gbs": gbs, "attn_kv_gbs": attn_gbs,
                          "roofline": {"bound": "hbm", "achieved": attn_gbs, "peak": hbm,
                                       "unit": "GB/s", "frac": attn_gbs / hbm,
                                       "kernel": "decode_kernel, K+V bytes of attended keys",
                                       "peak_source": f"{peak_kind} hbm_gbs"}}
    if page_res is not None:
        hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
        ms = page_res["ms"]
        gbs = page_res["page_ids_bytes"] / ms["page_ids"] / 1e6
        line["page_aware"] = {
            "workload": cfg["name"] + " + page-aware candidates (page_scope_prefill)",
            "ms": ms, "route_overhead_ms": ms["route_page"] - ms["route_plain"],
            "dense_path_ms": ms["dense_mask"] + ms["route_dense"],
            "compact_path_ms": ms["page_ids"] + ms["route_page"],
            "rows": page_res["rows"], "rows_with_page": page_res["rows_with_page"],
            "routes_equal_dense": page_res["equal_to_dense"],
            "l2": "inputs L2-resident (token ids 0.3 MB)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / hbm, "kernel": "page_ids_kernel, ids in + pages out",
                         "bytes_per_launch": page_res["page_ids_bytes"],
                         "peak_source": f"{peak_kind} hbm_gbs"}}
        if not args.no_cpu and world == 1:
            pc = page_cpu_baseline(cfg)
            pc.pop("seconds", None)
            line["page_aware"]["cpu_baseline"] = pc
    if fe_res is not None:
        hbm = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
        ms = fe_res["ms"]["index_proj"]
        gbs = fe_res["bytes"] / ms / 1e6
        line["frontend"] = {
            "workload": cfg["name"] + " router front end (hidden 1280 -> index q, k; RMSNorm; RoPE)",
            "ms": fe_res["ms"], "tokens_per_s": fe_res["tokens"] / (ms / 1e3),
            "tflops": fe_res["flops"] / (ms / 1e3) / 1e12,
            "l2": "flushed before every timed replay",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / hbm, "kernel": "index_proj_kernel, hidden + weights in, "
                                                      "q/k fp32 out, cos/sin in",
                         "bytes_per_launch": fe_res["bytes"],
                         "peak_source": f"{peak_kind} hbm_gbs"}}
    if bw_res is not None:
        peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        tf = bw_res["flops"] / (bw_res["ms"] / 1e3) / 1e12
        line["backward"] = {
            "workload": cfg["name"] + " attention backward (dq, dk, dv, slot-bias gradient), "
                                      "uniform random routes",
            "ms": bw_res["ms"], "tokens_per_s": bw_res["tokens"] / (bw_res["ms"] / 1e3),
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak, "kernel": "dash_attn_bwd: bwd_flags + bwd_delta + "
                                                     "bwd_tc_kernel (tcgen05) + bwd_dq_convert",
                         "flops_per_launch": bw_res["flops"],
                         "peak_source": f"{peak_kind} bf16_tflops"}}
    if b32_res is not None:
        peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
        c = C2_BS32
        tf = b32_res["alg"] / (b32_res["attn_ms"] / 1e3) / 1e12
        line["block32"] = {
            "workload": c["name"], "block_size": c["bs"], "local_blocks": c["lb"],
            "routed_k": c["K"], "entmax_window": c["topm"],
            "tokens_per_s": b32_res["tokens"] / ((b32_res["route_ms"] + b32_res["attn_ms"]) / 1e3),
            "route_ms": b32_res["route_ms"], "attn_ms": b32_res["attn_ms"],
            "alg_tflops": tf, "executed_tflops": b32_res["executed"] / (b32_res["attn_ms"] / 1e3) / 1e12,
            "alg_flops_per_step": b32_res["alg"], "executed_flops_per_step": b32_res["executed"],
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": tf / peak,
                         "kernel": "prefill_kernel (32-token blocks, two per key tile) + plan_kernel",
                         "peak_source": f"{peak_kind} bf16_tflops"}}
    if c4_res is not None:
        line["c4"] = c4_summary(c4_res, world, args.gather, peaks, peak_kind)
    if c5_res is not None:
        line["c5"] = c5_res
    if e2e is not None:
        line["e2e"] = e2e
    if not args.no_cpu and world == 1:   # the CPU baseline is timed at N = 1 only
        runs = [cpu_baseline(cfg, n_tokens=4096) for _ in range(3)]
        runs.sort(key=lambda r: r["value"])
        line["cpu_baseline"] = runs[1]
        line["cpu_baseline"]["sample"] += " (median of 3)"
        line["cpu_baseline"].pop("seconds", None)
    print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
