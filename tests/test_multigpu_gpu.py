"""Sharded prefill on two GPUs (one process each, NCCL): the output gather
fused into the attention kernel (peer stores over NVLink) and the NCCL
all-gather both give every rank the single-GPU output, bit for bit, for a
sequence split (4 sequences over 2 ranks) and a kv-head split (1 sequence over
2 ranks).  Skipped with fewer than two GPUs."""
import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

KW = dict(block_size=64, local_blocks=2, K=4, idx_scale=128.0 / math.sqrt(128), prior_floor=1e-4,
          sigma=1.0)


def _inputs(B, H, S):
    g = torch.Generator().manual_seed(7)
    q, k, v = ((torch.randn(B, H, S, 128, generator=g) * 0.5).bfloat16() for _ in range(3))
    iq, ik = (torch.randn(B, S, 128, generator=g) * 0.5 for _ in range(2))
    return q, k, v, iq, ik


def _worker(rank, world, port, B, H, S, res):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch.distributed as dist
    from datetime import timedelta
    from ananta_ocr_b200 import modeling_deepseekv2 as MD
    from ananta_ocr_b200.peer import PeerGather
    from ananta_ocr_b200.sharding import run_sharded, run_sharded_fused
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    q, k, v, iq, ik = (t.to(dev) for t in _inputs(B, H, S))

    def attn(q, k, v, iq, ik, out=None, peers=None):
        return MD.dash_prefill_forward(q, k, v, iq, ik, out=out, peers=peers, **KW)

    ref = attn(q, k, v, iq, ik)
    full = torch.full_like(ref, float("nan"))
    pg = PeerGather(full)
    for _ in range(2):                       # a second call rewrites the same buffers
        got = run_sharded_fused(attn, q, k, v, iq, ik, pg, rank=rank, world=world)
    torch.cuda.synchronize()
    nccl = run_sharded(lambda *a: attn(*a), q, k, v, iq, ik, rank=rank, world=world)
    torch.cuda.synchronize()
    ok = bool(torch.equal(got, ref)) and bool(torch.equal(nccl, ref))
    pg.close()
    dist.destroy_process_group()
    res[rank] = ok


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("B,H,S", [(4, 4, 700), (1, 4, 900)])
def test_fused_gather_two_gpus(B, H, S):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    res = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, H, S, res)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert res[0] and res[1]
