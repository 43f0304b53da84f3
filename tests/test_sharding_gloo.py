"""Multi-rank partitioning and output gather, world_size 2 and 4 on CPU (gloo).

The attention itself is a stand-in computed per (sequence, head) unit so the
test checks that every unit lands in its place after the gather."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ananta_ocr_b200.sharding import Shard, plan_shards, run_sharded


def test_plan_covers_every_unit_once():
    for B, Hkv, world in [(4, 10, 1), (4, 10, 2), (4, 10, 3), (8, 16, 8), (4, 10, 8), (1, 16, 4)]:
        try:
            plan = plan_shards(B, Hkv, world)
        except ValueError:
            assert world > B and (world % B or Hkv % (world // B))
            continue
        seen = torch.zeros(B, Hkv, dtype=torch.int32)
        for s in plan:
            seen[s.b0:s.b1, s.h0:s.h1] += 1
        assert bool((seen == 1).all()), (B, Hkv, world)


def test_plan_rejects_uneven_head_split():
    with pytest.raises(ValueError):
        plan_shards(4, 10, 12)


def fake_attn(q, k, v, iq, ik):
    # depends on the unit's own q/k/v and router inputs only
    return q * 2.0 + k.repeat_interleave(q.shape[1] // k.shape[1], 1) + iq.mean(-1)[:, None, :, None]


def _worker(rank, world, port, B, H, Hkv, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    S, D = 16, 8
    qq = torch.randn(B, H, S, D)
    kk = torch.randn(B, Hkv, S, D)
    vv = torch.randn(B, Hkv, S, D)
    iq = torch.randn(B, S, 4)
    ik = torch.randn(B, S, 4)
    full = run_sharded(fake_attn, qq, kk, vv, iq, ik, rank=rank, world=world)
    ref = fake_attn(qq, kk, vv, iq, ik)
    q.put((rank, bool(torch.allclose(full, ref))))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,B,H,Hkv", [(2, 4, 10, 10), (2, 3, 4, 2), (4, 2, 8, 4)])
def test_gather_reassembles_output(world, B, H, Hkv):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, H, Hkv, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res
