"""The end-to-end decoder (ananta_ocr_b200/e2e_decoder.py) on a small
configuration: a paged prefill of S tokens followed by one decode step gives
the last-token logits of a prefill of S + 1 tokens (KV cache, index cache,
k-bar refresh, decode routing and decode attention consistent with the
prefill path), and the decode step replayed from a CUDA graph equals the
eager step bit for bit.  The two paths sum in different orders (prefill vs
decode attention kernels, grouped vs dense MoE GEMMs), so the logits agree to
2% of their largest magnitude."""
import pytest
import torch

from ananta_ocr_b200.e2e_decoder import DashDecoder, DecoderConfig

pytestmark = pytest.mark.gpu

CFG = DecoderConfig(hidden=256, heads=2, kv_heads=2, layers=3, vocab=1000, dense_ffn=512,
                    moe_ffn=128, experts=8, topk=2, shared=1, block_size=64, local_blocks=2, K=4)


def make(seed=3):
    return DashDecoder(CFG, batch=2, max_len=420, device=torch.device("cuda"), seed=seed)


def test_prefill_plus_decode_equals_longer_prefill():
    S = 333
    ids = torch.randint(0, CFG.vocab, (2, S + 1), generator=torch.Generator().manual_seed(0)).cuda()
    full = make()
    ref = full.prefill(full.embed[ids])
    part = make()
    part.prefill(part.embed[ids[:, :S]])
    part.tok.copy_(ids[:, S])
    got = part.decode_step()
    assert torch.isfinite(got).all() and torch.isfinite(ref).all()
    err = (got.float() - ref.float()).abs().max().item()
    assert err <= 0.02 * ref.float().abs().max().item(), err
    assert torch.equal(part.seq_lens, torch.full_like(part.seq_lens, S + 1))


def test_graph_decode_equals_eager():
    S = 200
    ids = torch.randint(0, CFG.vocab, (2, S), generator=torch.Generator().manual_seed(1)).cuda()
    a, b = make(5), make(5)
    a.prefill(a.embed[ids])
    b.prefill(b.embed[ids])
    a.tok.fill_(7)
    b.tok.fill_(7)
    eager = [a.decode_step().clone() for _ in range(3)]
    b.decode_step()                       # warm-up (eager), then rewind one step
    b.seq_lens.sub_(1)
    b.tok.fill_(7)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            out = b.decode_step()
    torch.cuda.current_stream().wait_stream(s)
    replay = []
    for _ in range(3):
        g.replay()
        replay.append(out.clone())
    for e, r in zip(eager, replay):
        assert torch.equal(e, r)
    assert torch.equal(a.tok, b.tok) and torch.equal(a.seq_lens, b.seq_lens)
