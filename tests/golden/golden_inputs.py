"""Seeded inputs of the golden cases that the tests regenerate instead of
storing (numpy PCG64: identical on every machine).  Shared by
make_golden.py and the tests."""
from __future__ import annotations

import hashlib
import math

import numpy as np


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def dash_attention_inputs(seed, B, S, hidden, H, D, n_pages, page_tokens):
    """Seeded module weights and inputs for the DashAttention goldens (numpy
    PCG64, regenerated identically by the tests)."""
    rng = np.random.default_rng(seed)
    w = dict(q_proj=rng.standard_normal((128, hidden)) / math.sqrt(hidden),
             k_proj=rng.standard_normal((128, hidden)) / math.sqrt(hidden),
             q_norm=rng.standard_normal(128) * 0.1, k_norm=rng.standard_normal(128) * 0.1,
             head_cls=rng.standard_normal(128) * 0.5)
    h = rng.standard_normal((B, S, hidden))
    for p in range(n_pages):
        a, b = p * page_tokens, min(S, (p + 1) * page_tokens)
        h[:, a:b] += rng.standard_normal((B, 1, hidden)) * 0.5
    q, k, v = ((rng.standard_normal((B, H, S, D)) * 0.5) for _ in range(3))
    pos = np.arange(S, dtype=np.float64)
    inv = 1.0 / (10000.0 ** (np.arange(0, 64) / 64.0))
    ang = np.concatenate([pos[:, None] * inv, pos[:, None] * inv], -1)
    cos, sin = np.broadcast_to(np.cos(ang), (B, S, 128)), np.broadcast_to(np.sin(ang), (B, S, 128))
    dout = rng.standard_normal((B, H, S, D))
    f32 = lambda x: np.ascontiguousarray(x, dtype=np.float32)   # noqa: E731
    return {k_: f32(v_) for k_, v_ in w.items()}, dict(
        hidden=f32(h), q=f32(q), k=f32(k), v=f32(v), cos=f32(cos), sin=f32(sin), dout=f32(dout))
