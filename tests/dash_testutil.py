"""Shared helpers for the parity tests (not collected as tests)."""
import math

import numpy as np
import torch

# north_star tolerance for bf16 outputs against an fp32 reference
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def assert_close_bf16(got, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), "non-finite output"
    err = np.abs(got - ref)
    assert err.max() <= max_abs, f"max abs err {err.max():.3e} > {max_abs}"
    assert err.mean() <= mean_abs, f"mean abs err {err.mean():.3e} > {mean_abs}"


def random_routes(rng, B, T, K, bs, local_window, messy=True, n_index_heads=1):
    """Routed lists [B,HI,T,K] int32 + bias: mostly valid remote blocks; with
    ``messy`` also -1 slots, duplicates, future / local ids and unsorted order."""
    nblk = (T + bs - 1) // bs
    idx = np.full((B, n_index_heads, T, K), -1, np.int32)
    bias = (rng.standard_normal((B, n_index_heads, T, K)) * 2.0).astype(np.float32)
    for b in range(B):
        for h in range(n_index_heads):
            for t in range(T):
                hi = (t - local_window) // bs  # last block with a remote key
                if hi >= 0:
                    cnt = min(K, hi + 1)
                    ch = rng.choice(hi + 1, size=cnt, replace=False)
                    idx[b, h, t, :cnt] = ch
                if messy and K >= 3:
                    r = rng.random()
                    if r < 0.1:
                        idx[b, h, t, K - 1] = idx[b, h, t, 0]           # duplicate
                    elif r < 0.2:
                        idx[b, h, t, K - 1] = rng.integers(0, nblk)     # maybe future/local
                    elif r < 0.3:
                        idx[b, h, t, 1] = -1
                if messy:
                    rng.shuffle(idx[b, h, t])
    return idx, bias


def sample_rows(rng, T, n):
    rows = np.unique(np.concatenate([np.arange(min(T, 3)), np.arange(max(0, T - 3), T),
                                     rng.integers(0, T, size=n)]))
    return rows.astype(np.int64)


def scale_of(D):
    return 1.0 / math.sqrt(D)
