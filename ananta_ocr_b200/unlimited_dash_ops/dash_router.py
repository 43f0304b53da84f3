"""Drop-in for the serving path's ``unlimited_dash_ops/dash_router.py``
(WHL sglang/srt/layers/attention/unlimited_dash_ops/dash_router.py).

``DashRouterMath`` keeps the reference's configuration fields (idx_scale,
topm, budget_remote, out_slots, ...) and ``route_and_select`` its return
contract (block_indices int32 with -1 in unused slots, fp32 bias), computed by
the fused selection kernel of libdash_b200.so on precomputed scores.
Returned ids are in ascending order (the torch reference returns descending
score order; the set and the per-id bias are the same).
"""
from __future__ import annotations

import torch

from .. import ops

SCORE_NEG = -1.0e9
ENTMAX_NEG = -1.0e4
TOPM_DEFAULT = 16


class DashRouterMath:
    def __init__(self, *, index_dim: int, block_size: int, local_blocks: int, topk_blocks: int,
                 scaling_factor: float = 1.0, sigma: float = 1.0, prior_floor: float = 1.0e-2,
                 image_only: bool = True, image_fallback_remote=None, budget_remote=None,
                 topm=None) -> None:
        self.index_dim = int(index_dim)
        self.block_size = int(block_size)
        self.local_blocks = max(1, int(local_blocks))
        self.local_window = self.local_blocks * self.block_size
        self.topk_blocks = int(topk_blocks)
        self.remote_blocks = max(1, self.topk_blocks - self.local_blocks)
        self.budget_remote = max(1, int(budget_remote)) if budget_remote else self.remote_blocks
        self.image_fallback_remote = (int(image_fallback_remote) if image_fallback_remote
                                      else self.remote_blocks)
        self.scaling_factor = float(scaling_factor)
        self.sigma = float(sigma)
        self.prior_floor = float(prior_floor)
        self.image_only = bool(image_only)
        self.idx_scale = self.scaling_factor / (self.index_dim ** 0.5)
        self.topm = int(topm) if topm else TOPM_DEFAULT
        slots = 1 << max(0, int(self.budget_remote) - 1).bit_length()
        self.out_slots = max(1, min(slots, self.topm))

    @torch.no_grad()
    def route_and_select(self, block_scores: torch.Tensor, nblk: int,
                         image_block_mask: torch.Tensor | None = None):
        """block_scores [..., W] fp32 (SCORE_NEG = not remote) -> (idx int32
        [..., out_slots], bias fp32 [..., out_slots])."""
        lead = block_scores.shape[:-1]
        W = block_scores.shape[-1]
        sc = block_scores.reshape(-1, W).float().contiguous()
        rows = sc.shape[0]
        M = max(1, min(self.topm, int(nblk), W))
        K = max(1, min(self.budget_remote, M))
        cand = None
        if self.image_only and image_block_mask is not None:
            cand = torch.broadcast_to(image_block_mask, block_scores.shape).reshape(-1, W)
        seqs = ops.Seqs(n_seq=rows, q_len=1, kv_len=0, max_q_len=1)
        ow = M                                   # reference width: the top-M window
        idx, bias = ops.route(seqs, width=W, block_size=self.block_size,
                              local_blocks=self.local_blocks, idx_scale=self.idx_scale,
                              prior_floor=self.prior_floor, sigma=self.sigma, topm=M, K=K,
                              scores_in=sc, cand=cand, out_width=ow)
        return idx.reshape(*lead, ow), bias.reshape(*lead, ow)


def _sched_slot(sparse_cfg: dict, layer_idx: int) -> int:
    freq = sparse_cfg.get("sparse_attention_freq")
    if not isinstance(freq, (list, tuple)) or layer_idx >= len(freq):
        return int(layer_idx)
    return sum(1 for f in freq[:layer_idx] if f)


def _per_layer(sparse_cfg: dict, key: str, layer_idx):
    if layer_idx is None:
        return None
    arr = sparse_cfg.get(key)
    if not isinstance(arr, (list, tuple)) or not arr:
        return None
    slot = _sched_slot(sparse_cfg, int(layer_idx))
    if not 0 <= slot < len(arr):
        return None
    return float(arr[slot])


def router_from_sparse_config(sparse_cfg: dict, layer_idx=None) -> DashRouterMath:
    """Router configuration from checkpoint keys (dash_router.py:218-248)."""
    index_dim = int(sparse_cfg.get("sparse_index_dim", 128))
    scaling = _per_layer(sparse_cfg, "dash_scale_per_layer", layer_idx)
    floor = _per_layer(sparse_cfg, "dash_floor_per_layer", layer_idx)
    if scaling is None:
        scaling = float(sparse_cfg.get("dash_scaling_factor", 1.0))
    if floor is None:
        floor = float(sparse_cfg.get("dash_prior_floor", 1.0e-2))
    budget = sparse_cfg.get("dash_topk_blocks")
    if budget is None:
        budget = sparse_cfg.get("dash_image_fallback_remote")
    return DashRouterMath(
        index_dim=index_dim, block_size=int(sparse_cfg.get("sparse_block_size", 128)),
        local_blocks=int(sparse_cfg.get("sparse_local_block", 1)),
        topk_blocks=int(sparse_cfg.get("sparse_topk_blocks", 16)), scaling_factor=scaling,
        sigma=float(sparse_cfg.get("dash_sigma", 1.0)), prior_floor=floor,
        image_only=bool(sparse_cfg.get("dash_image_only", True)),
        image_fallback_remote=int(sparse_cfg.get("dash_image_fallback_remote", 0)) or None,
        budget_remote=int(budget) if budget else None,
        topm=int(sparse_cfg.get("dash_infer_topm", 0)) or None)
