"""B200-native (sm_100a) DASH block-sparse attention for ANANTA_OCR.

The hot path -- 1.5-entmax block router, prefill gather attention (tcgen05 /
TMEM / TMA) and paged decode gather attention (split-KV with fused combine) --
runs in ``libdash_b200.so`` (C ABI: include/dash_b200.h).  The modules below
keep the reference's module and function names so callers swap them in:

  ananta_ocr_b200.sparse_gather_e2e_triton   triton_gather_attention_e2e
  ananta_ocr_b200.sparse_gather_triton       triton_gather_attention, triton_block_max_score
  ananta_ocr_b200.modeling_deepseekv2        _block_scores_infer, _infer_route_select,
                                             _decode_attend, dash_prefill_forward
  ananta_ocr_b200.unlimited_dash_ops         attend_triton.{dash_sparse_attn,
                                             dash_sparse_attn_decode},
                                             route_triton.{route_prefill_triton,
                                             route_decode_triton, kbar_refresh_tail_triton},
                                             dash_router.DashRouterMath
"""
from . import _lib  # noqa: F401

__all__ = ["ops", "sparse_gather_e2e_triton", "sparse_gather_triton", "modeling_deepseekv2",
           "unlimited_dash_ops", "sharding"]
