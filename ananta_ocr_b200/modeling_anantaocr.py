"""Drop-in for the DASH decode helper of ANANTA_OCR ``modeling_anantaocr.py``,
backed by libdash_b200.so.

``_uocr_dash_decode_allow`` (modeling_anantaocr.py:450-496) keeps, per KV
block, the [min, max] image page it holds after the prompt, and gives each
decode query the blocks of its own page.  The prefill branch is one
``dash_page_ids`` pass (rule 1: per-token marker rule, block bounds, pp and the
marker count); the decode branch updates the marker count and builds the mask
on the device (``dash_page_decode_query`` + ``dash_page_allow``), with no host
synchronisation.  The state kept on the cache holds int32 tensors where the
reference keeps int64 (page ids and counts of one document fit).
"""
from __future__ import annotations

import torch

from . import pages


@torch.no_grad()
def _uocr_dash_decode_allow(indexer, input_ids, cache):
    """Prefill (q_len > 1): records the page state on ``cache`` and returns
    None.  Decode (q_len == 1): returns [B, nblk] bool, the blocks holding an
    image token of the query's page, or every block when there is none."""
    img_id, pg_id = indexer.image_token_id, indexer.page_token_id
    if img_id is None or pg_id is None:
        return None
    bs = int(indexer.block_size)
    ids = input_ids
    B, L = ids.shape
    if L > 1:
        nblk = -(-L // bs)
        r = pages.page_ids(ids, image_token_id=img_id, page_token_id=pg_id,
                           per_page=max(1, int(indexer.per_page_image_tokens)), key_length=L,
                           rule=1, block_size=bs, n_blocks=nblk, token_outputs=False, bits=False)
        cache._uocr_pg = {"bmin": r["lo"], "bmax": r["hi"], "pp": r["prompt_pages"].clone(),
                          "mcum": r["marker_count"].clone()}
        return None
    st = getattr(cache, "_uocr_pg", None)
    if st is None:
        return None
    q = pages.page_decode_query(ids[:, -1], st["mcum"], st["pp"], pg_id)
    total = int(cache.get_seq_length()) + L
    nblk = -(-total // bs)
    return pages.page_allow(q, st["bmin"], st["bmax"], width=nblk, rows=B, rows_per_seq=1,
                            desc_width=min(nblk, st["bmin"].shape[-1]), fallback=True)
