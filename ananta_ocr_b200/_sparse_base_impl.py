"""Drop-ins for the page-aware candidate builders of ANANTA_OCR's
``DeepseekV2Indexer`` (``_sparse_base_impl.py:2177-2484``), backed by
libdash_b200.so.

``DeepseekV2IndexerPages`` carries the methods under the reference's names and
signatures.  An indexer inherits it (or the methods are bound onto an existing
indexer object); they read the attributes the reference reads:
``block_size``, ``per_page_image_tokens``, ``image_bucket_constraint`` and, for
the device, ``q_proj`` (else the device of the input).

What changes against the reference is the data path, not the results:
* page ids come from one fused kernel pass over the token ids
  (``dash_page_ids``) instead of cumsum/gather/where chains;
* the candidate mask is computed from per-block page descriptors (lo, hi,
  page bits) and one query page per row (``dash_page_blocks`` +
  ``dash_page_allow``), never through the reference's
  [B, C, nblk, block_size] comparison tensor, so callers need not chunk it.
"""
from __future__ import annotations

import os

import torch

from . import pages

# _sparse_base_impl.py:36 -- keep the page of PREFILL query tokens (text before
# the last image token) instead of leaving them unconstrained.
_PAGE_SCOPE_PREFILL = os.environ.get("PAGE_SCOPE_PREFILL", "0") == "1"


class DeepseekV2IndexerPages:
    """Page-aware candidate-domain methods of the indexer."""

    def _pages_device(self, t):
        q = getattr(self, "q_proj", None)
        return q.weight.device if q is not None else t.device

    def _build_image_block_allow_mask(self, image_token_mask, num_key_blocks):
        """_sparse_base_impl.py:2177-2187: [B, nblk] bool, any image token in
        the block (mask padded with False / truncated to nblk * block_size)."""
        m = image_token_mask.to(device=self._pages_device(image_token_mask), dtype=torch.bool)
        return pages.block_any(m, num_key_blocks, self.block_size)

    def _build_page_aware_ids(self, source_input_ids, img_context_token_id, page_token_id,
                              key_length):
        """_sparse_base_impl.py:2189-2260: (image_token_mask bool, image page ids
        int64, query page ids int64) [B, key_length], or (None, None, None)
        when there are no ids, no image token, or no query with a page."""
        if source_input_ids is None or img_context_token_id is None or page_token_id is None:
            return None, None, None
        if source_input_ids.ndim != 2:
            return None, None, None
        ids = source_input_ids.to(device=self._pages_device(source_input_ids))
        r = pages.page_ids(ids, image_token_id=img_context_token_id, page_token_id=page_token_id,
                           per_page=max(1, int(self.per_page_image_tokens)),
                           key_length=int(key_length), rule=0,
                           page_scope_prefill=_PAGE_SCOPE_PREFILL, page_dtype=torch.int64)
        n_img, n_q = torch.stack([r["n_image"].sum(), r["n_query"].sum()]).tolist()
        if n_img == 0 or n_q == 0:
            return None, None, None
        return r["image_mask"], r["image_page"], r["query_page"]

    def _build_flat_image_token_mask(self, source_input_ids, img_context_token_id, key_length):
        """_sparse_base_impl.py:2363-2381: [B, key_length] bool image mask, or
        None when there are no ids or no image token."""
        if source_input_ids is None or img_context_token_id is None:
            return None
        if source_input_ids.ndim != 2:
            return None
        ids = source_input_ids.to(device=self._pages_device(source_input_ids))
        r = pages.page_ids(ids, image_token_id=img_context_token_id, page_token_id=None,
                           per_page=1, key_length=int(key_length), rule=1)
        if int(r["n_image"].sum()) == 0:
            return None
        return r["image_mask"]

    def _page_candidates(self, image_token_page_ids, query_token_page_ids, pos_chunk,
                         num_key_blocks, fallback):
        B, C = pos_chunk.shape
        bs = self.block_size
        k_len = image_token_page_ids.shape[-1]
        lo, hi, bits = pages.page_blocks(image_token_page_ids, num_key_blocks, bs,
                                         length=min(k_len, num_key_blocks * bs))
        out = pages.page_allow(query_token_page_ids, lo, hi, bits=bits, width=num_key_blocks,
                               rows=B * C, rows_per_seq=C, q_pos=pos_chunk, fallback=fallback)
        return out.view(B, 1, C, num_key_blocks)

    def _build_page_aware_image_block_mask(self, image_token_page_ids, query_token_page_ids,
                                           pos_chunk, num_key_blocks, cq):
        """_sparse_base_impl.py:2383-2402: [B, 1, cq, nblk] bool, the block holds
        an image token of the query's page (page gathered at the clamped position)."""
        return self._page_candidates(image_token_page_ids, query_token_page_ids, pos_chunk,
                                     num_key_blocks, fallback=False)

    def _build_kl_candidate_mask(self, pos_chunk, num_key_blocks, image_token_mask, batch, cq,
                                 image_token_page_ids=None, query_token_page_ids=None):
        """_sparse_base_impl.py:2457-2484: [B, 1, cq, nblk] bool candidate domain
        with the per-query fallback to every block."""
        device = pos_chunk.device
        if self.image_bucket_constraint and image_token_page_ids is not None \
                and query_token_page_ids is not None:
            return self._page_candidates(image_token_page_ids, query_token_page_ids, pos_chunk,
                                         num_key_blocks, fallback=True)
        if image_token_mask is not None:
            img_blk = self._build_image_block_allow_mask(image_token_mask, num_key_blocks)
            img_blk = img_blk | ~img_blk.any(dim=-1, keepdim=True)
            return img_blk[:, None, None, :].expand(batch, 1, cq, num_key_blocks).contiguous()
        return torch.ones(batch, 1, cq, num_key_blocks, dtype=torch.bool, device=device)
