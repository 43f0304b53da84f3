"""Serving-path (block-paged KV cache) drop-ins: routing and attend."""
