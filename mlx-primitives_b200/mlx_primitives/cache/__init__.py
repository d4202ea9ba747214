"""Paged-KV attention of mlx_primitives.cache (mlx_primitives/cache/__init__.py:98-102).

Only the attention entry points of the reference's cache package live here
(paged_attention, paged_attention_with_bias, create_block_table_from_lengths and the ALiBi
slopes helper).  The reference's cache managers (KVCache, block allocator, eviction,
speculative and compressed caches) are serving-side bookkeeping outside the attention path and
are not part of this package.
"""

from .paged_attention import (create_block_table_from_lengths, get_alibi_slopes,
                              paged_attention, paged_attention_with_bias)

__all__ = [
    "paged_attention",
    "paged_attention_with_bias",
    "create_block_table_from_lengths",
    "get_alibi_slopes",
]
