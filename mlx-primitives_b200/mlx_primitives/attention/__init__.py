"""Attention forward path of mlx_primitives, rebuilt for B200 (sm_100a).

The public names match mlx_primitives/attention/__init__.py of the reference for the attention
kernels: flash, sliding-window and chunked cross-attention, grouped-query and multi-query
attention, plus the two multi-GPU forms: the (batch, head) split of one call across GPUs
(partition.py, no collective) and the sequence-parallel ring pass that runs the causal
long-context case over several GPUs (ring.py).
"""

from .chunked import ChunkedCrossAttention, chunked_cross_attention, estimate_memory_savings
from .flash import FlashAttention, flash_attention, get_optimal_flash_config
from .grouped_query import GroupedQueryAttention, gqa_attention
from .multi_query import MultiQueryAttention, mqa_attention
from .partition import (attention_units, chunked_cross_attention_shard, flash_attention_shard,
                        rank_pieces, shard_units, sliding_window_attention_shard, unit_blocks)
from .sliding_window import (SlidingWindowAttention, create_sliding_window_mask,
                             sliding_window_attention)

__all__ = [
    "sliding_window_attention",
    "create_sliding_window_mask",
    "SlidingWindowAttention",
    "flash_attention",
    "FlashAttention",
    "get_optimal_flash_config",
    "chunked_cross_attention",
    "ChunkedCrossAttention",
    "estimate_memory_savings",
    "GroupedQueryAttention",
    "gqa_attention",
    "MultiQueryAttention",
    "mqa_attention",
    "shard_units",
    "unit_blocks",
    "rank_pieces",
    "attention_units",
    "flash_attention_shard",
    "sliding_window_attention_shard",
    "chunked_cross_attention_shard",
]
