"""mlx_primitives — the attention forward path of zakkeown/mlx-primitives on NVIDIA B200.

Drop-in for ``from mlx_primitives import flash_attention, FlashAttention,
SlidingWindowAttention, ChunkedCrossAttention, ...`` with torch tensors in place of mx.array.
All compute runs in libmlxp_attn.so (hand-written sm_100a CUDA); there is no CPU fallback.
"""

from .attention import (ChunkedCrossAttention, FlashAttention, SlidingWindowAttention,
                        chunked_cross_attention, create_sliding_window_mask,
                        estimate_memory_savings, flash_attention, get_optimal_flash_config,
                        sliding_window_attention)
from .cache import paged_attention
from .constants import Layout

__version__ = "0.2.0+b200"

__all__ = [
    "FlashAttention",
    "flash_attention",
    "get_optimal_flash_config",
    "SlidingWindowAttention",
    "sliding_window_attention",
    "create_sliding_window_mask",
    "ChunkedCrossAttention",
    "chunked_cross_attention",
    "estimate_memory_savings",
    "paged_attention",
    "Layout",
]
