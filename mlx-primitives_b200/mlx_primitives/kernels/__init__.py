"""Kernels next to attention in mlx_primitives/kernels of the reference: RoPE and the fused
RoPE + flash attention (the other kernels of that package are not part of this build)."""

from .fused_rope_attention import (FusedRoPEFlashAttention, fast_fused_rope_attention,
                                   fused_rope_attention)
from .rope import fast_rope, fast_rope_qk, precompute_rope_cache, rope, rope_qk

__all__ = [
    "precompute_rope_cache", "rope", "fast_rope", "rope_qk", "fast_rope_qk",
    "fused_rope_attention", "fast_fused_rope_attention", "FusedRoPEFlashAttention",
]
