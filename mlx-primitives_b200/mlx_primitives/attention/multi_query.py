"""Multi-query attention on B200 (drop-in for mlx_primitives/attention/multi_query.py).

``mqa_attention`` (multi_query.py:161-225) and ``MultiQueryAttention`` (multi_query.py:20-158):
every query head shares one K/V head.  The reference broadcasts K/V to all heads; here the
kernel reads the single K/V head for every query head (mlxp_attn_fwd_gqa with one K/V head).
Causal masking is bottom-right aligned as in the reference; a custom additive ``mask`` is added
to the scores (multi_query.py:218-219 of the reference) and fully masked rows return zeros
(see grouped_query.py).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch import nn

from .grouped_query import _grouped_attention

__all__ = ["MultiQueryAttention", "mqa_attention"]


def mqa_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: Optional[float] = None,
    mask: Optional[torch.Tensor] = None,
    causal: bool = False,
) -> torch.Tensor:
    """q: (batch, seq_q, num_heads, head_dim); k, v: (batch, seq_kv, head_dim) or
    (batch, seq_kv, 1, head_dim).  Returns (batch, seq_q, num_heads, head_dim)."""
    if k.ndim == 3:
        k = k[:, :, None, :]
        v = v[:, :, None, :]
    if k.ndim == 4 and k.shape[2] != 1:
        raise ValueError(f"multi-query attention takes one K/V head, got {k.shape[2]}")
    return _grouped_attention(q, k, v, scale, mask, causal)


class MultiQueryAttention(nn.Module):
    """Multi-query attention module (multi_query.py:20-158): one K/V head for all query heads,
    with input/output projections and a KV cache."""

    def __init__(
        self,
        dims: int,
        num_heads: int,
        head_dim: Optional[int] = None,
        causal: bool = False,
        dropout: float = 0.0,
        bias: bool = False,
    ):
        super().__init__()
        self.dims = dims
        self.num_heads = num_heads
        self.head_dim = head_dim or dims // num_heads
        self.causal = causal
        self.dropout = dropout
        self.scale = 1.0 / math.sqrt(self.head_dim)
        q_dim = num_heads * self.head_dim
        self.q_proj = nn.Linear(dims, q_dim, bias=bias)
        self.k_proj = nn.Linear(dims, self.head_dim, bias=bias)
        self.v_proj = nn.Linear(dims, self.head_dim, bias=bias)
        self.out_proj = nn.Linear(q_dim, dims, bias=bias)

    def forward(
        self,
        queries: torch.Tensor,
        keys: Optional[torch.Tensor] = None,
        values: Optional[torch.Tensor] = None,
        mask: Optional[torch.Tensor] = None,
        cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
    ) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
        """(batch, seq_q, dims) -> ((batch, seq_q, dims), (k, v) cache with the new keys)."""
        if keys is None:
            keys = queries
        if values is None:
            values = keys
        B, Sq, _ = queries.shape
        q = self.q_proj(queries).reshape(B, Sq, self.num_heads, self.head_dim)
        k = self.k_proj(keys)[:, :, None, :]
        v = self.v_proj(values)[:, :, None, :]
        if cache is not None:
            k = torch.cat([cache[0], k], dim=1)
            v = torch.cat([cache[1], v], dim=1)
        new_cache = (k, v)
        out = _grouped_attention(q, k, v, self.scale, mask, self.causal)
        return self.out_proj(out.reshape(B, Sq, -1)), new_cache
