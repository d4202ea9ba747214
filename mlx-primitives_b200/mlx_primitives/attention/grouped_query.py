"""Grouped-query attention on B200 (drop-in for mlx_primitives/attention/grouped_query.py).

Same names, signatures and defaults as the reference: ``gqa_attention`` (grouped_query.py:
195-261) on pre-projected BSHD tensors and the ``GroupedQueryAttention`` module
(grouped_query.py:21-192) with its q/k/v/out projections and KV cache.  The reference repeats
each K/V head ``num_kv_groups`` times (``mx.broadcast_to`` + reshape) and runs dense attention;
here the attention kernel reads K/V head ``h // num_kv_groups`` for query head ``h`` directly
(mlxp_attn_fwd_gqa), so the repeated K/V never exist.  Causal masking is bottom-right aligned
(``triu(k=seq_kv - seq_q + 1)``), as in the reference.

A custom additive ``mask`` (broadcastable to (batch, heads, seq_q, seq_kv)) is added to the
scores after the causal mask, as the reference does (grouped_query.py:253-254); the kernels
read it tile by tile (mlxp_attn_fwd_masked), never as a repeated dense copy.  Where the
reference has no defined result: a query row with no admissible key (causal with seq_q >
seq_kv, or a mask of -inf across the row) returns zeros where the reference's -inf would give
NaN.  Gradients through a custom mask are not supported (the backward kernels take causal and
window masks).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch import nn

from ._core import attention_forward

__all__ = ["GroupedQueryAttention", "gqa_attention"]


def _grouped_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       scale: Optional[float], mask, causal: bool) -> torch.Tensor:
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k and v must be 4-D (batch, seq, heads, head_dim)")
    if k.shape != v.shape:
        raise ValueError(f"k and v must have the same shape, got {tuple(k.shape)} and "
                         f"{tuple(v.shape)}")
    B, Sq, H, D = q.shape
    if k.shape[0] != B or k.shape[3] != D:
        raise ValueError("q and k must agree in batch size and head_dim")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    Sq, Skv = q.shape[1], k.shape[1]
    return attention_forward(q, k, v, layout="BSHD", scale=float(scale), causal=bool(causal),
                             q_offset=(Skv - Sq) if causal else 0, mask=mask)


def gqa_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    num_kv_groups: int,
    scale: Optional[float] = None,
    mask: Optional[torch.Tensor] = None,
    causal: bool = False,
) -> torch.Tensor:
    """Grouped-query attention on pre-projected tensors (grouped_query.py:195-261).

    q: (batch, seq_q, num_heads, head_dim); k, v: (batch, seq_kv, num_kv_heads, head_dim) with
    num_heads == num_kv_heads * num_kv_groups.  Returns (batch, seq_q, num_heads, head_dim).
    """
    if q.ndim == 4 and k.ndim == 4 and q.shape[2] != k.shape[2] * num_kv_groups:
        raise ValueError(
            f"num_heads ({q.shape[2]}) must equal num_kv_heads ({k.shape[2]}) * num_kv_groups "
            f"({num_kv_groups})")
    return _grouped_attention(q, k, v, scale, mask, causal)


class GroupedQueryAttention(nn.Module):
    """Grouped-query attention module (grouped_query.py:21-192): num_kv_heads K/V heads shared
    by groups of the num_heads query heads, with input/output projections and a KV cache."""

    def __init__(
        self,
        dims: int,
        num_heads: int,
        num_kv_heads: int,
        head_dim: Optional[int] = None,
        causal: bool = False,
        dropout: float = 0.0,
        bias: bool = False,
    ):
        super().__init__()
        if num_heads % num_kv_heads != 0:
            raise ValueError(
                f"num_heads ({num_heads}) must be divisible by num_kv_heads ({num_kv_heads})")
        self.dims = dims
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.num_groups = num_heads // num_kv_heads
        self.head_dim = head_dim or dims // num_heads
        self.causal = causal
        self.dropout = dropout
        self.scale = 1.0 / math.sqrt(self.head_dim)
        q_dim = num_heads * self.head_dim
        kv_dim = num_kv_heads * self.head_dim
        self.q_proj = nn.Linear(dims, q_dim, bias=bias)
        self.k_proj = nn.Linear(dims, kv_dim, bias=bias)
        self.v_proj = nn.Linear(dims, kv_dim, bias=bias)
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
        Skv = keys.shape[1]
        q = self.q_proj(queries).reshape(B, Sq, self.num_heads, self.head_dim)
        k = self.k_proj(keys).reshape(B, Skv, self.num_kv_heads, self.head_dim)
        v = self.v_proj(values).reshape(B, Skv, self.num_kv_heads, self.head_dim)
        if cache is not None:
            k = torch.cat([cache[0], k], dim=1)
            v = torch.cat([cache[1], v], dim=1)
        new_cache = (k, v)
        out = _grouped_attention(q, k, v, self.scale, mask, self.causal)
        return self.out_proj(out.reshape(B, Sq, -1)), new_cache
