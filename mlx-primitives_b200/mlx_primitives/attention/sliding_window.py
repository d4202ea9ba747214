"""sliding_window_attention / SlidingWindowAttention on B200 (drop-in for
mlx_primitives/attention/sliding_window.py).

Window semantics follow the reference exactly (sliding_window.py:136-161, 447-511): query i
attends key j when |i - j| <= window_size, and additionally j <= i when causal — so the causal
window holds window_size + 1 keys [i - W, i].  The B200 kernel skips every key tile outside the
band and masks only the tiles that straddle its edges; no mask is materialised.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from ._core import attention_forward

__all__ = ["sliding_window_attention", "SlidingWindowAttention", "create_sliding_window_mask"]


def sliding_window_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    window_size: int,
    scale: Optional[float] = None,
    causal: bool = True,
    use_metal: bool = True,
    dropout_p: float = 0.0,
    training: bool = True,
) -> torch.Tensor:
    """Attention restricted to a window of ``window_size`` keys on each side (one side if
    causal).  q, k, v are BSHD (batch, seq, heads, head_dim); ``use_metal`` is ignored.

    Positions are counted from 0 for both q and k (the reference's tiled path,
    sliding_window.py:363-444).  ``dropout_p > 0`` with ``training`` raises
    NotImplementedError (dropout needs the materialised weights).
    """
    if q.ndim != 4:
        raise ValueError(f"Expected 4D tensors (batch, seq, heads, dim), got {q.ndim}D")
    if k.ndim != 4 or v.ndim != 4:
        raise ValueError("Expected 4D K and V tensors (batch, seq, heads, dim)")
    if window_size < 0:
        raise ValueError(f"window_size must be >= 0, got {window_size}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"Q/K/V dtype mismatch: Q={q.dtype}, K={k.dtype}, V={v.dtype}")
    if k.shape != v.shape or k.shape[0] != q.shape[0] or k.shape[2:] != q.shape[2:]:
        raise ValueError(f"Incompatible shapes: Q={tuple(q.shape)}, K={tuple(k.shape)}, V={tuple(v.shape)}")
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if dropout_p > 0.0 and training:
        raise NotImplementedError(
            "sliding_window_attention: dropout needs the materialised attention matrix; "
            "call with dropout_p=0.0 or training=False")
    w = int(window_size)
    return attention_forward(q, k, v, layout="BSHD", scale=float(scale), causal=bool(causal),
                             window_left=w, window_right=-1 if causal else w)


def create_sliding_window_mask(seq_len: int, window_size: int, causal: bool = True,
                               device: Optional[torch.device] = None) -> torch.Tensor:
    """Boolean (seq_len, seq_len) mask, True where query i may attend key j
    (sliding_window.py:628-656).  A helper for callers; the kernels never build it."""
    pos = torch.arange(seq_len, device=device)
    mask = (pos[:, None] - pos[None, :]).abs() <= window_size
    if causal:
        mask &= pos[None, :] <= pos[:, None]
    return mask


class SlidingWindowAttention:
    """Sliding-window attention module (sliding_window.py:659-712): heads, head_dim,
    window_size, causal=True, scale = 1/sqrt(head_dim)."""

    def __init__(self, num_heads: int, head_dim: int, window_size: int,
                 causal: bool = True) -> None:
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.window_size = window_size
        self.causal = causal
        self.scale = 1.0 / math.sqrt(head_dim)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        return sliding_window_attention(q, k, v, window_size=self.window_size,
                                        scale=self.scale, causal=self.causal)
