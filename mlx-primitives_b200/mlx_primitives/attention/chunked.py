"""chunked_cross_attention / ChunkedCrossAttention on B200 (drop-in for
mlx_primitives/attention/chunked.py).

The reference walks the key sequence in ``chunk_size`` pieces and merges the partial softmax
states (chunked.py:129-169); here the key range is split across CTAs (split-KV), each split
writes its normalised fp32 partial and log-sum-exp, and an LSE-merge kernel combines them.
The number of splits is chosen to fill the GPU; the result does not depend on it (or on
``chunk_size``) beyond floating-point rounding.  Causal masking uses top-left absolute
positions (kv_pos <= q_pos), as the reference does (_online_softmax.py:149-161,
chunked.py:192-197).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from ._core import attention_forward

__all__ = ["chunked_cross_attention", "ChunkedCrossAttention", "estimate_memory_savings"]


def chunked_cross_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    chunk_size: int = 1024,
    scale: Optional[float] = None,
    causal: bool = False,
    use_metal: bool = True,
    dropout_p: float = 0.0,
    training: bool = True,
) -> torch.Tensor:
    """Cross-attention of q (batch, seq_q, heads, dim) over a long k/v (batch, seq_kv, heads,
    dim).  ``use_metal`` is ignored; ``dropout_p > 0`` with ``training`` raises
    NotImplementedError.

    ``chunk_size`` is validated (it must be positive, as in the reference) but does not pick
    the work split: the kernel cuts the key range into as many splits as fill the GPU and
    merges them by log-sum-exp.  Chunking never changes the mathematical result, so the output
    equals the reference's for any ``chunk_size`` up to floating-point rounding."""
    if q.ndim != 4:
        raise ValueError(f"Expected 4D tensors (batch, seq, heads, dim), got {q.ndim}D")
    if k.ndim != 4 or v.ndim != 4:
        raise ValueError("Expected 4D K and V tensors (batch, seq, heads, dim)")
    if chunk_size <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(f"Q/K/V dtype mismatch: Q={q.dtype}, K={k.dtype}, V={v.dtype}")
    if k.shape != v.shape or k.shape[0] != q.shape[0] or k.shape[2:] != q.shape[2:]:
        raise ValueError(f"Incompatible shapes: Q={tuple(q.shape)}, K={tuple(k.shape)}, V={tuple(v.shape)}")
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if dropout_p > 0.0 and training:
        raise NotImplementedError(
            "chunked_cross_attention: dropout needs the materialised attention matrix; "
            "call with dropout_p=0.0 or training=False")
    return attention_forward(q, k, v, layout="BSHD", scale=float(scale), causal=bool(causal),
                             kv_splits=0)


class ChunkedCrossAttention:
    """Chunked cross-attention module (chunked.py:410-469): heads, head_dim, chunk_size=1024,
    causal=False, scale = 1/sqrt(head_dim)."""

    def __init__(self, num_heads: int, head_dim: int, chunk_size: int = 1024,
                 causal: bool = False) -> None:
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.chunk_size = chunk_size
        self.causal = causal
        self.scale = 1.0 / math.sqrt(head_dim)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        return chunked_cross_attention(q, k, v, chunk_size=self.chunk_size, scale=self.scale,
                                       causal=self.causal)


def estimate_memory_savings(seq_q: int, seq_kv: int, num_heads: int, head_dim: int,
                            chunk_size: int, dtype_bytes: int = 4) -> Tuple[int, int, float]:
    """(full score-matrix bytes, one-chunk score-matrix bytes, ratio) as the reference reports
    them (chunked.py:472-512): seq_q*seq_kv*heads*bytes against seq_q*chunk*heads*bytes."""
    full = seq_q * seq_kv * num_heads * dtype_bytes
    chunk = seq_q * chunk_size * num_heads * dtype_bytes
    return full, chunk, full / max(chunk, 1)
