"""flash_attention / FlashAttention on B200 (drop-in for mlx_primitives/attention/flash.py).

Same names, signatures, defaults, validation and error types as the reference
(flash.py:52-254, 581-688); torch tensors replace mx.array.  The three-way dispatch of the
reference (SDPA, Metal kernel, Python tiled loop) is replaced by one call into the sm_100a
library: a tcgen05 tensor-core kernel for bf16/fp16 and a CUDA-core kernel for fp32.  The
output has the input's dtype and layout, as on the reference's SDPA path.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple, Union

import torch

from ..constants import Layout
from ._core import attention_forward

__all__ = ["flash_attention", "FlashAttention", "get_optimal_flash_config"]


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: Optional[float] = None,
    causal: bool = True,
    block_q: int = 32,
    block_kv: int = 32,
    use_metal: bool = True,
    dropout_p: float = 0.0,
    training: bool = True,
    layout: Union[str, Layout] = Layout.BSHD,
) -> torch.Tensor:
    """Exact softmax(scale * Q K^T + causal mask) V without materialising the score matrix.

    Args mirror the reference (flash.py:52-65): q/k/v are 4-D in ``layout`` ("BSHD" default
    or "BHSD"); ``scale`` defaults to 1/sqrt(head_dim); ``causal`` masks keys after the query,
    aligned bottom-right when Sq != Skv (utils/masking.py:14-66); ``block_q``, ``block_kv`` and
    ``use_metal`` are accepted for compatibility and ignored (the B200 kernel's tiles are fixed).

    Raises ValueError on bad ranks, layouts, mismatched shapes or dtypes (flash.py:123-169).
    ``dropout_p > 0`` with ``training`` on the BSHD path raises NotImplementedError: dropout
    needs the materialised weight matrix, which this library never builds.  On the BHSD path
    the reference ignores dropout (flash.py:172-192 returns before the dropout check), and so
    does this function.
    """
    if q.ndim != 4:
        raise ValueError(f"Expected 4D tensors, got {q.ndim}D")
    if k.ndim != 4:
        raise ValueError(f"Expected K to be 4D tensor, got {k.ndim}D")
    if v.ndim != 4:
        raise ValueError(f"Expected V to be 4D tensor, got {v.ndim}D")
    if isinstance(layout, str) and layout not in (Layout.BSHD.value, Layout.BHSD.value):
        raise ValueError(
            f"layout must be Layout.BSHD or Layout.BHSD (or 'BSHD'/'BHSD'), got '{layout}'")
    layout = Layout(layout)

    if layout == Layout.BSHD:
        (qb, qs, qh, qd), (kb, ks, kh, kd), (vb, vs, vh, vd) = q.shape, k.shape, v.shape
    else:
        (qb, qh, qs, qd), (kb, kh, ks, kd), (vb, vh, vs, vd) = q.shape, k.shape, v.shape
    if qb != kb or qb != vb:
        raise ValueError(f"Batch size mismatch: Q={qb}, K={kb}, V={vb}")
    if qh != kh or qh != vh:
        raise ValueError(f"Number of heads mismatch: Q={qh}, K={kh}, V={vh}")
    if qd != kd:
        raise ValueError(f"Head dimension mismatch between Q and K: Q={qd}, K={kd}")
    if ks != vs:
        raise ValueError(f"Sequence length mismatch between K and V: K={ks}, V={vs}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError(
            f"Q/K/V dtype mismatch: Q={q.dtype}, K={k.dtype}, V={v.dtype}. "
            "All tensors must have the same dtype to ensure numerical stability.")
    if vd != qd:
        raise ValueError(f"Head dimension mismatch between Q and V: Q={qd}, V={vd}")
    if scale is None:
        scale = 1.0 / math.sqrt(qd)
    if layout == Layout.BSHD and dropout_p > 0.0 and training:
        raise NotImplementedError(
            "flash_attention: dropout needs the materialised attention matrix; the B200 "
            "kernels never build it (call with dropout_p=0.0 or training=False)")
    return attention_forward(
        q, k, v, layout=layout.value, scale=float(scale), causal=bool(causal),
        q_offset=(ks - qs) if causal else 0)


class FlashAttention:
    """Flash Attention module (flash.py:581-647): stores heads, head_dim, causal and
    scale = 1/sqrt(head_dim); block sizes default to 32 (head_dim <= 64) or 16 and are kept
    only for API compatibility.  Calls flash_attention with BSHD tensors."""

    def __init__(self, num_heads: int, head_dim: int, causal: bool = True,
                 block_q: Optional[int] = None, block_kv: Optional[int] = None) -> None:
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.causal = causal
        self.scale = 1.0 / math.sqrt(head_dim)
        self.block_q = block_q if block_q is not None else (32 if head_dim <= 64 else 16)
        self.block_kv = block_kv if block_kv is not None else (32 if head_dim <= 64 else 16)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        return flash_attention(q, k, v, scale=self.scale, causal=self.causal,
                               block_q=self.block_q, block_kv=self.block_kv)


def get_optimal_flash_config(seq_len: int, head_dim: int, num_heads: int) -> Tuple[int, int]:
    """Block-size hint of the reference (flash.py:650-688), derived from a 26 KB three-tile
    shared-memory budget with a (head_dim + 4)-float row pitch.  Returned unchanged for API
    compatibility; the B200 kernel uses fixed 256x128 tiles whatever the hint."""
    per_row = (head_dim + 4) * 4
    cap = (26000 // 3) // per_row
    base = 32 if head_dim <= 64 else (16 if head_dim <= 128 else 8)
    block = min(base, cap, seq_len)
    return block, block
