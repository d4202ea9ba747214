"""Paged attention on B200 (drop-in for mlx_primitives/cache/paged_attention.py).

Same names, signatures and defaults as the reference: ``paged_attention``
(paged_attention.py:44-105), ``paged_attention_with_bias`` (323-384), ``get_alibi_slopes``
(17-41) and ``create_block_table_from_lengths`` (387-440), with torch tensors in place of
mx.array.  The reference gathers every block of every sequence into a dense
(batch, max_blocks * block_size, heads, dim) copy and runs masked dense attention; here one
call into libmlxp_attn.so (mlxp_paged_attn) reads the pool blocks in place through the block
table, splits long contexts over many CTAs and merges the shares by log-sum-exp.

Semantics follow the reference exactly: a key position t of sequence b counts when
t < context_lens[b] and its block-table slot holds an id >= 0; for more than one query row with
causal=True, query i sees positions t <= i (top-left); ALiBi adds slope[h] * (t - q_pos) with
q_pos = context_lens[b] for a single query row and i otherwise.  Differences, each where the
reference has no defined result: a query row with no admissible key returns zeros (the
reference's softmax gives NaN); block ids >= num_blocks count as missing (the reference would
index out of range).  Pools with fewer heads than q (heads h // (H / pool_heads) shared, as in
grouped-query attention) are accepted as an extension.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from .. import _lib

__all__ = [
    "get_alibi_slopes",
    "paged_attention",
    "paged_attention_with_bias",
    "create_block_table_from_lengths",
]

_HEAD_DIMS = (32, 64, 128)


def get_alibi_slopes(num_heads: int, device: Optional[torch.device] = None) -> torch.Tensor:
    """ALiBi slopes (2^(-8/num_heads))^(h+1) for h = 0..num_heads-1, float32 (shape (num_heads,)).

    The reference returns an mx.array; here a float32 tensor on ``device`` (default: host)."""
    ratio = 2 ** (-8 / num_heads)
    return torch.tensor([ratio ** (i + 1) for i in range(num_heads)], dtype=torch.float32,
                        device=device)


def _aligned(t: torch.Tensor) -> bool:
    es = t.element_size()
    return (t.data_ptr() % (4 * es) == 0 and t.stride(-1) == 1
            and all(s % 4 == 0 and s >= 0 for s in t.stride()[:-1]))


def _paged_forward(q, k_pool, v_pool, block_tables, context_lens, scale, block_size, causal,
                   alibi_slopes, kv_splits: int = 0) -> torch.Tensor:
    if q.ndim != 4:
        raise ValueError(f"q must be (batch, seq_q, num_heads, head_dim), got {tuple(q.shape)}")
    if k_pool.ndim != 4 or k_pool.shape != v_pool.shape:
        raise ValueError("k_pool and v_pool must both be (num_blocks, block_size, heads, head_dim)"
                         f", got {tuple(k_pool.shape)} and {tuple(v_pool.shape)}")
    B, Sq, H, D = q.shape
    num_blocks, bs, Hkv, Dk = k_pool.shape
    if bs != block_size:
        raise ValueError(f"pool block dimension ({bs}) must equal block_size ({block_size})")
    if Dk != D:
        raise ValueError(f"pool head_dim ({Dk}) must equal q's head_dim ({D})")
    if Hkv < 1 or H % Hkv:
        raise ValueError(f"num_heads ({H}) must be a multiple of the pool's heads ({Hkv})")
    if D not in _HEAD_DIMS:
        raise ValueError(f"paged attention supports head_dim {_HEAD_DIMS}, got {D}")
    if q.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {q.dtype}; expected float32, bfloat16 or float16")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise ValueError(f"q, k_pool and v_pool must share a dtype, got {q.dtype}, "
                         f"{k_pool.dtype}, {v_pool.dtype}")
    if block_tables.ndim != 2 or block_tables.shape[0] != B:
        raise ValueError(f"block_tables must be (batch, max_blocks), got {tuple(block_tables.shape)}")
    if context_lens.ndim != 1 or context_lens.shape[0] != B:
        raise ValueError(f"context_lens must be (batch,), got {tuple(context_lens.shape)}")
    if alibi_slopes is not None and tuple(alibi_slopes.shape) != (H,):
        raise ValueError(f"alibi_slopes must be (num_heads,) = ({H},), got {tuple(alibi_slopes.shape)}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)

    host = q.device.type == "cpu"
    dev = torch.device("cuda", torch.cuda.current_device()) if host else q.device
    if dev.type != "cuda":
        raise ValueError(f"tensors must be on a CUDA device (or the host), got {q.device}")
    if not host and (k_pool.device != dev or v_pool.device != dev):
        raise ValueError("q, k_pool and v_pool must be on the same device")
    q, k_pool, v_pool = (t.to(dev, non_blocking=True) for t in (q, k_pool, v_pool))
    q, k_pool, v_pool = (t if _aligned(t) else t.contiguous() for t in (q, k_pool, v_pool))
    bt = block_tables.to(dev, torch.int32).contiguous()
    ctx = context_lens.to(dev, torch.int32).contiguous()
    slopes = (alibi_slopes.to(dev, torch.float32).contiguous()
              if alibi_slopes is not None else None)
    out = torch.empty((B, Sq, H, D), dtype=q.dtype, device=dev)
    max_blocks = bt.shape[1]

    L = _lib.lib()
    dt = _lib.DTYPE_CODES[q.dtype]
    ps = k_pool.stride()
    if v_pool.stride() != ps:
        v_pool = v_pool.contiguous()
        if k_pool.stride() != v_pool.stride():
            k_pool = k_pool.contiguous()
        ps = k_pool.stride()
    with torch.cuda.device(dev):
        ws_bytes = L.mlxp_paged_attn_workspace_size(dt, B, H, Sq, D, Hkv, num_blocks, block_size,
                                                    max_blocks, kv_splits)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        rc = L.mlxp_paged_attn(
            q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), bt.data_ptr(), ctx.data_ptr(),
            slopes.data_ptr() if slopes is not None else None, out.data_ptr(), dt,
            B, H, Sq, D, Hkv, num_blocks, block_size, max_blocks,
            _lib.strides4(q, "BSHD"), (ctypes.c_int64 * 4)(*ps), bt.stride(0),
            _lib.strides4(out, "BSHD"), ctypes.c_float(scale), int(bool(causal)), kv_splits,
            ws.data_ptr() if ws is not None else None, ws_bytes, _lib.stream_handle(dev))
    _lib.check(rc, "mlxp_paged_attn")
    return out.cpu() if host else out


def paged_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: Optional[float] = None,
    block_size: int = 16,
    causal: bool = True,
    alibi_slopes: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Attention of q (batch, seq_q, num_heads, head_dim) over K/V stored in a block pool.

    k_pool, v_pool: (num_blocks, block_size, num_heads, head_dim); block_tables:
    (batch, max_blocks) int, -1 for unused slots; context_lens: (batch,) cached tokens per
    sequence.  seq_q == 1 is decode (the query sits at position context_lens[b]); seq_q > 1 is
    prefill (query i at position i, causal keeps positions <= i).  Returns q's shape and dtype.
    """
    return _paged_forward(q, k_pool, v_pool, block_tables, context_lens, scale, block_size,
                          causal, alibi_slopes)


def paged_attention_with_bias(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    attention_bias: Optional[torch.Tensor] = None,
    alibi_slopes: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    block_size: int = 16,
    causal: bool = True,
) -> torch.Tensor:
    """paged_attention with ALiBi slopes; a pre-computed ``attention_bias`` is not implemented
    (NotImplementedError, as in the reference) and giving both raises ValueError."""
    if attention_bias is not None and alibi_slopes is not None:
        raise ValueError("Cannot specify both attention_bias and alibi_slopes")
    if attention_bias is not None:
        raise NotImplementedError(
            "Pre-computed attention_bias support in paged_attention is not yet implemented. "
            "Use alibi_slopes parameter for ALiBi-style position encoding instead.")
    return paged_attention(q, k_pool, v_pool, block_tables, context_lens, scale, block_size,
                           causal, alibi_slopes=alibi_slopes)


def create_block_table_from_lengths(
    sequence_lengths: torch.Tensor,
    block_size: int,
    max_blocks: Optional[int] = None,
) -> torch.Tensor:
    """Block tables (batch, max_blocks) int32 giving sequence b the consecutive block ids
    cum[b] .. cum[b] + ceil(len_b / block_size) - 1 (cum = exclusive prefix sum), -1 after."""
    lens = torch.as_tensor(sequence_lengths).to(torch.int64)
    n = (lens + block_size - 1) // block_size
    mb = int(n.max().item()) if max_blocks is None else int(max_blocks)
    cum = torch.cumsum(n, 0) - n
    pos = torch.arange(mb, device=lens.device)[None, :]
    ids = cum[:, None] + pos
    return torch.where(pos < n[:, None], ids, torch.full_like(ids, -1)).to(torch.int32)
