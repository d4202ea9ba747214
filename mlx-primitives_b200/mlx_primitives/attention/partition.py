"""Data-parallel split of one attention call over several GPUs by (batch, head) unit.

New component (the reference is single-device).  Attention is independent per (batch, head)
pair, so a call over B x H units shards without any exchange: the units, numbered
u = b * H + h, are cut into ``world_size`` contiguous ranges of equal size (the first
``U % world_size`` ranks take one more), and each rank computes its range in place through the
tensors' strides (no copy, no collective).  A range is at most three rectangles of
(batch, head): the tail of one batch, whole batches, the head of another; BASELINE configs 2,
3 and 4 at 1, 2, 4 and 8 ranks always give one rectangle, i.e. one kernel launch per rank.

``attention_units`` is the launch; ``flash_attention_shard``, ``sliding_window_attention_shard``
and ``chunked_cross_attention_shard`` apply the mask conventions of the public functions
(flash.py:52-254, sliding_window.py:227-312, chunked.py:43-126) to one rank's units.
"""

from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple

import torch

from ._core import _dims, attention_forward

__all__ = ["shard_units", "unit_blocks", "rank_pieces", "attention_units",
           "flash_attention_shard", "sliding_window_attention_shard",
           "chunked_cross_attention_shard"]


def shard_units(num_batch: int, num_heads: int, world_size: int, rank: int) -> range:
    """The contiguous range of units u = b * num_heads + h that ``rank`` computes.

    Every unit belongs to exactly one rank; ranges differ in length by at most one unit.
    """
    if num_batch < 0 or num_heads <= 0:
        raise ValueError(f"invalid shape: batch {num_batch}, heads {num_heads}")
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world size {world_size}")
    total = num_batch * num_heads
    base, extra = divmod(total, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def unit_blocks(units: range, num_heads: int) -> List[Tuple[int, int, int, int]]:
    """Rectangles (b0, b1, h0, h1) — batches [b0, b1) x heads [h0, h1) — that cover the unit
    range in order, at most three."""
    u0, u1 = units.start, units.stop
    blocks = []
    while u0 < u1:
        b, h = divmod(u0, num_heads)
        if h == 0 and u1 - u0 >= num_heads:  # whole batches
            nb = (u1 - u0) // num_heads
            blocks.append((b, b + nb, 0, num_heads))
            u0 += nb * num_heads
        else:  # part of one batch
            h1 = min(num_heads, h + (u1 - u0))
            blocks.append((b, b + 1, h, h1))
            u0 += h1 - h
    return blocks


def _view(t: torch.Tensor, layout: str, b0: int, b1: int, h0: int, h1: int) -> torch.Tensor:
    return t[b0:b1, h0:h1] if layout == "BHSD" else t[b0:b1, :, h0:h1]


def _group_pieces(h0: int, h1: int, group: int) -> List[Tuple[int, int]]:
    """Query-head ranges covering [h0, h1) in order, each either a whole number of K/V groups
    or a part of one group (at most three)."""
    pieces, s = [], h0
    while s < h1:
        if s % group == 0 and h1 - s >= group:  # whole groups
            e = s + (h1 - s) // group * group
        else:  # up to the end of this group
            e = min(h1, (s // group + 1) * group)
        pieces.append((s, e))
        s = e
    return pieces


def rank_pieces(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, units: range, layout: str
                ) -> List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Tuple[int, int, int, int]]]:
    """The independent attention calls that make up ``units``: (q view, k view, v view,
    (b0, b1, h0, h1)) per piece, views of the whole call's tensors (no copy).  A piece's query
    heads read exactly the K/V heads of its k/v views under the call's head grouping (query
    head h reads K/V head h // (H / H_kv)), so each piece is a complete attention call."""
    B, H, _, _ = _dims(q, layout)
    Bk, Hkv, _, _ = _dims(k, layout)
    if units.start < 0 or units.stop > B * H:
        raise ValueError(f"units {units} outside the {B * H} (batch, head) units of the call")
    if Hkv < 1 or H % Hkv:
        raise ValueError(f"num_heads ({H}) must be divisible by num_kv_heads ({Hkv})")
    group = H // Hkv
    pieces = []
    for b0, b1, h0, h1 in unit_blocks(units, H):
        kb0, kb1 = (0, 1) if Bk == 1 and B > 1 else (b0, b1)
        for g0, g1 in _group_pieces(h0, h1, group):
            # query heads [g0, g1) read K/V heads [g0 // group, (g1 - 1) // group + 1): either a
            # whole number of groups or part of one group (one K/V head for all of them)
            k0, k1 = g0 // group, (g1 - 1) // group + 1
            pieces.append((_view(q, layout, b0, b1, g0, g1), _view(k, layout, kb0, kb1, k0, k1),
                           _view(v, layout, kb0, kb1, k0, k1), (b0, b1, g0, g1)))
    return pieces


def attention_units(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, units: range, *,
                    layout: str, scale: float, causal: bool, window_left: int = -1,
                    window_right: int = -1, q_offset: int = 0, kv_offset: int = 0,
                    kv_splits: int = 0, out: Optional[torch.Tensor] = None,
                    backend: Optional[Callable] = None) -> torch.Tensor:
    """Attention of the (batch, head) units in ``units`` only, written into ``out``.

    q/k/v are the whole call's tensors (4-D, ``layout``); K/V may have fewer heads (grouped
    query heads) or one broadcast batch.  ``out`` (allocated when None: q's shape, dtype and
    layout) receives the units' rows; its other rows are left untouched.  Masks as in
    attention_forward.  ``backend`` (tests only) replaces the kernel launch: it is called with
    attention_forward's arguments plus ``out``.
    """
    pieces = rank_pieces(q, k, v, units, layout)
    if out is None:
        out = torch.empty(q.shape[:-1] + (v.shape[-1],), dtype=q.dtype, device=q.device)
    run = backend if backend is not None else attention_forward
    for qv, kv, vv, (b0, b1, h0, h1) in pieces:
        run(qv, kv, vv, layout=layout, scale=scale, causal=causal, window_left=window_left,
            window_right=window_right, q_offset=q_offset, kv_offset=kv_offset,
            kv_splits=kv_splits, out=_view(out, layout, b0, b1, h0, h1))
    return out


def _layout_str(layout) -> str:
    return layout.value if hasattr(layout, "value") else str(layout)


def flash_attention_shard(q, k, v, world_size: int, rank: int, scale: Optional[float] = None,
                          causal: bool = True, layout="BSHD", out=None) -> torch.Tensor:
    """This rank's share of flash_attention(q, k, v, scale, causal, layout=layout): the rows
    of its (batch, head) units in ``out`` (bottom-right aligned causal mask, as the public
    function)."""
    layout = _layout_str(layout)
    B, H, Sq, D = _dims(q, layout)
    Skv = _dims(k, layout)[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return attention_units(q, k, v, shard_units(B, H, world_size, rank), layout=layout,
                           scale=float(scale), causal=bool(causal),
                           q_offset=(Skv - Sq) if causal else 0, out=out)


def sliding_window_attention_shard(q, k, v, window_size: int, world_size: int, rank: int,
                                   scale: Optional[float] = None, causal: bool = True,
                                   out=None) -> torch.Tensor:
    """This rank's share of sliding_window_attention (BSHD; keys with |i - j| <= window_size,
    and j <= i when causal)."""
    B, H, S, D = _dims(q, "BSHD")
    if window_size < 0:
        raise ValueError(f"window_size must be >= 0, got {window_size}")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    w = int(window_size)
    return attention_units(q, k, v, shard_units(B, H, world_size, rank), layout="BSHD",
                           scale=float(scale), causal=bool(causal), window_left=w,
                           window_right=-1 if causal else w, out=out)


def chunked_cross_attention_shard(q, k, v, world_size: int, rank: int,
                                  scale: Optional[float] = None, causal: bool = False,
                                  out=None) -> torch.Tensor:
    """This rank's share of chunked_cross_attention (BSHD; top-left causal positions)."""
    B, H, Sq, D = _dims(q, "BSHD")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    return attention_units(q, k, v, shard_units(B, H, world_size, rank), layout="BSHD",
                           scale=float(scale), causal=bool(causal), out=out)
