"""RoPE + flash attention on B200 (drop-in for mlx_primitives/kernels/fused_rope_attention.py).

``fused_rope_attention`` (fused_rope_attention.py:939-985), ``fast_fused_rope_attention``
(:637-733) and ``FusedRoPEFlashAttention`` (:988-1080): the reference rotates Q and K inside
its attention kernel (fused_rope_attention.py:52-198).  Here too RoPE and attention are one
launch (mlxp_rope_attn_fwd): the persistent tcgen05 attention kernel also runs rotation work
items that rotate 256-row chunks of Q and K into an L2-resident workspace one scheduling group
ahead of the attention items that read them.  Where that launch does not apply (grouped K/V
heads, head_dims other than 64 and 128, fp32, autograd) Q and K are rotated by one RoPE launch
(mlxp_rope_qk) and attention runs on the rotated tensors — the same arithmetic, bit for bit.
Q/K/V are (batch, seq, heads, head_dim); Q positions start at ``q_offset``, K positions at
``kv_offset``; the causal mask is the reference's: bottom-right aligned (SDPA "causal"),
independent of the offsets.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch import nn

import ctypes

from .. import _lib
from ..attention._core import attention_forward
from .rope import fast_rope_qk, precompute_rope_cache

__all__ = ["fused_rope_attention", "fast_fused_rope_attention", "FusedRoPEFlashAttention"]

_CACHE_LIMIT = 8
_rope_caches = {}


def _default_cache(max_pos: int, head_dim: int, base: float, device):
    """fp32 cos/sin tables, kept per (length, head_dim, base, device) like the reference's
    automatic cache management, so repeated calls do not recompute them."""
    key = (max_pos, head_dim, float(base), str(device))
    hit = _rope_caches.get(key)
    if hit is None:
        if len(_rope_caches) >= _CACHE_LIMIT:
            _rope_caches.pop(next(iter(_rope_caches)))
        hit = _rope_caches[key] = precompute_rope_cache(max_pos, head_dim, base=base,
                                                        device=device)
    return hit


def fast_fused_rope_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: Optional[float] = None,
    cos_cache: Optional[torch.Tensor] = None,
    sin_cache: Optional[torch.Tensor] = None,
    rope_base: float = 10000.0,
    q_offset: int = 0,
    kv_offset: int = 0,
    causal: bool = False,
    use_tiled: Optional[bool] = None,
) -> torch.Tensor:
    """RoPE on Q and K, then attention (fused_rope_attention.py:637-733)."""
    if q.ndim != 4:
        raise ValueError(f"Q must be 4D (batch, seq_q, num_heads, head_dim), got {q.ndim}D")
    if k.ndim != 4:
        raise ValueError(f"K must be 4D (batch, seq_kv, num_heads, head_dim), got {k.ndim}D")
    if v.ndim != 4:
        raise ValueError(f"V must be 4D (batch, seq_kv, num_heads, head_dim), got {v.ndim}D")
    _, seq_q, _, head_dim = q.shape
    seq_kv = k.shape[1]
    if head_dim % 2 != 0:
        raise ValueError(f"head_dim must be even for RoPE, got {head_dim}")
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    if q.device.type == "cpu":
        # host tensors: one copy in (from pinned memory when the caller pinned it), RoPE and
        # attention on the device, one copy out into pinned memory
        if not torch.cuda.is_available():
            raise RuntimeError("fused_rope_attention requires a CUDA device (no CPU fallback)")
        dev = torch.device("cuda", torch.cuda.current_device())
        qd, kd, vd = (t.to(dev, non_blocking=True) for t in (q, k, v))
        out = fast_fused_rope_attention(qd, kd, vd, scale, cos_cache, sin_cache, rope_base,
                                        q_offset, kv_offset, causal, use_tiled)
        host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        host.copy_(out, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return host
    if cos_cache is None or sin_cache is None:
        max_pos = max(seq_q + q_offset, seq_kv + kv_offset)
        dev = q.device if q.device.type == "cuda" else torch.device(
            "cuda", torch.cuda.current_device())
        cos_cache, sin_cache = _default_cache(max_pos, head_dim, rope_base, dev)
    mask_off = (seq_kv - seq_q) if causal else 0
    if _single_launch_applies(q, k, v, cos_cache, sin_cache):
        return _rope_attention_launch(q, k, v, cos_cache, sin_cache, q_offset, kv_offset,
                                      float(scale), bool(causal), mask_off)
    q_rot, k_rot = fast_rope_qk(q, k, cos_cache, sin_cache, q_offset, k_offset=kv_offset)
    return attention_forward(q_rot, k_rot, v, layout="BSHD", scale=float(scale),
                             causal=bool(causal), q_offset=mask_off)


def _single_launch_applies(q, k, v, cos_cache, sin_cache) -> bool:
    """mlxp_rope_attn_fwd covers bf16/fp16 CUDA tensors with head_dim 64 or 128, as many K/V
    heads as query heads, 16-byte aligned rows, fp32 tables, and no gradient to record."""
    if q.device.type != "cuda" or q.dtype not in (torch.bfloat16, torch.float16):
        return False
    if q.shape[-1] not in (64, 128) or k.shape[2] != q.shape[2] or k.shape[0] != q.shape[0]:
        return False
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        return False
    if cos_cache.dtype != torch.float32 or sin_cache.dtype != torch.float32:
        return False
    for t in (q, k):
        if t.stride(-1) != 1 or t.data_ptr() % 16 or any(st % 8 for st in t.stride()[:3]):
            return False
    return True


def _rope_attention_launch(q, k, v, cos_cache, sin_cache, q_offset, kv_offset, scale, causal,
                           mask_off):
    """One mlxp_rope_attn_fwd launch on (batch, seq, heads, head_dim) tensors."""
    B, Sq, H, D = q.shape
    Skv = k.shape[1]
    v = v if v.stride(-1) == 1 else v.contiguous()
    cos_cache, sin_cache = (t.contiguous() for t in (cos_cache, sin_cache))
    out = torch.empty((B, Sq, H, D), dtype=q.dtype, device=q.device)
    L = _lib.lib()
    dt = _lib.DTYPE_CODES[q.dtype]
    with torch.cuda.device(q.device):
        ws_bytes = L.mlxp_rope_attn_workspace_size(dt, B, H, Sq, Skv, D, int(causal), -1, -1,
                                                   mask_off, 0, 0)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        rc = L.mlxp_rope_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), None,
                                  dt, B, H, Sq, Skv, D, _lib.strides4(q, "BSHD"),
                                  _lib.strides4(k, "BSHD"), _lib.strides4(v, "BSHD"),
                                  _lib.strides4(out, "BSHD"), cos_cache.data_ptr(),
                                  sin_cache.data_ptr(), cos_cache.shape[0], q_offset, kv_offset,
                                  ctypes.c_float(scale), int(causal), -1, -1, mask_off, 0, 0,
                                  ws.data_ptr(), ws_bytes, _lib.stream_handle(q.device))
    _lib.check(rc, "mlxp_rope_attn_fwd")
    return out


def fused_rope_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: Optional[float] = None,
    cos_cache: Optional[torch.Tensor] = None,
    sin_cache: Optional[torch.Tensor] = None,
    rope_base: float = 10000.0,
    q_offset: int = 0,
    kv_offset: int = 0,
    causal: bool = False,
    use_metal: bool = True,
) -> torch.Tensor:
    """fused_rope_attention.py:939-985 (``use_metal`` accepted for API compatibility)."""
    return fast_fused_rope_attention(q, k, v, scale, cos_cache, sin_cache, rope_base, q_offset,
                                     kv_offset, causal)


class FusedRoPEFlashAttention(nn.Module):
    """Attention module with Q/K/V/out projections, RoPE and a KV cache
    (fused_rope_attention.py:988-1080)."""

    def __init__(self, dims: int, num_heads: int, head_dim: Optional[int] = None,
                 max_seq_len: int = 8192, rope_base: float = 10000.0, causal: bool = False,
                 bias: bool = False):
        super().__init__()
        self.dims = dims
        self.num_heads = num_heads
        self.head_dim = head_dim or dims // num_heads
        self.max_seq_len = max_seq_len
        self.rope_base = rope_base
        self.causal = causal
        self.scale = 1.0 / math.sqrt(self.head_dim)
        inner = self.num_heads * self.head_dim
        self.q_proj = nn.Linear(dims, inner, bias=bias)
        self.k_proj = nn.Linear(dims, inner, bias=bias)
        self.v_proj = nn.Linear(dims, inner, bias=bias)
        self.out_proj = nn.Linear(inner, dims, bias=bias)

    def forward(self, queries: torch.Tensor, keys: Optional[torch.Tensor] = None,
                values: Optional[torch.Tensor] = None,
                cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                offset: int = 0) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
        """(batch, seq_q, dims) -> ((batch, seq_q, dims), (k, v) cache).  As in the reference,
        queries start at position ``offset`` and the (cached + new) keys at position 0."""
        if keys is None:
            keys = queries
        if values is None:
            values = keys
        B, Sq, _ = queries.shape
        Skv = keys.shape[1]
        q = self.q_proj(queries).reshape(B, Sq, self.num_heads, self.head_dim)
        k = self.k_proj(keys).reshape(B, Skv, self.num_heads, self.head_dim)
        v = self.v_proj(values).reshape(B, Skv, self.num_heads, self.head_dim)
        if cache is not None:
            k = torch.cat([cache[0], k], dim=1)
            v = torch.cat([cache[1], v], dim=1)
        new_cache = (k, v)
        out = fused_rope_attention(q, k, v, scale=self.scale, rope_base=self.rope_base,
                                   q_offset=offset, kv_offset=0, causal=self.causal)
        return self.out_proj(out.reshape(B, Sq, -1)), new_cache
