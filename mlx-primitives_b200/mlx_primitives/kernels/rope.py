"""Rotary position embedding on B200 (drop-in for mlx_primitives/kernels/rope.py).

``precompute_rope_cache`` (rope.py:223-255), ``rope`` / ``fast_rope`` (rope.py:451-496,
350-381) and ``rope_qk`` / ``fast_rope_qk`` (rope.py:499-533, 384-448) with the reference's
names, shapes and half-split rotation: for x of shape (batch, seq, heads, head_dim), h =
head_dim / 2 and the row's position p = offset + s,
    y[..., :h] = x[..., :h] * cos[p] - x[..., h:] * sin[p]
    y[..., h:] = x[..., :h] * sin[p] + x[..., h:] * cos[p].
The rotation runs in libmlxp_attn.so (mlxp_rope / mlxp_rope_qk: one memory-bound kernel, Q and
K in one launch), in fp32, rounded once to the input dtype.  There is no CPU fallback: host
tensors are staged through the current CUDA device.  Differentiable in x (q, k): the rotation
is orthogonal, so its gradient is the same kernel with the sine table negated.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from .. import _lib

__all__ = ["precompute_rope_cache", "rope", "fast_rope", "rope_qk", "fast_rope_qk"]


def precompute_rope_cache(
    seq_len: int,
    head_dim: int,
    base: float = 10000.0,
    dtype: torch.dtype = torch.float32,
    device: Optional[torch.device] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin), each (seq_len, head_dim // 2): theta_i = base^(-i / (head_dim/2)),
    angle = position * theta_i, computed in fp32 (rope.py:240-253) and cast to ``dtype``."""
    half = head_dim // 2
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
            else torch.device("cpu")
    inv_freq = base ** (-torch.arange(0, half, dtype=torch.float32, device=device) / half)
    t = torch.arange(seq_len, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv_freq)
    return torch.cos(freqs).to(dtype), torch.sin(freqs).to(dtype)


def _device_of(*ts):
    for t in ts:
        if t.device.type == "cuda":
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("RoPE requires a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _f32_cache(c: torch.Tensor, dev: torch.device) -> torch.Tensor:
    return c.to(device=dev, dtype=torch.float32).contiguous()


def _check(x: torch.Tensor, name: str = "Input"):
    if x.ndim != 4:
        raise ValueError(f"{name} must be 4D (batch, seq_len, num_heads, head_dim), got {x.ndim}D")
    if x.shape[-1] % 2 != 0:
        raise ValueError(f"head_dim must be even, got {x.shape[-1]}")
    if x.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {x.dtype}")


def _rope_raw(xd: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, offset: int) -> torch.Tensor:
    """mlxp_rope on a device tensor with fp32 device caches."""
    if xd.stride(-1) != 1:
        xd = xd.contiguous()
    y = torch.empty_like(xd)
    B, S, H, D = xd.shape
    dev = xd.device
    with torch.cuda.device(dev):
        rc = _lib.lib().mlxp_rope(xd.data_ptr(), y.data_ptr(), _lib.DTYPE_CODES[xd.dtype], B, H, S,
                                  D, _lib.strides4(xd, "BSHD"), _lib.strides4(y, "BSHD"),
                                  cos.data_ptr(), sin.data_ptr(), cos.shape[0], int(offset),
                                  _lib.stream_handle(dev))
    _lib.check(rc, "mlxp_rope")
    return y


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin, offset):
        ctx.save_for_backward(cos, sin)
        ctx.offset = offset
        return _rope_raw(x, cos, sin, offset)

    @staticmethod
    def backward(ctx, gy):
        cos, sin = ctx.saved_tensors
        return _rope_raw(gy.contiguous(), cos, -sin, ctx.offset), None, None, None


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in ts)


def fast_rope(x: torch.Tensor, cos_cache: torch.Tensor, sin_cache: torch.Tensor,
              offset: int = 0) -> torch.Tensor:
    """RoPE of x (batch, seq_len, num_heads, head_dim) at positions offset .. offset+seq_len-1."""
    _check(x)
    dev = _device_of(x)
    host = x.device.type == "cpu"
    xd = x.to(dev) if host else x
    cos, sin = _f32_cache(cos_cache, dev), _f32_cache(sin_cache, dev)
    if cos.shape != sin.shape or cos.ndim != 2 or cos.shape[1] != x.shape[-1] // 2:
        raise ValueError("cos/sin caches must both be (max_seq, head_dim // 2)")
    if _needs_grad(x):
        if host:
            raise NotImplementedError("RoPE gradients need CUDA tensors")
        return _RopeFn.apply(xd, cos.detach(), sin.detach(), int(offset))
    y = _rope_raw(xd, cos, sin, offset)
    return y.cpu() if host else y


def rope(x: torch.Tensor, cos_cache: torch.Tensor, sin_cache: torch.Tensor, offset: int = 0,
         use_metal: bool = True) -> torch.Tensor:
    """rope.py:451-496: every path is the B200 kernel (``use_metal`` is accepted for API
    compatibility)."""
    return fast_rope(x, cos_cache, sin_cache, offset)


def fast_rope_qk(q: torch.Tensor, k: torch.Tensor, cos_cache: torch.Tensor,
                 sin_cache: torch.Tensor, offset: int = 0,
                 k_offset: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """RoPE of Q and K in one launch.  The reference requires equal shapes here
    (rope.py:384-448); K may also have its own head count, length and position offset
    (``k_offset``, default ``offset``), which fused_rope_attention uses for KV caches."""
    _check(q, "Q")
    _check(k, "K")
    if q.shape[0] != k.shape[0] or q.shape[-1] != k.shape[-1] or q.dtype != k.dtype:
        raise ValueError(f"Q and K must agree in batch, head_dim and dtype, got {tuple(q.shape)} "
                         f"and {tuple(k.shape)}")
    dev = _device_of(q, k)
    host = q.device.type == "cpu"
    qd, kd = (t.to(dev) if t.device.type == "cpu" else t for t in (q, k))
    cos, sin = _f32_cache(cos_cache, dev), _f32_cache(sin_cache, dev)
    if cos.shape != sin.shape or cos.ndim != 2 or cos.shape[1] != q.shape[-1] // 2:
        raise ValueError("cos/sin caches must both be (max_seq, head_dim // 2)")
    k_off = int(offset if k_offset is None else k_offset)
    if _needs_grad(q, k):
        if host:
            raise NotImplementedError("RoPE gradients need CUDA tensors")
        return _RopeQKFn.apply(qd, kd, cos.detach(), sin.detach(), int(offset), k_off)
    qo, ko = _rope_qk_raw(qd, kd, cos, sin, int(offset), k_off)
    return (qo.cpu(), ko.cpu()) if host else (qo, ko)


def _rope_qk_raw(qd, kd, cos, sin, offset: int, k_offset: int):
    """mlxp_rope_qk on device tensors with fp32 device caches."""
    qd, kd = (t if t.stride(-1) == 1 else t.contiguous() for t in (qd, kd))
    qo, ko = torch.empty_like(qd), torch.empty_like(kd)
    B, Sq, Hq, D = qd.shape
    _, Sk, Hk, _ = kd.shape
    dev = qd.device
    with torch.cuda.device(dev):
        rc = _lib.lib().mlxp_rope_qk(
            qd.data_ptr(), kd.data_ptr(), qo.data_ptr(), ko.data_ptr(), _lib.DTYPE_CODES[qd.dtype],
            B, Hq, Hk, Sq, Sk, D, _lib.strides4(qd, "BSHD"), _lib.strides4(kd, "BSHD"),
            _lib.strides4(qo, "BSHD"), _lib.strides4(ko, "BSHD"), cos.data_ptr(), sin.data_ptr(),
            cos.shape[0], offset, k_offset, _lib.stream_handle(dev))
    _lib.check(rc, "mlxp_rope_qk")
    return qo, ko


class _RopeQKFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, cos, sin, offset, k_offset):
        ctx.save_for_backward(cos, sin)
        ctx.offsets = (offset, k_offset)
        return _rope_qk_raw(q, k, cos, sin, offset, k_offset)

    @staticmethod
    def backward(ctx, gq, gk):
        cos, sin = ctx.saved_tensors
        gq = torch.zeros_like(gq) if gq is None else gq.contiguous()
        gk = torch.zeros_like(gk) if gk is None else gk.contiguous()
        dq, dk = _rope_qk_raw(gq, gk, cos, -sin, *ctx.offsets)
        return dq, dk, None, None, None, None


def rope_qk(q: torch.Tensor, k: torch.Tensor, cos_cache: torch.Tensor, sin_cache: torch.Tensor,
            offset: int = 0, use_metal: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """rope.py:499-533 (``use_metal`` accepted for API compatibility)."""
    return fast_rope_qk(q, k, cos_cache, sin_cache, offset)
