"""The one forward entry point every public attention function of this package goes through.

It replaces the reference's three-way dispatch (MLX SDPA -> Metal kernel -> Python tiled loop,
mlx_primitives/attention/flash.py:172-254, sliding_window.py:288-312, chunked.py:113-126) with
a single call into libmlxp_attn.so: bf16/fp16 inputs run the tcgen05 tensor-core kernel, fp32
inputs the CUDA-core kernel.  Nothing here computes attention on the CPU; host tensors are
staged through the current CUDA device and the result is copied back.
"""

from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib

_TC_HEAD_DIMS = (64, 128)
_F32_HEAD_DIMS = (32, 64, 128)
MAX_HEAD_DIM = 128


def _padded_head_dim(d: int, dtype: torch.dtype) -> int:
    dims = _F32_HEAD_DIMS if dtype == torch.float32 else _TC_HEAD_DIMS
    for cand in dims:
        if d <= cand:
            return cand
    raise ValueError(f"head_dim={d} exceeds the kernel limit of {MAX_HEAD_DIM}")


def _dims(t: torch.Tensor, layout: str):
    if layout == "BHSD":
        b, h, s, d = t.shape
    else:
        b, s, h, d = t.shape
    return b, h, s, d


def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, layout: str,
                      scale: float, causal: bool, window_left: int = -1, window_right: int = -1,
                      q_offset: int = 0, kv_offset: int = 0, kv_splits: int = 1,
                      return_lse: bool = False):
    """O = softmax(scale * Q K^T + mask) V for 4-D q/k/v in `layout` ("BSHD" or "BHSD").

    Masking is in absolute positions (qpos = i + q_offset, kpos = j + kv_offset): causal keeps
    kpos <= qpos, window_left keeps qpos - kpos <= window_left, window_right keeps
    kpos - qpos <= window_right (-1 = unbounded).  Returns O with q's layout and dtype and,
    if return_lse, the fp32 log-sum-exp [B, H, Sq].
    """
    if q.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {q.dtype}; expected float32, bfloat16 or float16")
    host = q.device.type == "cpu"
    if host:
        if not torch.cuda.is_available():
            raise RuntimeError("attention requires a CUDA device (there is no CPU fallback)")
        dev = torch.device("cuda", torch.cuda.current_device())
        q, k, v = (t.to(dev, non_blocking=True) for t in (q, k, v))
    elif q.device.type != "cuda":
        raise ValueError(f"tensors must be on a CUDA device (or the host), got {q.device}")
    if k.device != q.device or v.device != q.device:
        raise ValueError("q, k and v must be on the same device")

    B, H, Sq, D = _dims(q, layout)
    _, Hkv, Skv, _ = _dims(k, layout)
    if Hkv != H and (Hkv < 1 or H % Hkv):
        raise ValueError(f"num_heads ({H}) must be divisible by num_kv_heads ({Hkv})")
    Dp = _padded_head_dim(D, q.dtype)
    if Dp != D:
        # Zero-padding the head dimension leaves Q K^T unchanged; the extra output columns
        # (zero V columns) are dropped below.  The scale was fixed from the true head_dim.
        pad = (0, Dp - D)
        q, k, v = (torch.nn.functional.pad(t, pad) for t in (q, k, v))
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, v))

    shape = (B, H, Sq, Dp) if layout == "BHSD" else (B, Sq, H, Dp)
    out = torch.empty(shape, dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, Sq), dtype=torch.float32, device=q.device) if return_lse else None

    L = _lib.lib()
    dt = _lib.DTYPE_CODES[q.dtype]
    with torch.cuda.device(q.device):
        ws_bytes = L.mlxp_attn_workspace_size(dt, B, H, Sq, Skv, Dp, int(causal), window_left,
                                              window_right, q_offset, kv_offset, kv_splits)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        common = (_lib.strides4(q, layout), _lib.strides4(k, layout), _lib.strides4(v, layout),
                  _lib.strides4(out, layout), ctypes.c_float(scale), int(causal), window_left,
                  window_right, q_offset, kv_offset, kv_splits,
                  ws.data_ptr() if ws is not None else None, ws_bytes,
                  _lib.stream_handle(q.device))
        lse_ptr = lse.data_ptr() if lse is not None else None
        if Hkv == H:
            rc = L.mlxp_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 lse_ptr, dt, B, H, Sq, Skv, Dp, *common)
            what = "mlxp_attn_fwd"
        else:  # grouped-query / multi-query: H_kv K/V heads shared by the H query heads
            rc = L.mlxp_attn_fwd_gqa(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                     lse_ptr, dt, B, H, Hkv, Sq, Skv, Dp, *common)
            what = "mlxp_attn_fwd_gqa"
    _lib.check(rc, what)
    if Dp != D:
        out = out[..., :D]
    if host:
        out = _to_host(out)
        lse = _to_host(lse) if lse is not None else None
    return (out, lse) if return_lse else out


def _to_host(t: torch.Tensor) -> torch.Tensor:
    """Device -> pinned host copy on the current stream, then wait for it."""
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t, non_blocking=True)
    torch.cuda.current_stream(t.device).synchronize()
    return h


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
