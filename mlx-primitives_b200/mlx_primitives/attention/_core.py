"""The one forward entry point every public attention function of this package goes through.

It replaces the reference's three-way dispatch (MLX SDPA -> Metal kernel -> Python tiled loop,
mlx_primitives/attention/flash.py:172-254, sliding_window.py:288-312, chunked.py:113-126) with
a single call into libmlxp_attn.so: bf16/fp16 inputs run the tcgen05 tensor-core kernel, fp32
inputs the CUDA-core kernel.  Nothing here computes attention on the CPU; host tensors are
staged through the current CUDA device (pipelined in batch chunks) and the result is copied
back into pinned host memory.
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
                      q_offset: int = 0, kv_offset: int = 0, kv_splits: int = 0,
                      return_lse: bool = False, out: torch.Tensor | None = None,
                      mask: torch.Tensor | None = None):
    """O = softmax(scale * Q K^T + mask) V for 4-D q/k/v in `layout` ("BSHD" or "BHSD").

    Masking is in absolute positions (qpos = i + q_offset, kpos = j + kv_offset): causal keeps
    kpos <= qpos, window_left keeps qpos - kpos <= window_left, window_right keeps
    kpos - qpos <= window_right (-1 = unbounded).  kv_splits: 0 = the library's choice of key
    splits (merged by log-sum-exp), 1 = none, n = n.  Returns O with q's layout and dtype and,
    if return_lse, the fp32 log-sum-exp [B, H, Sq].

    ``out`` (optional): a tensor of O's shape, dtype and layout, e.g. a slice of a larger
    output, that receives the result in place and is returned.

    ``mask`` (optional): an additive score mask broadcastable to (B, H, Sq, Skv) — the custom
    mask of the reference's gqa/mqa attention, added to scale * Q K^T (booleans count 0/1, as
    in the reference's addition); -inf excludes a key.  Forward only.

    Differentiable: when autograd records and q, k or v requires grad, the backward runs the
    library's backward kernels (mlxp_attn_bwd) from the saved O and log-sum-exp.
    """
    kw = dict(layout=layout, scale=scale, causal=causal, window_left=window_left,
              window_right=window_right, q_offset=q_offset, kv_offset=kv_offset,
              kv_splits=kv_splits)
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        if out is not None:
            raise ValueError("out= cannot be used while recording gradients")
        if mask is not None:
            raise NotImplementedError("gradients through a custom attention mask are not "
                                      "supported (the backward kernels take causal/window masks)")
        if q.device.type != "cuda":
            raise NotImplementedError("attention gradients need CUDA tensors (host tensors are "
                                      "only staged for the forward)")
        out, lse = _AttentionFn.apply(q, k, v, kw)
        return (out, lse) if return_lse else out
    return _forward_impl(q, k, v, return_lse=return_lse, out=out, mask=mask, **kw)


def _prepare_mask(mask, B: int, H: int, Sq: int, Skv: int, device) -> torch.Tensor:
    """fp32 view of `mask` broadcast to (B, H, Sq, Skv) that the kernels can read: unit key
    stride, rows and base on 16 bytes.  Broadcast dims stay stride 0 (a (Sq, Skv) mask is not
    expanded over batch and heads); rows are padded to a multiple of 4 keys when needed."""
    m = torch.as_tensor(mask, device=device)
    m = m.to(torch.float32)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    if m.dim() != 4:
        raise ValueError(f"mask must broadcast to (batch, heads, seq_q, seq_kv), got {tuple(m.shape)}")
    try:
        torch.broadcast_shapes(tuple(m.shape), (B, H, Sq, Skv))
    except RuntimeError as e:
        raise ValueError(f"mask of shape {tuple(mask.shape)} does not broadcast to "
                         f"(batch, heads, seq_q, seq_kv) = {(B, H, Sq, Skv)}") from e
    small = m.expand(*(s if s != 1 else 1 for s in m.shape))
    ok = (small.stride(3) == 1 or small.shape[3] == 1) and small.data_ptr() % 16 == 0 and \
        all(st % 4 == 0 for st, n in zip(small.stride()[:3], small.shape[:3]) if n > 1)
    if not ok or small.shape[3] != Skv:
        pad = -(-Skv // 4) * 4
        buf = torch.zeros(tuple(small.shape[:3]) + (pad,), dtype=torch.float32, device=device)
        buf[..., :Skv] = small
        small = buf
    return small.expand(B, H, Sq, small.shape[3])[..., :Skv]


class _AttentionFn(torch.autograd.Function):
    """Forward through the attention kernels, backward through mlxp_attn_bwd."""

    @staticmethod
    def forward(ctx, q, k, v, kw):
        out, lse = _forward_impl(q, k, v, return_lse=True, **kw)
        ctx.kw = kw
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, dout, _dlse):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(q, k, v, out, lse, dout, **ctx.kw)
        return dq, dk, dv, None


_BWD_HEAD_DIMS = (32, 64, 128)


def attention_backward(q, k, v, out, lse, dout, *, layout: str, scale: float, causal: bool,
                       window_left: int = -1, window_right: int = -1, q_offset: int = 0,
                       kv_offset: int = 0, kv_splits: int = 0):
    """dQ, dK, dV of attention_forward (same arguments) from its output and log-sum-exp."""
    B, H, Sq, D = _dims(q, layout)
    _, Hkv, Skv, _ = _dims(k, layout)
    Dp = next((c for c in _BWD_HEAD_DIMS if D <= c), None)
    if Dp is None:
        raise ValueError(f"head_dim={D} exceeds the kernel limit of {MAX_HEAD_DIM}")
    if dout is None:
        dout = torch.zeros_like(out)
    dout = dout.to(q.dtype)
    ts = [q, k, v, out, dout]
    if Dp != D:
        ts = [torch.nn.functional.pad(t, (0, Dp - D)) for t in ts]
    q_, k_, v_, o_, do_ = (t if t.stride(-1) == 1 else t.contiguous() for t in ts)
    do_ = do_.contiguous()
    dq = torch.empty(q_.shape, dtype=q.dtype, device=q.device)
    dk = torch.empty(k_.shape, dtype=k.dtype, device=q.device)
    dv = torch.empty(v_.shape, dtype=v.dtype, device=q.device)
    L = _lib.lib()
    dt = _lib.DTYPE_CODES[q.dtype]
    with torch.cuda.device(q.device):
        ws_bytes = L.mlxp_attn_bwd_workspace_size(dt, B, H, Sq, Skv, Dp)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        st = [_lib.strides4(t, layout) for t in (q_, k_, v_, o_, do_, dq, dk, dv)]
        rc = L.mlxp_attn_bwd(q_.data_ptr(), k_.data_ptr(), v_.data_ptr(), o_.data_ptr(),
                             do_.data_ptr(), lse.contiguous().data_ptr(), dq.data_ptr(),
                             dk.data_ptr(), dv.data_ptr(), dt, B, H, Hkv, Sq, Skv, Dp, *st,
                             ctypes.c_float(scale), int(causal), window_left, window_right,
                             q_offset, kv_offset, ws.data_ptr(), ws_bytes,
                             _lib.stream_handle(q.device))
    _lib.check(rc, "mlxp_attn_bwd")
    if Dp != D:
        dq, dk, dv = dq[..., :D], dk[..., :D], dv[..., :D]
    return dq, dk, dv


def _forward_impl(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, layout: str,
                  scale: float, causal: bool, window_left: int = -1, window_right: int = -1,
                  q_offset: int = 0, kv_offset: int = 0, kv_splits: int = 0,
                  return_lse: bool = False, out: torch.Tensor | None = None,
                  mask: torch.Tensor | None = None):
    """The forward launch.  ``out``: a tensor of the output's shape, dtype and layout (any
    strides, e.g. a slice of a larger output) that receives the result; it is returned."""
    if q.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {q.dtype}; expected float32, bfloat16 or float16")
    if q.device.type == "cpu" and mask is not None:
        # host tensors with a mask: staged whole (the mask need not split by batch)
        if not torch.cuda.is_available():
            raise RuntimeError("attention requires a CUDA device (there is no CPU fallback)")
        dev = torch.device("cuda", torch.cuda.current_device())
        res = _forward_impl(*(t.to(dev, non_blocking=True) for t in (q, k, v)), layout=layout,
                            scale=scale, causal=causal, window_left=window_left,
                            window_right=window_right, q_offset=q_offset, kv_offset=kv_offset,
                            kv_splits=kv_splits, return_lse=return_lse,
                            mask=torch.as_tensor(mask).to(dev))
        res = tuple(r.cpu() for r in res) if return_lse else res.cpu()
        if out is None:
            return res
        out.copy_(res[0] if return_lse else res)
        return (out, res[1]) if return_lse else out
    if q.device.type == "cpu":
        res = _host_attention(q, k, v, layout=layout, scale=scale, causal=causal,
                              window_left=window_left, window_right=window_right,
                              q_offset=q_offset, kv_offset=kv_offset, kv_splits=kv_splits,
                              return_lse=return_lse)
        if out is None:
            return res
        out.copy_(res[0] if return_lse else res)
        return (out, res[1]) if return_lse else out
    if q.device.type != "cuda":
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
    dest = None
    if out is not None:
        want = (B, H, Sq, D) if layout == "BHSD" else (B, Sq, H, D)
        if tuple(out.shape) != want or out.dtype != q.dtype or out.device != q.device:
            raise ValueError(f"out must be a {q.dtype} tensor of shape {want} on {q.device}, got "
                             f"{out.dtype} {tuple(out.shape)} on {out.device}")
        dest = out
        # written in place when the kernel can store into it directly; otherwise (padded
        # head_dim, strided columns) through a temporary
        out = out if (Dp == D and out.stride(-1) == 1) else None
    if out is None:
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
        if mask is not None:
            mk = _prepare_mask(mask, B, H, Sq, Skv, q.device)
            rc = L.mlxp_attn_fwd_masked(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lse_ptr, dt, B, H, Hkv, Sq, Skv, Dp, *common[:4],
                                        mk.data_ptr(), (ctypes.c_int64 * 4)(*mk.stride()),
                                        *common[4:])
            what = "mlxp_attn_fwd_masked"
        elif Hkv == H:
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
    if dest is not None and out is not dest:
        dest.copy_(out)
        out = dest
    return (out, lse) if return_lse else out


_HOST_CHUNKS = 4
# BHSD host tensors are pipelined in (batch, head-range) pieces, each a contiguous block of
# q, k, v and o, so that the last piece's kernel and copy back, the part of the call that no
# copy to the device hides, are a small fraction of it.
_HOST_PIECES_BHSD = 16
_copy_streams = {}


def _streams(dev: torch.device):
    """Two copy streams per device (host-to-device, device-to-host), created once."""
    if dev.index not in _copy_streams:
        _copy_streams[dev.index] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _copy_streams[dev.index]


def _host_pieces(B, dim1_q, dim1_k, layout, kv_whole):
    """The pieces _host_attention stages host tensors in: ((b0, b1), (h0, h1) or None for every
    head).  BHSD tensors with fewer batches than _HOST_PIECES_BHSD and as many K/V heads as query
    heads (dim 1 of q and k) are cut into (batch, head-range) blocks; otherwise into batch
    chunks.  Every (batch, head) is in exactly one piece."""
    if layout == "BHSD" and not kv_whole and dim1_q == dim1_k and B < _HOST_PIECES_BHSD:
        H = dim1_q
        per_b = max(1, min(H, _HOST_PIECES_BHSD // B))
        return [((b, b + 1), (H * i // per_b, H * (i + 1) // per_b))
                for b in range(B) for i in range(per_b)]
    n = max(1, min(B, _HOST_CHUNKS))
    return [((B * i // n, B * (i + 1) // n), None) for i in range(n)]


def _host_attention(q, k, v, *, layout, scale, causal, window_left, window_right, q_offset,
                    kv_offset, kv_splits, return_lse):
    """Host tensors: staged through the current CUDA device in pieces (batch chunks; for BHSD
    tensors with fewer batches than _HOST_PIECES_BHSD, (batch, head-range) blocks), pipelined
    so that the copy of piece i+1 to the device, the kernel of piece i and the copy of piece
    i-1's result back run at the same time (two copy streams, the two copy engines of the GPU,
    and the compute stream).  The result lands in pinned host memory."""
    if not torch.cuda.is_available():
        raise RuntimeError("attention requires a CUDA device (there is no CPU fallback)")
    dev = torch.device("cuda", torch.cuda.current_device())
    B = q.shape[0]
    kv_whole = k.shape[0] != B  # a broadcast K/V batch is copied once, whole
    pieces = _host_pieces(B, q.shape[1], k.shape[1], layout, kv_whole)
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _streams(dev)
    s_in.wait_stream(cur)
    with torch.cuda.device(dev):
        dq = torch.empty(q.shape, dtype=q.dtype, device=dev)
        dk = torch.empty(k.shape, dtype=k.dtype, device=dev)
        dv = torch.empty(v.shape, dtype=v.dtype, device=dev)
    out_host = torch.empty(q.shape[:-1] + (v.shape[-1],), dtype=q.dtype, pin_memory=True)
    lse_host = None
    if return_lse:
        _, H, Sq, _ = _dims(q, layout)
        lse_host = torch.empty((B, H, Sq), dtype=torch.float32, pin_memory=True)
    for t in (dq, dk, dv):
        t.record_stream(s_in)
    if kv_whole:
        with torch.cuda.stream(s_in):
            dk.copy_(k, non_blocking=True)
            dv.copy_(v, non_blocking=True)
    for (b0, b1), hr in pieces:
        sl = (slice(b0, b1),) if hr is None else (slice(b0, b1), slice(*hr))
        with torch.cuda.stream(s_in):
            dq[sl].copy_(q[sl], non_blocking=True)
            if not kv_whole:
                dk[sl].copy_(k[sl], non_blocking=True)
                dv[sl].copy_(v[sl], non_blocking=True)
        cur.wait_stream(s_in)
        kk, vv = (dk, dv) if kv_whole else (dk[sl], dv[sl])
        res = attention_forward(dq[sl], kk, vv, layout=layout, scale=scale, causal=causal,
                                window_left=window_left, window_right=window_right,
                                q_offset=q_offset, kv_offset=kv_offset, kv_splits=kv_splits,
                                return_lse=return_lse)
        o, lse = res if return_lse else (res, None)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_out):
            out_host[sl].copy_(o, non_blocking=True)
            if lse is not None:
                lse_host[sl].copy_(lse, non_blocking=True)
        o.record_stream(s_out)
        if lse is not None:
            lse.record_stream(s_out)
    cur.wait_stream(s_out)
    s_out.synchronize()
    return (out_host, lse_host) if return_lse else out_host


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
