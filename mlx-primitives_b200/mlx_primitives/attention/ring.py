"""Sequence-parallel causal attention over several GPUs: a zig-zag ring pass of K/V blocks.

New component (the reference is single-device).  The sequence of length S is cut into 2P chunks
of C = S / (2P) tokens; rank r holds chunks r and 2P-1-r of Q, K and V back to back (zig-zag, so
every rank gets the same amount of causal work).  In P steps each rank computes its two local
query chunks against the K/V block it currently holds, sends that block to rank r+1 and
receives the next from rank r-1 (torch.distributed P2P: NCCL send/recv over NVLink on GPUs,
gloo on CPU), overlapping the transfer with the compute.  Each (query chunk, key chunk) pair is
a partial attention — normalised O and its log-sum-exp — with absolute positions so that the
causal mask is exact; pairs entirely above the diagonal are skipped and pairs entirely below
it are unmasked.  Partials are merged in fp32 with the LSE form of the reference's
online_softmax_merge (mlx_primitives/attention/_online_softmax.py:42-106).

The compute backend is pluggable: ``CudaRingBackend`` runs the sm_100a kernels through the
C-ABI — mlxp_attn_fwd_accumulate folds each chunk pair into the rank's fp32 accumulator inside
the attention kernel's epilogue (one launch per pair), mlxp_cast_output writes the result.  A
backend without ``accumulate`` (the CPU oracle backend of the tests) gets ``partial`` + ``merge``
calls instead.
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .. import _lib

__all__ = ["zigzag_chunks", "zigzag_shard", "zigzag_unshard", "ring_flash_attention",
           "CudaRingBackend", "nccl_unique_id", "NcclRing"]


def zigzag_chunks(world: int, rank: int) -> Tuple[int, int]:
    """Global chunk ids held by `rank` when the sequence is cut into 2 * world chunks."""
    return rank, 2 * world - 1 - rank


def zigzag_shard(x: torch.Tensor, world: int, rank: int, seq_dim: int = 2) -> torch.Tensor:
    """This rank's two chunks of a full-length tensor, concatenated along seq_dim."""
    chunks = x.chunk(2 * world, dim=seq_dim)
    a, b = zigzag_chunks(world, rank)
    return torch.cat([chunks[a], chunks[b]], dim=seq_dim)


def zigzag_unshard(parts: Sequence[torch.Tensor], seq_dim: int = 2) -> torch.Tensor:
    """Inverse of zigzag_shard given every rank's shard (rank order)."""
    world = len(parts)
    out: List[Optional[torch.Tensor]] = [None] * (2 * world)
    for r, part in enumerate(parts):
        a, b = zigzag_chunks(world, r)
        out[a], out[b] = part.chunk(2, dim=seq_dim)
    return torch.cat(out, dim=seq_dim)


class CudaRingBackend:
    """Partial attention and LSE merges on the GPU through libmlxp_attn.so (BHSD bf16/fp16)."""

    def partial(self, q, k, v, scale, q_off, kv_off, o_part, lse_part):
        L = _lib.lib()
        B, H, Sq, D = q.shape
        Skv = k.shape[2]
        rc = L.mlxp_attn_fwd_partial(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o_part.data_ptr(), lse_part.data_ptr(),
            _lib.DTYPE_CODES[q.dtype], B, H, Sq, Skv, D, _lib.strides4(q, "BHSD"),
            _lib.strides4(k, "BHSD"), _lib.strides4(v, "BHSD"), _lib.strides4(o_part, "BHSD"),
            ctypes.c_float(scale), 1, -1, -1, q_off, kv_off, _lib.stream_handle(q.device))
        _lib.check(rc, "mlxp_attn_fwd_partial")

    def accumulate(self, q, k, v, scale, q_off, kv_off, o_acc, lse_acc):
        """(o_acc, lse_acc) <- merge with attention of q against this k/v range, in place."""
        L = _lib.lib()
        B, H, Sq, D = q.shape
        Skv = k.shape[2]
        rc = L.mlxp_attn_fwd_accumulate(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o_acc.data_ptr(), lse_acc.data_ptr(),
            _lib.DTYPE_CODES[q.dtype], B, H, Sq, Skv, D, _lib.strides4(q, "BHSD"),
            _lib.strides4(k, "BHSD"), _lib.strides4(v, "BHSD"), _lib.strides4(o_acc, "BHSD"),
            ctypes.c_float(scale), 1, -1, -1, q_off, kv_off, _lib.stream_handle(q.device))
        _lib.check(rc, "mlxp_attn_fwd_accumulate")

    def merge(self, o_acc, lse_acc, o_new, lse_new):
        B, H, S, D = o_acc.shape
        rc = _lib.lib().mlxp_lse_merge_accumulate(o_acc.data_ptr(), lse_acc.data_ptr(),
                                                  o_new.data_ptr(), lse_new.data_ptr(), B, H, S,
                                                  D, _lib.stream_handle(o_acc.device))
        _lib.check(rc, "mlxp_lse_merge_accumulate")

    def finish(self, o_acc, out):
        B, H, S, D = o_acc.shape
        rc = _lib.lib().mlxp_cast_output(o_acc.data_ptr(), out.data_ptr(),
                                         _lib.DTYPE_CODES[out.dtype], B, H, S, D,
                                         _lib.strides4(out, "BHSD"),
                                         _lib.stream_handle(out.device))
        _lib.check(rc, "mlxp_cast_output")


def ring_flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         scale: Optional[float] = None, group=None, backend=None) -> torch.Tensor:
    """Causal attention of a zig-zag sharded sequence (see module docstring).

    q, k, v: this rank's shard, BHSD [B, H, 2*C, D] (chunks r and 2P-1-r back to back), all
    ranks with the same shapes.  Returns this rank's shard of the output (same shape, q's
    dtype).  Every rank must call it (a collective over `group`).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if q.ndim != 4 or q.shape != k.shape or k.shape != v.shape:
        raise ValueError("q, k, v must be BHSD shards of equal shape")
    if q.shape[2] % 2:
        raise ValueError("a zig-zag shard holds two equal chunks (even local length)")
    B, H, S2, D = q.shape
    C = S2 // 2
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if backend is None:
        backend = CudaRingBackend()
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    # global ranks of the neighbours (P2P ops take global ranks)
    if group is not None:
        nxt = dist.get_global_rank(group, nxt)
        prv = dist.get_global_rank(group, prv)

    dev = q.device
    fused = hasattr(backend, "accumulate")
    o_acc = torch.zeros((2, B, H, C, D), dtype=torch.float32, device=dev)
    lse_acc = torch.full((2, B, H, C), float("-inf"), dtype=torch.float32, device=dev)
    if not fused:
        o_part = torch.empty((B, H, C, D), dtype=torch.float32, device=dev)
        lse_part = torch.empty((B, H, C), dtype=torch.float32, device=dev)
    bufs = [(torch.empty_like(k), torch.empty_like(v)) for _ in range(2 if world > 1 else 0)]
    q_chunks = zigzag_chunks(world, rank)

    kv = (k, v)
    for step in range(world):
        src = (rank - step) % world
        reqs = []
        if step + 1 < world:
            recv_k, recv_v = bufs[step % 2]
            ops = [dist.P2POp(dist.isend, kv[0], nxt, group),
                   dist.P2POp(dist.isend, kv[1], nxt, group),
                   dist.P2POp(dist.irecv, recv_k, prv, group),
                   dist.P2POp(dist.irecv, recv_v, prv, group)]
            reqs = dist.batch_isend_irecv(ops)
        for qi, qc in enumerate(q_chunks):
            qs = q[:, :, qi * C:(qi + 1) * C]
            for ki, kc in enumerate(zigzag_chunks(world, src)):
                if kc > qc:
                    continue  # every key after every query of this chunk
                ks = kv[0][:, :, ki * C:(ki + 1) * C]
                vs = kv[1][:, :, ki * C:(ki + 1) * C]
                if fused:
                    backend.accumulate(qs, ks, vs, scale, qc * C, kc * C, o_acc[qi], lse_acc[qi])
                else:
                    backend.partial(qs, ks, vs, scale, qc * C, kc * C, o_part, lse_part)
                    backend.merge(o_acc[qi], lse_acc[qi], o_part, lse_part)
        for req in reqs:
            req.wait()
        if step + 1 < world:
            kv = bufs[step % 2]
    out = torch.empty_like(q)
    backend.finish(o_acc[0], out[:, :, :C])
    backend.finish(o_acc[1], out[:, :, C:])
    return out


def nccl_unique_id() -> bytes:
    """A new 128-byte NCCL unique id for NcclRing (create on one rank, share with the others)."""
    buf = ctypes.create_string_buffer(128)
    _lib.check(_lib.lib().mlxp_ring_unique_id(ctypes.cast(buf, ctypes.c_void_p)),
               "mlxp_ring_unique_id")
    return buf.raw


class NcclRing:
    """The same zig-zag ring run entirely by the C library (mlxp_ring_*) over its own NCCL
    communicator, without torch.distributed: the path a non-Python caller of the C ABI takes.
    Construct on every rank with the same id and nranks, on the rank's current CUDA device."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int):
        if len(unique_id) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        self._comm = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(unique_id, 128)
        _lib.check(_lib.lib().mlxp_ring_init(ctypes.cast(idbuf, ctypes.c_void_p), nranks, rank,
                                             ctypes.byref(self._comm)), "mlxp_ring_init")
        self.nranks, self.rank = nranks, rank

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                scale: Optional[float] = None, layout: str = "BHSD") -> torch.Tensor:
        """Causal attention of this rank's zig-zag shard (q, k, v: [B, H, S_local, D] for
        BHSD or [B, S_local, H, D] for BSHD); returns this rank's shard of the output."""
        if self._comm.value is None:
            raise RuntimeError("the ring has been closed")
        if q.shape != k.shape or k.shape != v.shape or q.ndim != 4:
            raise ValueError("q, k, v must be 4-D shards of equal shape")
        if layout == "BHSD":
            B, H, S, D = q.shape
        else:
            B, S, H, D = q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        L = _lib.lib()
        code = _lib.DTYPE_CODES[q.dtype]
        nbytes = L.mlxp_ring_workspace_size(code, B, H, S, D)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
        out = torch.empty_like(q)
        rc = L.mlxp_ring_attn_fwd(self._comm, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  out.data_ptr(), code, B, H, S, D, _lib.strides4(q, layout),
                                  _lib.strides4(k, layout), _lib.strides4(v, layout),
                                  _lib.strides4(out, layout), ctypes.c_float(scale),
                                  ws.data_ptr(), nbytes, _lib.stream_handle(q.device))
        _lib.check(rc, "mlxp_ring_attn_fwd")
        return out

    def close(self) -> None:
        if self._comm.value is not None:
            _lib.check(_lib.lib().mlxp_ring_destroy(self._comm), "mlxp_ring_destroy")
            self._comm = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
