"""ctypes binding of libmlxp_attn.so (include/mlxp_attn.h).

Replaces the reference's kernel registry (mlx_primitives/kernels/_registry.py:122-156,
``get_kernel``): instead of JIT-compiling Metal source per process, the attention kernels are
compiled ahead of time for sm_100a into one shared library that is loaded once.  There is no
fallback: if the library cannot be loaded, every attention call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

__all__ = [
    "MLXP_OK", "MLXP_ERR_INVALID", "MLXP_ERR_UNSUPPORTED", "MLXP_ERR_TIMEOUT",
    "DTYPE_CODES", "lib", "lib_path", "check", "EXPORTED_SYMBOLS",
]

MLXP_OK = 0
MLXP_ERR_INVALID = 1
MLXP_ERR_UNSUPPORTED = 2
MLXP_ERR_CUDA = 3
MLXP_ERR_NCCL = 4
MLXP_ERR_TIMEOUT = 5
MLXP_ERR_WORKSPACE = 6

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_i64x4 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/mlxp_attn.h one to one.
_SIGNATURES = {
    "mlxp_version": (ctypes.c_int, []),
    "mlxp_last_error": (ctypes.c_char_p, []),
    "mlxp_attn_fwd": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _i64,
        _i64, _p, ctypes.c_size_t, _p]),
    "mlxp_attn_fwd_gqa": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _i64,
        _i64, _p, ctypes.c_size_t, _p]),
    "mlxp_attn_workspace_size": (ctypes.c_size_t, [
        ctypes.c_int, _i64, _i64, _i64, _i64, _i64, ctypes.c_int, _i64, _i64, _i64, _i64, _i64]),
    "mlxp_attn_fwd_split_noalloc": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _i64,
        _i64, _p]),
    "mlxp_attn_fwd_partial": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _i64,
        _p]),
    "mlxp_attn_fwd_masked": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, _p, _i64x4, ctypes.c_float, ctypes.c_int,
        _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_size_t, _p]),
    "mlxp_rope_attn_fwd": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, _p, _p, _i64, _i64, _i64, ctypes.c_float, ctypes.c_int,
        _i64, _i64, _i64, _i64, _i64, _p, ctypes.c_size_t, _p]),
    "mlxp_rope_attn_workspace_size": (ctypes.c_size_t, [
        ctypes.c_int, _i64, _i64, _i64, _i64, _i64, ctypes.c_int, _i64, _i64, _i64, _i64, _i64]),
    "mlxp_attn_fwd_accumulate": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _i64, _i64, _i64,
        _p]),
    "mlxp_lse_merge": (ctypes.c_int, [
        _p, _p, _i64, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64x4, _p]),
    "mlxp_lse_merge_accumulate": (ctypes.c_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "mlxp_cast_output": (ctypes.c_int, [_p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64x4, _p]),
    "mlxp_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
    "mlxp_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "mlxp_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, _p]),
    "mlxp_rope": (ctypes.c_int, [_p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64x4, _i64x4,
                                 _p, _p, _i64, _i64, _p]),
    "mlxp_rope_qk": (ctypes.c_int, [_p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _i64x4, _i64x4, _i64x4, _i64x4, _p, _p, _i64, _i64,
                                    _i64, _p]),
    "mlxp_attn_bwd": (ctypes.c_int, [
        _p, _p, _p, _p, _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float,
        ctypes.c_int, _i64, _i64, _i64, _i64, _p, ctypes.c_size_t, _p]),
    "mlxp_attn_bwd_workspace_size": (ctypes.c_size_t, [ctypes.c_int, _i64, _i64, _i64, _i64, _i64]),
    "mlxp_set_backward_path": (ctypes.c_int, [ctypes.c_int]),
    "mlxp_paged_attn": (ctypes.c_int, [
        _p, _p, _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
        _i64, _i64x4, _i64x4, _i64, _i64x4, ctypes.c_float, ctypes.c_int, _i64, _p,
        ctypes.c_size_t, _p]),
    "mlxp_paged_attn_workspace_size": (ctypes.c_size_t, [
        ctypes.c_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "mlxp_ring_unique_id": (ctypes.c_int, [_p]),
    "mlxp_ring_init": (ctypes.c_int, [_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_p)]),
    "mlxp_ring_workspace_size": (ctypes.c_size_t, [ctypes.c_int, _i64, _i64, _i64, _i64]),
    "mlxp_ring_attn_fwd": (ctypes.c_int, [
        _p, _p, _p, _p, _p, ctypes.c_int, _i64, _i64, _i64, _i64,
        _i64x4, _i64x4, _i64x4, _i64x4, ctypes.c_float, _p, ctypes.c_size_t, _p]),
    "mlxp_ring_destroy": (ctypes.c_int, [_p]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def lib_path() -> Path:
    env = os.environ.get("MLXP_LIB")
    return Path(env) if env else Path(__file__).with_name("libmlxp_attn.so")


def lib() -> ctypes.CDLL:
    """Load libmlxp_attn.so once (thread-safe).  Raises ImportError when it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = lib_path()
                if not path.exists():
                    raise ImportError(
                        f"libmlxp_attn.so not found at {path}; build it with "
                        "`python mlx-primitives_b200/csrc/build.py` (there is no CPU fallback)")
                handle = ctypes.CDLL(str(path))
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().mlxp_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Map a status code to the reference's exception types (flash.py:123-169, 236-251)."""
    if rc == MLXP_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (MLXP_ERR_INVALID, MLXP_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def strides4(t: torch.Tensor, layout: str) -> ctypes.Array:
    """Element strides of a 4-D tensor in (batch, head, seq, dim) order."""
    s = t.stride()
    if layout == "BHSD":
        vals = (s[0], s[1], s[2], s[3])
    elif layout == "BSHD":
        vals = (s[0], s[2], s[1], s[3])
    else:
        raise ValueError(f"unknown layout {layout!r}")
    return (ctypes.c_int64 * 4)(*vals)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
