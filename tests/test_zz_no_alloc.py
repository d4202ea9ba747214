"""The allocation-free split-KV entry point (mlxp_attn_fwd_split_noalloc) against the regular
one (mlxp_attn_fwd with a caller workspace), through the C-ABI.

It serves callers that cannot allocate device memory (plugins handed only input/output
pointers, loops that must not trigger cudaMalloc), so it keeps its scratch in a static device
array shared by every call.  The test makes two calls in a row — the second finds the first
call's partials still in the array — and compares each with the regular entry point within the
bf16 tolerance the other GPU tests use (2e-2 max-abs; the LSE within 1e-2).  It also checks that
a size whose scratch exceeds the array is rejected with a clear error before anything runs.
This file is collected last on purpose; it must also pass when run alone.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _case(B, H, Sq, Skv, D, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((B, Sq, H, D), generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, Skv, H, D), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, Skv, H, D), generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v


def test_no_alloc_split_matches_workspace_split_twice():
    from mlx_primitives import _lib

    L = _lib.lib()
    B, H, Sq, Skv, D, splits = 2, 8, 384, 9000, 128, 4
    scale = D ** -0.5
    stream = torch.cuda.current_stream().cuda_stream
    st = lambda t: _lib.strides4(t, "BSHD")

    q, k, v = _case(B, H, Sq, Skv, D, seed=5)
    o_ref = torch.empty_like(q)
    lse_ref = torch.empty((B, H, Sq), device="cuda")
    ws_bytes = L.mlxp_attn_workspace_size(1, B, H, Sq, Skv, D, 0, -1, -1, 0, 0, splits)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.check(L.mlxp_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_ref.data_ptr(),
                               lse_ref.data_ptr(), 1, B, H, Sq, Skv, D, st(q), st(k), st(v),
                               st(o_ref), ctypes.c_float(scale), 0, -1, -1, 0, 0, splits,
                               ws.data_ptr(), ws_bytes, stream), "mlxp_attn_fwd")

    for call in range(2):
        o = torch.full_like(q, float("nan"))
        lse = torch.full((B, H, Sq), float("nan"), device="cuda")
        rc = L.mlxp_attn_fwd_split_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                           o.data_ptr(), lse.data_ptr(), 1, B, H, Sq, Skv, D,
                                           st(q), st(k), st(v), st(o), ctypes.c_float(scale),
                                           0, -1, -1, 0, 0, splits, stream)
        _lib.check(rc, "mlxp_attn_fwd_split_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(o.float()).all(), f"call {call}"
        err = (o.float() - o_ref.float()).abs().max().item()
        assert err <= TOL, f"call {call}: max-abs {err}"
        assert (lse - lse_ref).abs().max().item() <= 1e-2, f"call {call}"


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    from mlx_primitives import _lib

    L = _lib.lib()
    # 16 splits x (8*16*4096 rows) x 129 floats is far beyond 32 MiB: rejected, nothing runs.
    B, H, Sq, Skv, D, splits = 8, 16, 4096, 65536, 128, 16
    st = (ctypes.c_int64 * 4)(Sq * H * D, D, H * D, 1)
    rc = L.mlxp_attn_fwd_split_noalloc(16, 16, 16, 16, None, 1, B, H, Sq, Skv, D, st, st, st, st,
                                       ctypes.c_float(0.1), 0, -1, -1, 0, 0, splits, None)
    assert rc == _lib.MLXP_ERR_WORKSPACE
    assert b"static scratch" in L.mlxp_last_error()
