"""The allocation-free split-KV entry point (mlxp_attn_fwd_split_noalloc) against the regular
one (mlxp_attn_fwd with a caller workspace), through the C-ABI.

It serves callers that cannot allocate device memory (plugins handed only input/output
pointers, loops that must not trigger cudaMalloc), so it keeps its scratch in a static device
array shared by every call.  The test makes calls in a row on different data and shapes — each
finds the previous call's partials and counters still in the array: a non-causal case, then a
causal one with explicit key splits of which some reach no key of some query tiles, then the
first again — and compares each with the regular entry point given a NaN-filled workspace.  Both
run the same kernel with the same splits and merge the partials in the same order, so output and
LSE must agree bit for bit (which also keeps them within the bf16 tolerance, 2e-2 max-abs, of
the other GPU tests).  A size whose scratch exceeds the array is rejected with a clear error
before anything runs.  This file is collected last on purpose; it must also pass when run alone.
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


def _run(L, _lib, q, k, v, causal, splits, noalloc):
    B, Sq, H, D = q.shape
    Skv = k.shape[1]
    st = lambda t: _lib.strides4(t, "BSHD")
    stream = torch.cuda.current_stream().cuda_stream
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B, H, Sq), float("nan"), device="cuda")
    qoff = (Skv - Sq) if causal else 0
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), 1, B, H, Sq,
            Skv, D, st(q), st(k), st(v), st(o), ctypes.c_float(D ** -0.5), int(causal), -1, -1,
            qoff, 0, splits)
    if noalloc:
        _lib.check(L.mlxp_attn_fwd_split_noalloc(*args, stream), "mlxp_attn_fwd_split_noalloc")
    else:
        ws_bytes = L.mlxp_attn_workspace_size(1, B, H, Sq, Skv, D, int(causal), -1, -1, qoff, 0,
                                              splits)
        assert ws_bytes > 0
        ws = torch.full((ws_bytes // 4,), float("nan"), device="cuda")  # stale garbage
        _lib.check(L.mlxp_attn_fwd(*args, ws.data_ptr(), ws_bytes, stream), "mlxp_attn_fwd")
    torch.cuda.synchronize()
    return o, lse


def test_no_alloc_split_matches_workspace_split_on_calls_in_a_row():
    from mlx_primitives import _lib

    L = _lib.lib()
    cases = [
        # (B, H, Sq, Skv, D, seed, causal, splits)
        (2, 8, 384, 9000, 128, 5, False, 4),
        # causal, 4 splits of 8 key tiles: query tiles near the start reach only split 0, so
        # the other splits write nothing for them; later tiles merge 2 to 4 partials
        (3, 4, 1000, 3968, 64, 6, True, 4),
        (2, 8, 384, 9000, 128, 5, False, 4),
    ]
    for n, (B, H, Sq, Skv, D, seed, causal, splits) in enumerate(cases):
        q, k, v = _case(B, H, Sq, Skv, D, seed)
        o_ref, lse_ref = _run(L, _lib, q, k, v, causal, splits, noalloc=False)
        o, lse = _run(L, _lib, q, k, v, causal, splits, noalloc=True)
        assert torch.isfinite(o.float()).all(), f"call {n}"
        assert torch.equal(o, o_ref), f"call {n}: max-abs {(o.float() - o_ref.float()).abs().max()}"
        assert torch.equal(lse, lse_ref), f"call {n}"
        assert (o.float() - o_ref.float()).abs().max().item() <= TOL


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
