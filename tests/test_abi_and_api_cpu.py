"""CPU-only checks of the boundary: libmlxp_attn.so loads and exports every entry point
include/mlxp_attn.h declares (no compute call — there is no GPU here), and the Python API
validates its arguments exactly like the reference before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "mlxp_attn.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mlxp_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("mlxp_attn_fwd", "mlxp_attn_workspace_size", "mlxp_attn_fwd_partial",
                     "mlxp_lse_merge", "mlxp_last_error", "mlxp_version"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from mlx_primitives import _lib

    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} declared in mlxp_attn.h but not exported"
    assert set(declared_functions()) == set(_lib.EXPORTED_SYMBOLS)


def test_version_and_error_string_need_no_gpu():
    from mlx_primitives import _lib

    L = _lib.lib()
    assert L.mlxp_version() == 100
    assert isinstance(L.mlxp_last_error(), bytes)


def test_workspace_size_is_zero_without_split():
    from mlx_primitives import _lib

    L = _lib.lib()
    # kv_splits = 1: no workspace.  Pure host arithmetic, no device call.
    assert L.mlxp_attn_workspace_size(1, 4, 32, 4096, 4096, 128, 1, -1, -1, 0, 0, 1) == 0
    # explicit split: fp32 partial O + LSE for each split
    n = L.mlxp_attn_workspace_size(1, 8, 16, 512, 65536, 64, 0, -1, -1, 0, 0, 4)
    rows = 4 * 8 * 16 * 512
    assert n >= rows * 64 * 4 + rows * 4


def test_fp32_split_workspace_holds_partials_lses_and_block_counters():
    from mlx_primitives import _lib

    L = _lib.lib()
    L.mlxp_attn_workspace_size.restype = ctypes.c_size_t
    # fp32 (dtype 0), explicit 3 splits of config 1's shape: 256-byte aligned partials
    # [split][B][H][Sq][D], then LSEs [split][B][H][Sq], then one counter per 64-row query block
    B, H, Sq, Skv, D, s = 2, 12, 1024, 1024, 64, 3
    up = lambda x: (x + 255) // 256 * 256
    rows = s * B * H * Sq
    want = up(up(rows * D * 4) + rows * 4) + ((Sq + 63) // 64) * B * H * 4
    assert L.mlxp_attn_workspace_size(0, B, H, Sq, Skv, D, 1, -1, -1, 0, 0, s) == want
    # splits are capped at one per 32 keys
    assert (L.mlxp_attn_workspace_size(0, 1, 1, 100, 64, 32, 0, -1, -1, 0, 0, 8) ==
            L.mlxp_attn_workspace_size(0, 1, 1, 100, 64, 32, 0, -1, -1, 0, 0, 2))


def test_invalid_arguments_are_rejected_before_any_launch():
    from mlx_primitives import _lib

    L = _lib.lib()
    st = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    # unsupported head_dim on the tensor-core path
    rc = L.mlxp_attn_fwd(16, 16, 16, 16, None, 1, 1, 1, 8, 8, 96, st, st, st, st,
                         ctypes.c_float(0.1), 1, -1, -1, 0, 0, 1, None, 0, None)
    assert rc == _lib.MLXP_ERR_UNSUPPORTED and b"head_dim" in L.mlxp_last_error()
    # non-positive scale
    rc = L.mlxp_attn_fwd(16, 16, 16, 16, None, 1, 1, 1, 8, 8, 64, st, st, st, st,
                         ctypes.c_float(-1.0), 1, -1, -1, 0, 0, 1, None, 0, None)
    assert rc == _lib.MLXP_ERR_INVALID
    # null pointers
    rc = L.mlxp_attn_fwd(None, None, None, None, None, 1, 1, 1, 8, 8, 64, st, st, st, st,
                         ctypes.c_float(0.1), 1, -1, -1, 0, 0, 1, None, 0, None)
    assert rc == _lib.MLXP_ERR_INVALID


# ---- API validation mirrors flash.py:123-169 (raised before any device work) ----
def _t(*shape, dtype=torch.float32):
    return torch.zeros(shape, dtype=dtype)


def test_flash_validation_errors():
    import mlx_primitives as mp

    with pytest.raises(ValueError, match="Expected 4D"):
        mp.flash_attention(_t(2, 3, 4), _t(2, 3, 4, 8), _t(2, 3, 4, 8))
    with pytest.raises(ValueError, match="layout must be"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 8), _t(1, 4, 2, 8), layout="SBHD")
    with pytest.raises(ValueError, match="Batch size mismatch"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(2, 4, 2, 8), _t(1, 4, 2, 8))
    with pytest.raises(ValueError, match="Number of heads mismatch"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 3, 8), _t(1, 4, 2, 8))
    with pytest.raises(ValueError, match="Head dimension mismatch"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 16), _t(1, 4, 2, 8))
    with pytest.raises(ValueError, match="Sequence length mismatch"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 8), _t(1, 5, 2, 8))
    with pytest.raises(ValueError, match="dtype mismatch"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 8, dtype=torch.bfloat16), _t(1, 4, 2, 8))
    with pytest.raises(NotImplementedError, match="dropout"):
        mp.flash_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 8), _t(1, 4, 2, 8), dropout_p=0.1)


def test_grouped_query_validation():
    from mlx_primitives.attention import (GroupedQueryAttention, gqa_attention, mqa_attention)

    with pytest.raises(ValueError, match="num_kv_heads"):
        gqa_attention(_t(1, 4, 6, 8), _t(1, 4, 4, 8), _t(1, 4, 4, 8), num_kv_groups=2)
    with pytest.raises(ValueError, match="one K/V head"):
        mqa_attention(_t(1, 4, 4, 8), _t(1, 4, 2, 8), _t(1, 4, 2, 8))
    with pytest.raises(ValueError, match="divisible"):
        GroupedQueryAttention(64, 6, num_kv_heads=4)
    m = GroupedQueryAttention(64, 8, num_kv_heads=2, causal=True)
    assert (m.num_groups, m.head_dim) == (4, 8) and m.scale == pytest.approx(8 ** -0.5)


def test_other_entry_points_validate():
    import mlx_primitives as mp

    with pytest.raises(ValueError, match="Expected 4D"):
        mp.sliding_window_attention(_t(4, 2, 8), _t(1, 4, 2, 8), _t(1, 4, 2, 8), window_size=2)
    with pytest.raises(ValueError, match="window_size"):
        mp.sliding_window_attention(_t(1, 4, 2, 8), _t(1, 4, 2, 8), _t(1, 4, 2, 8), window_size=-1)
    with pytest.raises(ValueError, match="chunk_size"):
        mp.chunked_cross_attention(_t(1, 4, 2, 8), _t(1, 9, 2, 8), _t(1, 9, 2, 8), chunk_size=0)
    with pytest.raises(ValueError, match="dtype mismatch"):
        mp.chunked_cross_attention(_t(1, 4, 2, 8), _t(1, 9, 2, 8, dtype=torch.float16), _t(1, 9, 2, 8))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error")
def test_no_cpu_fallback():
    import mlx_primitives as mp

    with pytest.raises(RuntimeError, match="no CPU fallback"):
        mp.flash_attention(_t(1, 4, 2, 64), _t(1, 4, 2, 64), _t(1, 4, 2, 64))


def test_modules_store_reference_attributes():
    import mlx_primitives as mp

    fa = mp.FlashAttention(num_heads=8, head_dim=64)
    assert (fa.causal, fa.block_q, fa.block_kv, fa.scale) == (True, 32, 32, 0.125)
    assert mp.FlashAttention(8, 128).block_q == 16
    sw = mp.SlidingWindowAttention(8, 64, 128)
    assert (sw.window_size, sw.causal, sw.scale) == (128, True, 0.125)
    ca = mp.ChunkedCrossAttention(8, 64)
    assert (ca.chunk_size, ca.causal) == (1024, False)
    assert mp.Layout("BSHD") == "BSHD" and mp.Layout.BHSD == "BHSD"


@pytest.mark.parametrize("B,H,Hkv,layout,kv_whole", [
    (4, 32, 32, "BHSD", False), (1, 20, 20, "BHSD", False), (3, 5, 5, "BHSD", False),
    (16, 8, 8, "BHSD", False), (4, 32, 8, "BHSD", False), (2, 128, 128, "BSHD", False),
    (8, 16, 16, "BHSD", True), (1, 1, 1, "BHSD", False)])
def test_host_pieces_cover_every_unit_once(B, H, Hkv, layout, kv_whole):
    # host tensors are staged in these pieces; each (batch, head) must be copied, computed
    # and copied back exactly once (for BSHD, dim 1 is the sequence: batch chunks only)
    from mlx_primitives.attention._core import _host_pieces
    pieces = _host_pieces(B, H, Hkv, layout, kv_whole)
    seen = {}
    for (b0, b1), hr in pieces:
        assert 0 <= b0 < b1 <= B
        h0, h1 = hr if hr is not None else (0, H)
        assert 0 <= h0 < h1 <= H
        if hr is not None:
            assert layout == "BHSD" and not kv_whole and H == Hkv
        for b in range(b0, b1):
            for h in range(h0, h1):
                seen[(b, h)] = seen.get((b, h), 0) + 1
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(H)]
    assert set(seen.values()) == {1}
