"""GPU parity: the sm_100a kernels (through the C-ABI) against the CPU oracle.

Tolerances (written per the contract): fp32 path <= 1e-4 max-abs; bf16/fp16 <= 2e-2 max-abs
against an fp64 oracle fed the same bf16/fp16-rounded inputs.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def dev():
    return torch.device("cuda", 0)


def inputs(shape_q, shape_kv, dtype, seed=42, std=1.0):
    q, k, v = O.make_qkv(shape_q, shape_kv, seed=seed, std=std)
    tq, tk, tv = (torch.from_numpy(a).to(dev()).to(dtype) for a in (q, k, v))
    # the oracle sees exactly the values the GPU sees
    nq, nk, nv = (t.float().cpu().numpy() for t in (tq, tk, tv))
    return (tq, tk, tv), (nq, nk, nv)


def maxabs(got: torch.Tensor, want: np.ndarray) -> float:
    return float(np.max(np.abs(got.float().cpu().numpy().astype(np.float64) - want))) if want.size else 0.0


def core():
    from mlx_primitives.attention._core import attention_forward
    return attention_forward


# ----------------------------------------------------------------------------- basics
def test_library_loads_and_reports_version():
    from mlx_primitives import _lib
    assert _lib.lib().mlxp_version() >= 100


def test_bounded_wait_gives_up_and_reports():
    from mlx_primitives import _lib
    L = _lib.lib()
    rc = L.mlxp_selftest_wait_timeout(2_000_000, None)  # 2 ms limit on a wait nobody ends
    assert rc == _lib.MLXP_ERR_TIMEOUT, _lib.last_error()
    st = ctypes.c_int(0)
    assert L.mlxp_device_status(ctypes.byref(st), 1) == 0
    assert (st.value & 0xFF) == _lib.MLXP_ERR_TIMEOUT and (st.value >> 8) == 7
    assert L.mlxp_device_status(ctypes.byref(st), 0) == 0 and st.value == 0
    # the context is still usable
    (q, k, v), (nq, nk, nv) = inputs((1, 1, 128, 64), (1, 1, 128, 64), torch.bfloat16)
    o = core()(q, k, v, layout="BHSD", scale=0.125, causal=True)
    assert maxabs(o, O.attention_bhsd(nq, nk, nv, 0.125, causal=True)) < 2e-2


# ----------------------------------------------------------------------------- tensor-core path
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [1, 63, 128, 129, 255, 256, 257, 300, 640])
def test_tc_bhsd_causal_shapes(dtype, D, S):
    (q, k, v), (nq, nk, nv) = inputs((1, 2, S, D), (1, 2, S, D), dtype, seed=S + D)
    o = core()(q, k, v, layout="BHSD", scale=D ** -0.5, causal=True)
    assert o.dtype == dtype and o.shape == q.shape
    assert maxabs(o, O.attention_bhsd(nq, nk, nv, D ** -0.5, causal=True)) <= TOL[dtype]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("Sq,Skv", [(128, 128), (100, 333), (333, 100), (513, 1000), (1, 4096)])
@pytest.mark.parametrize("causal", [False, True])
def test_tc_bshd_cross_lengths(D, Sq, Skv, causal):
    (q, k, v), (nq, nk, nv) = inputs((2, Sq, 3, D), (2, Skv, 3, D), torch.bfloat16, seed=Sq * 7 + Skv)
    off = (Skv - Sq) if causal else 0  # bottom-right aligned, as flash_attention passes it
    o = core()(q, k, v, layout="BSHD", scale=D ** -0.5, causal=causal, q_offset=off)
    want = O.attention_bhsd(*(np.swapaxes(a, 1, 2) for a in (nq, nk, nv)), D ** -0.5,
                            causal=causal, q_offset=off)
    assert maxabs(o, np.swapaxes(want, 1, 2)) <= TOL[torch.bfloat16]


@pytest.mark.parametrize("W,causal", [(0, True), (5, True), (127, True), (128, True), (200, True),
                                      (20, False), (300, False)])
@pytest.mark.parametrize("D", [64, 128])
def test_tc_sliding_window(W, causal, D):
    S = 777
    (q, k, v), (nq, nk, nv) = inputs((1, S, 2, D), (1, S, 2, D), torch.bfloat16, seed=W + 3)
    import mlx_primitives as mp
    o = mp.sliding_window_attention(q, k, v, window_size=W, causal=causal)
    want = O.sliding_window_attention(nq, nk, nv, W, causal=causal)
    assert maxabs(o, want) <= TOL[torch.bfloat16]


@pytest.mark.parametrize("q_off,kv_off", [(0, 0), (256, 0), (300, 17), (0, 500), (4096, 4096 - 128)])
def test_tc_position_offsets(q_off, kv_off):
    (q, k, v), (nq, nk, nv) = inputs((1, 2, 384, 128), (1, 2, 640, 128), torch.bfloat16, seed=q_off + 1)
    o, lse = core()(q, k, v, layout="BHSD", scale=0.1, causal=True, q_offset=q_off,
                    kv_offset=kv_off, return_lse=True)
    want, want_lse = O.attention_bhsd(nq, nk, nv, 0.1, causal=True, q_offset=q_off,
                                      kv_offset=kv_off, return_lse=True)
    assert maxabs(o, want) <= TOL[torch.bfloat16]
    got_lse = lse.cpu().numpy()
    finite = np.isfinite(want_lse)
    assert np.array_equal(np.isfinite(got_lse), finite)
    if finite.any():
        assert np.max(np.abs(got_lse[finite] - want_lse[finite])) < 1e-2


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 0])
def test_tc_split_kv_matches_oracle(splits):
    (q, k, v), (nq, nk, nv) = inputs((2, 300, 4, 64), (2, 5000, 4, 64), torch.bfloat16, seed=11, std=0.5)
    o, lse = core()(q, k, v, layout="BSHD", scale=0.125, causal=False, kv_splits=splits,
                    return_lse=True)
    want, want_lse = O.attention_bhsd(*(np.swapaxes(a, 1, 2) for a in (nq, nk, nv)), 0.125,
                                      return_lse=True)
    assert maxabs(o, np.swapaxes(want, 1, 2)) <= TOL[torch.bfloat16]
    assert np.max(np.abs(lse.cpu().numpy() - want_lse)) < 1e-2


def test_tc_deterministic():
    (q, k, v), _ = inputs((2, 4, 1000, 128), (2, 4, 1000, 128), torch.bfloat16, seed=12)
    f = core()
    a = f(q, k, v, layout="BHSD", scale=0.09, causal=True)
    b = f(q, k, v, layout="BHSD", scale=0.09, causal=True)
    assert torch.equal(a, b)


def test_tc_broadcast_batch_kv():
    # K/V with batch stride 0 (one shared context for every query batch)
    (q, _, _), (nq, _, _) = inputs((3, 2, 200, 64), (1, 2, 1, 64), torch.bfloat16, seed=13)
    (k1, v1, _), (nk1, nv1, _) = inputs((1, 2, 500, 64), (1, 2, 500, 64), torch.bfloat16, seed=14)
    k, v = k1.expand(3, -1, -1, -1), v1.expand(3, -1, -1, -1)
    o = core()(q, k, v, layout="BHSD", scale=0.125, causal=False)
    want = O.attention_bhsd(nq, np.broadcast_to(nk1, (3, 2, 500, 64)),
                            np.broadcast_to(nv1, (3, 2, 500, 64)), 0.125)
    assert maxabs(o, want) <= TOL[torch.bfloat16]


def test_tc_no_keys_gives_zero_and_neg_inf():
    (q, k, v), _ = inputs((1, 1, 130, 64), (1, 1, 130, 64), torch.bfloat16, seed=15)
    # every key is after every query: nothing admissible
    o, lse = core()(q, k, v, layout="BHSD", scale=0.125, causal=True, q_offset=0, kv_offset=1000,
                    return_lse=True)
    assert torch.count_nonzero(o) == 0 and torch.isneginf(lse).all()
    o, lse = core()(q, k[:, :, :0], v[:, :, :0], layout="BHSD", scale=0.125, causal=False,
                    return_lse=True)
    assert torch.count_nonzero(o) == 0 and torch.isneginf(lse).all()


def test_partial_and_merge_entry_points():
    from mlx_primitives import _lib
    L = _lib.lib()
    (q, k, v), (nq, nk, nv) = inputs((1, 2, 256, 128), (1, 2, 900, 128), torch.bfloat16, seed=16)
    cuts = [(0, 300), (300, 301), (301, 900)]
    B, H, S, D = 1, 2, 256, 128
    o_parts = torch.empty((len(cuts), B, H, S, D), device=dev())
    l_parts = torch.empty((len(cuts), B, H, S), device=dev())
    stream = torch.cuda.current_stream().cuda_stream
    for i, (a, b) in enumerate(cuts):
        kk, vv = k[:, :, a:b], v[:, :, a:b]
        rc = L.mlxp_attn_fwd_partial(q.data_ptr(), kk.data_ptr(), vv.data_ptr(), o_parts[i].data_ptr(),
                                     l_parts[i].data_ptr(), 1, B, H, S, b - a, D,
                                     _lib.strides4(q, "BHSD"), _lib.strides4(kk, "BHSD"),
                                     _lib.strides4(vv, "BHSD"), _lib.strides4(o_parts[i], "BHSD"),
                                     ctypes.c_float(0.1), 1, -1, -1, 600, a, stream)
        _lib.check(rc, "partial")
    out = torch.empty((B, H, S, D), dtype=torch.bfloat16, device=dev())
    lse = torch.empty((B, H, S), device=dev())
    _lib.check(L.mlxp_lse_merge(o_parts.data_ptr(), l_parts.data_ptr(), len(cuts), out.data_ptr(),
                                lse.data_ptr(), 1, B, H, S, D, _lib.strides4(out, "BHSD"), stream), "merge")
    want, want_lse = O.attention_bhsd(nq, nk, nv, 0.1, causal=True, q_offset=600, return_lse=True)
    assert maxabs(out, want) <= TOL[torch.bfloat16]
    assert np.max(np.abs(lse.cpu().numpy() - want_lse)) < 1e-2
    # running merge (the ring's accumulator) gives the same answer
    acc_o, acc_l = o_parts[0].clone(), l_parts[0].clone()
    for i in (1, 2):
        _lib.check(L.mlxp_lse_merge_accumulate(acc_o.data_ptr(), acc_l.data_ptr(), o_parts[i].data_ptr(),
                                               l_parts[i].data_ptr(), B, H, S, D, stream), "acc")
    assert maxabs(acc_o, want) <= 1e-2
    out2 = torch.empty_like(out)
    _lib.check(L.mlxp_cast_output(acc_o.data_ptr(), out2.data_ptr(), 1, B, H, S, D,
                                  _lib.strides4(out2, "BHSD"), stream), "cast")
    assert maxabs(out2, want) <= TOL[torch.bfloat16]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("layout", ["BHSD", "BSHD"])
def test_accumulate_entry_point_folds_key_ranges(D, layout):
    """mlxp_attn_fwd_accumulate folds key ranges into a running fp32 (O, LSE) in the attention
    kernel's epilogue: the result equals attention over the union (fp64 oracle).  The ranges
    include one no query row reaches (rows left unchanged), one that only some rows reach, and
    an accumulator whose O starts as NaN garbage (rows with LSE -inf must not read it)."""
    from mlx_primitives import _lib
    L = _lib.lib()
    B, H, S, Skv = 2, 3, 300, 1100
    (q, k, v), (nq, nk, nv) = inputs((B, H, S, D), (B, H, Skv, D), torch.bfloat16, seed=17 + D)
    qoff = 520  # causal: query i sees keys j <= i + 520
    cuts = [(850, 1100), (0, 400), (400, 401), (401, 850)]
    if layout == "BSHD":
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    acc = torch.full((B, H, S, D), float("nan"), device=dev())
    acc_lse = torch.full((B, H, S), float("-inf"), device=dev())
    stream = torch.cuda.current_stream().cuda_stream
    kv_view = (lambda t, a, b: t[:, :, a:b]) if layout == "BHSD" else (lambda t, a, b: t[:, a:b])
    for a, b in cuts:
        kk, vv = kv_view(k, a, b), kv_view(v, a, b)
        rc = L.mlxp_attn_fwd_accumulate(q.data_ptr(), kk.data_ptr(), vv.data_ptr(), acc.data_ptr(),
                                        acc_lse.data_ptr(), 1, B, H, S, b - a, D,
                                        _lib.strides4(q, layout), _lib.strides4(kk, layout),
                                        _lib.strides4(vv, layout), _lib.strides4(acc, "BHSD"),
                                        ctypes.c_float(D ** -0.5), 1, -1, -1, qoff, a, stream)
        _lib.check(rc, "mlxp_attn_fwd_accumulate")
    torch.cuda.synchronize()
    want, want_lse = O.attention_bhsd(nq, nk, nv, D ** -0.5, causal=True, q_offset=qoff,
                                      return_lse=True)
    assert torch.isfinite(acc).all()
    assert maxabs(acc, want) <= 1e-2
    assert np.max(np.abs(acc_lse.cpu().numpy() - want_lse)) < 1e-2
    out = torch.empty((B, H, S, D), dtype=torch.bfloat16, device=dev())
    _lib.check(L.mlxp_cast_output(acc.data_ptr(), out.data_ptr(), 1, B, H, S, D,
                                  _lib.strides4(out, "BHSD"), stream), "cast")
    assert maxabs(out, want) <= TOL[torch.bfloat16]
    # a key range that reaches no row leaves the accumulator bit-for-bit as it was
    before, before_lse = acc.clone(), acc_lse.clone()
    kk, vv = kv_view(k, 0, 10), kv_view(v, 0, 10)
    _lib.check(L.mlxp_attn_fwd_accumulate(q.data_ptr(), kk.data_ptr(), vv.data_ptr(), acc.data_ptr(),
                                          acc_lse.data_ptr(), 1, B, H, S, 10, D,
                                          _lib.strides4(q, layout), _lib.strides4(kk, layout),
                                          _lib.strides4(vv, layout), _lib.strides4(acc, "BHSD"),
                                          ctypes.c_float(D ** -0.5), 1, -1, -1, qoff, 5000, stream),
               "accumulate (no admissible key)")
    torch.cuda.synchronize()
    assert torch.equal(acc, before) and torch.equal(acc_lse, before_lse)


# ----------------------------------------------------------------------------- fp32 CUDA-core path
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("S", [1, 31, 64, 65, 200])
@pytest.mark.parametrize("causal", [True, False])
def test_fp32_shapes(D, S, causal):
    (q, k, v), (nq, nk, nv) = inputs((2, S, 3, D), (2, S, 3, D), torch.float32, seed=S + D)
    import mlx_primitives as mp
    o = mp.flash_attention(q, k, v, causal=causal)
    assert o.dtype == torch.float32
    assert maxabs(o, O.flash_attention(nq, nk, nv, causal=causal)) <= TOL[torch.float32]


def test_fp32_config1_full_size():
    # BSHD fp32 causal, batch 2, seq 1024, 12 heads, head_dim 64
    (q, k, v), (nq, nk, nv) = inputs((2, 1024, 12, 64), (2, 1024, 12, 64), torch.float32, seed=42)
    import mlx_primitives as mp
    o = mp.flash_attention(q, k, v, causal=True)
    assert maxabs(o, O.flash_attention(nq, nk, nv, causal=True)) <= 1e-4


def test_fp32_window_and_offsets():
    (q, k, v), (nq, nk, nv) = inputs((1, 2, 150, 64), (1, 2, 300, 64), torch.float32, seed=17)
    o, lse = core()(q, k, v, layout="BHSD", scale=0.125, causal=True, window_left=40,
                    q_offset=120, kv_offset=0, return_lse=True)
    want, want_lse = O.attention_bhsd(nq, nk, nv, 0.125, causal=True, window_left=40, q_offset=120,
                                      return_lse=True)
    assert maxabs(o, want) <= 1e-4
    assert np.max(np.abs(lse.cpu().numpy() - want_lse)) < 1e-4


# ----------------------------------------------------------------------------- golden fixtures
def _golden():
    from pathlib import Path
    return np.load(Path(__file__).parent / "golden" / "reference_outputs.npz")


# case -> (public API, kwargs): the same calls tests/golden/make_golden.py made on the reference
GOLDEN_CALLS = {
    "flash_bshd_tiled_causal_d64": ("flash", dict(causal=True)),
    "flash_bshd_tiled_noncausal_d64": ("flash", dict(causal=False)),
    "flash_bshd_tiled_causal_d128_b16": ("flash", dict(causal=True)),
    "flash_bshd_tiled_causal_d32_ragged": ("flash", dict(causal=True)),
    "flash_bshd_dense_causal_d64": ("flash", dict(causal=True)),
    "flash_bshd_dense_scale_d64": ("flash", dict(scale=0.3, causal=False)),
    "flash_bshd_single_token": ("flash", dict(causal=True)),
    "flash_bshd_large_values": ("flash", dict(causal=True)),
    "flash_bhsd_causal_d128": ("flash", dict(causal=True, layout="BHSD")),
    "flash_bhsd_noncausal_d64": ("flash", dict(causal=False, layout="BHSD")),
    "swa_tiled_causal_w37": ("swa", dict(window_size=37, causal=True)),
    "swa_tiled_bidir_w20": ("swa", dict(window_size=20, causal=False)),
    "swa_tiled_causal_w130_d128": ("swa", dict(window_size=130, causal=True)),
    "swa_dense_causal_w5": ("swa", dict(window_size=5, scale=0.125, causal=True)),
    "chunked_loop_noncausal": ("chunked", dict(chunk_size=128)),
    "chunked_loop_causal": ("chunked", dict(chunk_size=64, causal=True)),
    "chunked_loop_q_longer_causal": ("chunked", dict(chunk_size=64, causal=True)),
    "chunked_dense_short_kv": ("chunked", dict(chunk_size=1024)),
    "gqa_g4_causal_d64": ("gqa", dict(num_kv_groups=4, causal=True)),
    "gqa_g2_noncausal_d128": ("gqa", dict(num_kv_groups=2, causal=False)),
    "gqa_g2_causal_kv_longer_d64": ("gqa", dict(num_kv_groups=2, scale=0.2, causal=True)),
    "mqa_causal_d64": ("mqa", dict(causal=True)),
    "mqa_3d_kv_noncausal_d128": ("mqa3d", dict(causal=False)),
    # custom additive masks, stored with the case ("<case>__mask")
    "gqa_mask_bias_g2_d64": ("gqa", dict(num_kv_groups=2, mask_case="gqa_mask_bias_g2_d64")),
    "gqa_mask_exclude_causal_d128": ("gqa", dict(num_kv_groups=2, causal=True,
                                                 mask_case="gqa_mask_exclude_causal_d128")),
    "mqa_mask_head_bias_d64": ("mqa", dict(mask_case="mqa_mask_head_bias_d64")),
    "rope_only_offset7_d64": ("rope", dict(offset=7)),
    "fused_rope_causal_d64": ("frope", dict(causal=True)),
    "fused_rope_offsets_noncausal_d128": ("frope", dict(q_offset=30, kv_offset=0, causal=False)),
    "fused_rope_decode_causal_base500": ("frope", dict(rope_base=500.0, q_offset=32, causal=True)),
}
# paged attention: block tables, lengths and options are stored with each case
GOLDEN_CALLS.update({c: ("paged", c) for c in (
    "paged_decode_batch_d64", "paged_decode_alibi_d128", "paged_decode_hole_d32",
    "paged_prefill_causal_d64", "paged_prefill_alibi_noncausal_d64",
    "paged_prefill_alibi_causal_d128")})


def _paged_call(mod, case, q, k_pool, v_pool):
    g = _golden()
    bs, causal, alibi, scale = g[f"{case}__opts"]
    kw = dict(scale=None if scale < 0 else float(scale), block_size=int(bs), causal=bool(causal))
    bt, ctx = g[f"{case}__bt"], g[f"{case}__ctx"]
    if mod is O:
        slopes = O.get_alibi_slopes(q.shape[2]) if alibi else None
        # rows with no admissible key: NaN in the reference, zeros by the library's definition
        return np.nan_to_num(O.paged_attention(q, k_pool, v_pool, bt, ctx, alibi_slopes=slopes,
                                               **kw), nan=0.0)
    from mlx_primitives.cache import get_alibi_slopes, paged_attention
    slopes = get_alibi_slopes(q.shape[2], device=q.device) if alibi else None
    return paged_attention(q, k_pool, v_pool, torch.from_numpy(bt).to(q.device),
                           torch.from_numpy(ctx).to(q.device), alibi_slopes=slopes, **kw)


def _call(api, mod, q, k, v, kw):
    if api == "paged":
        return _paged_call(mod, kw, q, k, v)
    if api == "flash":
        return mod.flash_attention(q, k, v, **kw)
    if api == "swa":
        return mod.sliding_window_attention(q, k, v, **kw)
    if api == "rope":
        if mod is O:
            return O.rope(q, *O.precompute_rope_cache(80, 64), **kw)
        from mlx_primitives.kernels import precompute_rope_cache, rope
        cos, sin = precompute_rope_cache(80, 64)
        return rope(q, cos, sin, **kw)
    if api == "frope":
        if mod is O:
            return O.fused_rope_attention(q, k, v, **kw)
        from mlx_primitives.kernels import fused_rope_attention
        return fused_rope_attention(q, k, v, **kw)
    if api in ("gqa", "mqa", "mqa3d"):
        m = getattr(mod, "attention", mod)  # the package keeps them in mlx_primitives.attention
        if "mask_case" in kw:
            kw = dict(kw)
            mask = _golden()[f"{kw.pop('mask_case')}__mask"]
            kw["mask"] = mask if mod is O else torch.from_numpy(mask).cuda()
        if api == "gqa":
            return m.gqa_attention(q, k, v, **kw)
        if api == "mqa3d":
            k, v = k[:, :, 0], v[:, :, 0]
        return m.mqa_attention(q, k, v, **kw)
    return mod.chunked_cross_attention(q, k, v, **kw)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_golden_fixtures_through_public_api(dtype):
    import mlx_primitives as mp
    g = _golden()
    cases = sorted({n.split("__")[0] for n in g.files if n.endswith("__out")})
    assert set(cases) == set(GOLDEN_CALLS)
    for case in cases:
        api, kw = GOLDEN_CALLS[case]
        meta = g[f"{case}__meta"]
        seed, std = int(meta[0]), float(meta[1])
        sq, skv = tuple(int(x) for x in meta[2:6]), tuple(int(x) for x in meta[6:10])
        (q, k, v), (nq, nk, nv) = inputs(sq, skv, dtype, seed=seed, std=std)
        out = _call(api, mp, q, k, v, kw)
        if dtype == torch.float32:
            # same inputs as the reference run: compare with its output directly
            tol = 2e-3 if "large_values" in case else 1e-4
            assert maxabs(out, np.nan_to_num(g[f"{case}__out"], nan=0.0)) <= tol, case
        else:
            # bf16-rounded inputs: compare with the oracle on those inputs
            want = _call(api, O, nq, nk, nv, kw)
            tol = 0.15 if "large_values" in case else 2e-2  # |o| ~ 10 there: bf16 ulp is 0.06
            assert maxabs(out, want) <= tol, case


def test_host_tensors_are_staged_through_the_gpu():
    import mlx_primitives as mp
    q, k, v = (torch.from_numpy(a).to(torch.bfloat16) for a in O.make_qkv((1, 300, 2, 64), (1, 300, 2, 64), seed=18))
    o_host = mp.flash_attention(q, k, v)
    assert o_host.device.type == "cpu"
    o_dev = mp.flash_attention(q.cuda(), k.cuda(), v.cuda())
    assert torch.equal(o_host, o_dev.cpu())


@pytest.mark.parametrize("B,H", [(2, 6), (3, 5), (1, 20)])
def test_host_bhsd_tensors_staged_in_head_pieces(B, H):
    # BHSD host tensors with few batches are pipelined in (batch, head-range) pieces; every
    # piece's output and LSE must land in its place, bit-identical to one device call
    from mlx_primitives.attention._core import attention_forward
    q, k, v = (torch.from_numpy(np.ascontiguousarray(np.swapaxes(a, 1, 2))).to(torch.bfloat16)
               for a in O.make_qkv((B, 200, H, 64), (B, 230, H, 64), seed=40 + B))
    kw = dict(layout="BHSD", scale=0.125, causal=True, q_offset=30, return_lse=True)
    o_host, lse_host = attention_forward(q, k, v, **kw)
    assert o_host.device.type == "cpu" and lse_host.device.type == "cpu"
    o_dev, lse_dev = attention_forward(q.cuda(), k.cuda(), v.cuda(), **kw)
    assert torch.equal(o_host, o_dev.cpu())
    assert torch.equal(lse_host, lse_dev.cpu())


def test_padded_head_dims():
    import mlx_primitives as mp
    for D, dt in ((48, torch.bfloat16), (100, torch.bfloat16), (16, torch.float32), (80, torch.float32)):
        (q, k, v), (nq, nk, nv) = inputs((1, 150, 2, D), (1, 150, 2, D), dt, seed=D)
        o = mp.flash_attention(q, k, v)
        assert o.shape == q.shape
        assert maxabs(o, O.flash_attention(nq, nk, nv)) <= TOL[dt]
