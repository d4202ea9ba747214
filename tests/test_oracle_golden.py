"""Pin the CPU oracle to the reference: every golden case in tests/golden/reference_outputs.npz
is the output of the reference's own code path (see tests/golden/make_golden.py); the oracle's
semantic definition (fp64) and its blockwise fp32 restatements must reproduce it."""

from pathlib import Path

import numpy as np
import pytest

from oracle import attention_oracle as O

GOLDEN = np.load(Path(__file__).parent / "golden" / "reference_outputs.npz")
CASES = sorted({k.split("__")[0] for k in GOLDEN.files if k.endswith("__out")})

# case -> (semantic oracle call, blockwise restatement call or None, atol)
SEMANTIC = {
    "flash_bshd_tiled_causal_d64": (lambda q, k, v: O.flash_attention(q, k, v, causal=True),
                                    lambda q, k, v: O.tiled_flash_attention(q, k, v, 0.125, True)),
    "flash_bshd_tiled_noncausal_d64": (lambda q, k, v: O.flash_attention(q, k, v, causal=False),
                                       lambda q, k, v: O.tiled_flash_attention(q, k, v, 0.125, False)),
    "flash_bshd_tiled_causal_d128_b16": (
        lambda q, k, v: O.flash_attention(q, k, v, causal=True),
        lambda q, k, v: O.tiled_flash_attention(q, k, v, 128 ** -0.5, True, 16, 16)),
    "flash_bshd_tiled_causal_d32_ragged": (
        lambda q, k, v: O.flash_attention(q, k, v, causal=True),
        lambda q, k, v: O.tiled_flash_attention(q, k, v, 32 ** -0.5, True)),
    "flash_bshd_dense_causal_d64": (lambda q, k, v: O.flash_attention(q, k, v, causal=True), None),
    "flash_bshd_dense_scale_d64": (lambda q, k, v: O.flash_attention(q, k, v, scale=0.3, causal=False), None),
    "flash_bshd_single_token": (lambda q, k, v: O.flash_attention(q, k, v, causal=True), None),
    "flash_bshd_large_values": (lambda q, k, v: O.flash_attention(q, k, v, causal=True), None),
    "flash_bhsd_causal_d128": (lambda q, k, v: O.flash_attention(q, k, v, causal=True, layout="BHSD"), None),
    "flash_bhsd_noncausal_d64": (lambda q, k, v: O.flash_attention(q, k, v, causal=False, layout="BHSD"), None),
    "swa_tiled_causal_w37": (
        lambda q, k, v: O.sliding_window_attention(q, k, v, 37, causal=True),
        lambda q, k, v: O.tiled_sliding_window_attention(q, k, v, 37, 0.125, True)),
    "swa_tiled_bidir_w20": (
        lambda q, k, v: O.sliding_window_attention(q, k, v, 20, causal=False),
        lambda q, k, v: O.tiled_sliding_window_attention(q, k, v, 20, 0.125, False)),
    "swa_tiled_causal_w130_d128": (
        lambda q, k, v: O.sliding_window_attention(q, k, v, 130, causal=True),
        lambda q, k, v: O.tiled_sliding_window_attention(q, k, v, 130, 128 ** -0.5, True)),
    "swa_dense_causal_w5": (lambda q, k, v: O.sliding_window_attention(q, k, v, 5, scale=0.125, causal=True), None),
    "chunked_loop_noncausal": (
        lambda q, k, v: O.chunked_cross_attention(q, k, v, 128),
        lambda q, k, v: O.chunked_cross_attention_loop(q, k, v, 128, 0.125)),
    "chunked_loop_causal": (
        lambda q, k, v: O.chunked_cross_attention(q, k, v, 64, causal=True),
        lambda q, k, v: O.chunked_cross_attention_loop(q, k, v, 64, 0.125, True)),
    "chunked_loop_q_longer_causal": (
        lambda q, k, v: O.chunked_cross_attention(q, k, v, 64, causal=True),
        lambda q, k, v: O.chunked_cross_attention_loop(q, k, v, 64, 0.125, True)),
    "chunked_dense_short_kv": (lambda q, k, v: O.chunked_cross_attention(q, k, v, 1024), None),
    "gqa_g4_causal_d64": (lambda q, k, v: O.gqa_attention(q, k, v, 4, causal=True), None),
    "gqa_g2_noncausal_d128": (lambda q, k, v: O.gqa_attention(q, k, v, 2, causal=False), None),
    "gqa_g2_causal_kv_longer_d64": (
        lambda q, k, v: O.gqa_attention(q, k, v, 2, scale=0.2, causal=True), None),
    "mqa_causal_d64": (lambda q, k, v: O.mqa_attention(q, k, v, causal=True), None),
    "mqa_3d_kv_noncausal_d128": (
        lambda q, k, v: O.mqa_attention(q, k[:, :, 0], v[:, :, 0], causal=False), None),
    "gqa_mask_bias_g2_d64": (
        lambda q, k, v: O.gqa_attention(q, k, v, 2, mask=GOLDEN["gqa_mask_bias_g2_d64__mask"]),
        None),
    "gqa_mask_exclude_causal_d128": (
        lambda q, k, v: O.gqa_attention(q, k, v, 2, causal=True,
                                        mask=GOLDEN["gqa_mask_exclude_causal_d128__mask"]), None),
    "mqa_mask_head_bias_d64": (
        lambda q, k, v: O.mqa_attention(q, k, v, mask=GOLDEN["mqa_mask_head_bias_d64__mask"]),
        None),
    "rope_only_offset7_d64": (
        lambda q, k, v: O.rope(q, *O.precompute_rope_cache(80, 64), offset=7), None),
    "fused_rope_causal_d64": (lambda q, k, v: O.fused_rope_attention(q, k, v, causal=True), None),
    "fused_rope_offsets_noncausal_d128": (
        lambda q, k, v: O.fused_rope_attention(q, k, v, q_offset=30, kv_offset=0, causal=False),
        None),
    "fused_rope_decode_causal_base500": (
        lambda q, k, v: O.fused_rope_attention(q, k, v, rope_base=500.0, q_offset=32, causal=True),
        None),
}


def _paged(case):
    """Oracle call of a paged-attention case: tables, lengths and options are stored with it."""
    def call(q, k, v):
        bs, causal, alibi, scale = GOLDEN[f"{case}__opts"]
        slopes = O.get_alibi_slopes(q.shape[2]) if alibi else None
        return O.paged_attention(q, k, v, GOLDEN[f"{case}__bt"], GOLDEN[f"{case}__ctx"],
                                 scale=None if scale < 0 else float(scale), block_size=int(bs),
                                 causal=bool(causal), alibi_slopes=slopes)
    return call


SEMANTIC.update({c: (_paged(c), None) for c in CASES if c.startswith("paged_")})


def golden_inputs(case):
    meta = GOLDEN[f"{case}__meta"]
    seed, std = int(meta[0]), float(meta[1])
    shape_q, shape_kv = tuple(int(x) for x in meta[2:6]), tuple(int(x) for x in meta[6:10])
    q, k, v = O.make_qkv(shape_q, shape_kv, seed=seed, std=std)
    return q, k, v


def test_every_case_has_an_oracle():
    assert set(CASES) == set(SEMANTIC)


@pytest.mark.parametrize("case", CASES)
def test_inputs_regenerate_bit_exact(case):
    import hashlib

    q, k, v = golden_inputs(case)
    h = hashlib.sha256()
    for a in (q, k, v):
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    assert h.hexdigest()[:16] == str(GOLDEN[f"{case}__digest"])


@pytest.mark.parametrize("case", CASES)
def test_semantic_oracle_matches_reference(case):
    q, k, v = golden_inputs(case)
    want = GOLDEN[f"{case}__out"]
    got = SEMANTIC[case][0](q, k, v)
    # std-10 inputs give scores of magnitude ~100, where the reference's fp32 softmax differs
    # from fp64 by ~1e-4 relative.
    tol = 1e-3 if "large_values" in case else 2e-5
    np.testing.assert_allclose(got, want, rtol=max(tol, 1e-4), atol=tol)


@pytest.mark.parametrize("case", [c for c in CASES if SEMANTIC[c][1] is not None])
def test_blockwise_restatement_matches_reference(case):
    q, k, v = golden_inputs(case)
    want = GOLDEN[f"{case}__out"]
    got = SEMANTIC[case][1](q, k, v)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)


def test_online_softmax_merge_and_chunk_helpers():
    q, k, v = O.make_qkv((1, 16, 2, 64), (1, 48, 2, 64), seed=119)
    o1, m1, l1 = O.compute_chunk_attention(q, k[:, :24], v[:, :24], 0.125, True, 30, 0)
    o2, m2, l2 = O.compute_chunk_attention(q, k[:, 24:], v[:, 24:], 0.125, True, 30, 24)
    om, mm, lm = O.online_softmax_merge(o1, m1, l1, o2, m2, l2)
    for name, got in dict(o1=o1, m1=m1, l1=l1, o2=o2, m2=m2, l2=l2, om=om, mm=mm, lm=lm).items():
        np.testing.assert_allclose(got, GOLDEN[f"merge__{name}"], rtol=1e-5, atol=1e-5, err_msg=name)
    # the merged, normalised result equals one-shot attention over the first 48 keys
    full = O.attention_bhsd(np.swapaxes(q, 1, 2), np.swapaxes(k, 1, 2), np.swapaxes(v, 1, 2),
                            0.125, causal=True, q_offset=30)
    np.testing.assert_allclose(np.swapaxes(om / lm[..., None], 1, 2), full, rtol=1e-4, atol=1e-5)


def test_rope_cache_matches_reference():
    cos, sin = O.precompute_rope_cache(80, 64)
    np.testing.assert_allclose(cos, GOLDEN["rope__cos_80x64"], atol=1e-6)
    np.testing.assert_allclose(sin, GOLDEN["rope__sin_80x64"], atol=1e-6)


def test_paged_helpers_match_reference():
    """get_alibi_slopes and create_block_table_from_lengths (paged_attention.py:17-41,
    387-440): the oracle's restatement and the package's torch versions."""
    import torch
    from mlx_primitives.cache import create_block_table_from_lengths, get_alibi_slopes

    for h in (8, 12):
        want = GOLDEN[f"paged__alibi_{h}"]
        np.testing.assert_array_equal(O.get_alibi_slopes(h), want)
        np.testing.assert_array_equal(get_alibi_slopes(h).numpy(), want)
    for lens, bs, mb, key in (([16, 33, 5], 16, None, "paged__table_16_33_5"),
                              ([7, 0, 64], 8, 10, "paged__table_7_0_64_b8_max10")):
        want = GOLDEN[key]
        np.testing.assert_array_equal(O.create_block_table_from_lengths(lens, bs, mb), want)
        got = create_block_table_from_lengths(torch.tensor(lens, dtype=torch.int32), bs, mb)
        assert got.dtype == torch.int32
        np.testing.assert_array_equal(got.numpy(), want)


def test_paged_empty_context_is_nan_in_reference():
    """The reference's softmax over an all-masked row gives NaN (context length 0); the oracle
    reproduces it, and the GPU tests expect zeros there instead."""
    want = GOLDEN["paged_decode_alibi_d128__out"]
    assert np.isnan(want[3]).all() and np.isfinite(want[:3]).all()


def test_masks_match_reference():
    np.testing.assert_array_equal(O.create_causal_mask(4, 7), GOLDEN["mask__causal_4x7"])
    np.testing.assert_array_equal(O.create_causal_mask(5, 5), GOLDEN["mask__causal_5x5"])
    np.testing.assert_array_equal(O.create_sliding_window_mask(8, 2, True), GOLDEN["mask__window_causal_8_2"])
    np.testing.assert_array_equal(O.create_sliding_window_mask(8, 2, False), GOLDEN["mask__window_bidir_8_2"])
    # the causal window keeps W + 1 keys: [i - W, i]
    assert O.create_sliding_window_mask(8, 2, True).sum(axis=1).tolist() == [1, 2, 3, 3, 3, 3, 3, 3]


def test_api_helpers_match_reference():
    import mlx_primitives as mp
    from mlx_primitives.attention import estimate_memory_savings, get_optimal_flash_config

    got = np.array([get_optimal_flash_config(s, d, 8) for s in (4, 64, 4096) for d in (32, 64, 128, 256)])
    np.testing.assert_array_equal(got, GOLDEN["api__flash_config"])
    np.testing.assert_allclose(estimate_memory_savings(512, 65536, 16, 64, 4096),
                               GOLDEN["api__memory_savings"])
    torch_mask = mp.create_sliding_window_mask(8, 2, causal=True).numpy()
    np.testing.assert_array_equal(torch_mask, GOLDEN["mask__window_causal_8_2"])
    from mlx_primitives.utils.masking import create_causal_mask

    np.testing.assert_array_equal(create_causal_mask(4, 7).numpy(), GOLDEN["mask__causal_4x7"])


# ---- known-answer tests from the reference's own test-suite semantics ----
def test_kat_single_token_returns_v():
    # tests/attention/test_flash.py:217-230
    q, k, v = O.make_qkv((1, 1, 1, 64), (1, 1, 1, 64), seed=3)
    np.testing.assert_allclose(O.flash_attention(q, k, v, causal=True), v, rtol=1e-6)


def test_kat_first_causal_row_sees_only_itself():
    # tests/attention/test_metal_python_parity.py:159-184
    q, k, v = O.make_qkv((1, 50, 2, 64), (1, 50, 2, 64), seed=4)
    o = O.flash_attention(q, k, v, causal=True)
    np.testing.assert_allclose(o[:, 0], v[:, 0], rtol=1e-6)


def test_kat_uniform_attention_gives_mean_position():
    # tests/attention/test_metal_python_parity.py:207-232: Q = K = 0 -> uniform weights over
    # the causal prefix; with V = position the output of row i is i / 2.
    S = 64
    q = np.zeros((1, S, 1, 64), np.float32)
    v = np.broadcast_to(np.arange(S, dtype=np.float32)[None, :, None, None], (1, S, 1, 64))
    o = O.flash_attention(q, q, v, causal=True)
    np.testing.assert_allclose(o[0, :, 0, 0], np.arange(S) / 2.0, rtol=1e-6)


def test_kat_full_window_equals_causal():
    # tests/attention/test_sliding_window.py:192-210
    q, k, v = O.make_qkv((1, 40, 2, 64), (1, 40, 2, 64), seed=5)
    np.testing.assert_allclose(O.sliding_window_attention(q, k, v, 1000, causal=True),
                               O.flash_attention(q, k, v, causal=True), rtol=1e-10)


def test_kat_chunk_size_invariance():
    # tests/attention/test_chunked.py:110-148
    q, k, v = O.make_qkv((1, 20, 2, 64), (1, 300, 2, 64), seed=6)
    dense = O.chunked_cross_attention(q, k, v)
    for c in (16, 64, 100, 1024):
        np.testing.assert_allclose(O.chunked_cross_attention_loop(q, k, v, c, 0.125), dense,
                                   rtol=1e-4, atol=1e-5)


def test_lse_merge_equals_one_shot():
    q, k, v = O.make_qkv((2, 3, 40, 64), (2, 3, 90, 64), seed=7)
    parts = [(0, 30), (30, 31), (31, 90)]
    os_, ls_ = [], []
    for a, b in parts:
        o, l = O.attention_bhsd(q, k[:, :, a:b], v[:, :, a:b], 0.125, return_lse=True)
        os_.append(o)
        ls_.append(l)
    o, lse = O.lse_merge(np.stack(os_), np.stack(ls_))
    want, want_lse = O.attention_bhsd(q, k, v, 0.125, return_lse=True)
    np.testing.assert_allclose(o, want, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, want_lse, rtol=1e-12)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_zigzag_ring_schedule_equals_causal_attention(world):
    S = 16 * 2 * world
    q, k, v = O.make_qkv((1, 2, S, 32), (1, 2, S, 32), seed=8)
    got = O.ring_reference(q, k, v, world, 0.2)
    want = O.attention_bhsd(q, k, v, 0.2, causal=True)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)


def test_round_bf16_matches_torch():
    import torch

    x = np.random.RandomState(0).standard_normal(10000).astype(np.float32) * 100
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(O.round_bf16(x), want)
