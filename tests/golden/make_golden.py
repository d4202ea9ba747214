"""Generate tests/golden/reference_outputs.npz by running the REFERENCE's own Python code.

zakkeown/mlx-primitives computes its attention with MLX (mlx >= 0.20; its benchmarks used
0.30.3), which is not installed here and cannot be (no network).  Its attention modules only
use a small set of mlx.core array functions on their CPU paths (full, zeros, arange, einsum,
where, max, exp, sum, maximum, concatenate, abs, softmax, transpose, triu, matmul via @), so
this script installs a numpy-backed stand-in for `mlx.core` with MLX's float32 defaults, loads
the reference's modules from the reference checkout WITHOUT modification, disables its SDPA /
Metal branches (as on an MLX build without them), and records what its own code returns:

  flash.py:257-316       _tiled_flash_attention   (flash_attention BSHD, S > 512)
  flash.py:479-525       _reference_flash_attention dense fallback (BSHD, short S)
  flash.py:172-192       BHSD branch, dense fallback with create_causal_mask
  sliding_window.py:363-511  _tiled_sliding_window_attention (causal and bidirectional)
  sliding_window.py:514-560  _reference_sliding_window_attention (dense mask)
  chunked.py:129-169     _chunked_cross_attention_impl (causal and not)
  chunked.py:172-203     _reference_cross_attention (Skv <= chunk_size)
  _online_softmax.py:42-176  online_softmax_merge / compute_chunk_attention
  utils/masking.py:14-66 create_causal_mask; sliding_window.py:628-656 create_sliding_window_mask
  grouped_query.py:195-261  gqa_attention;  multi_query.py:161-225  mqa_attention
  kernels/rope.py:223-255, 451-496  precompute_rope_cache, rope (Python path)
  kernels/fused_rope_attention.py:766-800, 939-985  fused_rope_attention (use_metal=False)
  cache/paged_attention.py:17-440  get_alibi_slopes, paged_attention (decode and prefill,
                         with and without ALiBi), create_block_table_from_lengths

Inputs come from numpy's legacy RandomState (frozen stream) through
oracle.attention_oracle.make_qkv, so tests regenerate them bit-for-bit from the seed; only the
outputs (and a checksum of each input set) are stored.

Run from the repository root, in a container that has the reference checkout:
    python tests/golden/make_golden.py --reference /path/to/mlx-primitives
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import sys
import types
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from oracle.attention_oracle import make_qkv  # noqa: E402

OUT = Path(__file__).with_name("reference_outputs.npz")


# ---------------------------------------------------------------------------------------
# numpy stand-in for mlx.core (float32 defaults, like MLX)
# ---------------------------------------------------------------------------------------
def _stand_in_mlx() -> types.ModuleType:
    mx = types.ModuleType("mlx.core")
    f32 = np.float32

    def _f(x):
        return np.asarray(x)

    def array(x, dtype=None):
        a = np.asarray(x)
        if dtype is not None:
            return a.astype(dtype)
        if a.dtype == np.float64:
            return a.astype(f32)
        return a

    mx.array = array
    mx.Dtype = type(np.dtype(f32))
    mx.float32, mx.float16, mx.uint32, mx.int32 = f32, np.float16, np.uint32, np.int32
    mx.bfloat16 = f32
    mx.full = lambda shape, val, dtype=None: np.full(shape, val, dtype=dtype or f32)
    mx.zeros = lambda shape, dtype=None: np.zeros(shape, dtype=dtype or f32)
    mx.ones = lambda shape, dtype=None: np.ones(shape, dtype=dtype or f32)
    def arange(*a, dtype=None, **k):
        r = np.arange(*a, **k)
        return r.astype(dtype) if dtype is not None else r.astype(np.int32)

    mx.arange = arange
    mx.outer = np.outer
    mx.cos = np.cos
    mx.sin = np.sin

    class _CustomFunction:  # @mx.custom_function: the recorded paths only call it
        def __init__(self, f):
            self.f = f

        def __call__(self, *a, **k):
            return self.f(*a, **k)

        def vjp(self, g):
            return g

    mx.custom_function = _CustomFunction
    mx.einsum = lambda spec, *ops: np.einsum(spec, *ops).astype(np.result_type(*ops))
    mx.where = lambda c, a, b: np.where(c, a, b).astype(np.result_type(_f(a), _f(b)))
    mx.max = lambda x, axis=None, keepdims=False: np.max(x, axis=axis, keepdims=keepdims)
    mx.exp = np.exp
    mx.sum = lambda x, axis=None, keepdims=False: np.sum(x, axis=axis, keepdims=keepdims, dtype=x.dtype)
    mx.maximum = np.maximum
    mx.take = lambda a, idx, axis=None: np.take(a, idx, axis=axis)
    mx.cumsum = lambda x, axis=None: np.cumsum(x, axis=axis)
    mx.concatenate = lambda arrs, axis=0: np.concatenate(arrs, axis=axis)
    mx.abs = np.abs
    mx.transpose = lambda x, axes=None: np.transpose(x, axes)
    mx.triu = lambda x, k=0: np.triu(x, k=k)
    mx.contiguous = np.ascontiguousarray
    mx.broadcast_to = lambda x, shape: np.broadcast_to(x, shape)
    mx.eval = lambda *a, **k: None

    def softmax(x, axis=-1):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / np.sum(e, axis=axis, keepdims=True)

    mx.softmax = softmax
    # attributes the modules reference in annotations; the branches that would call them are
    # disabled after import (module flags) and by use_metal=False.
    fast = types.SimpleNamespace(metal_kernel=object, scaled_dot_product_attention=None)
    mx.fast = fast
    mx.random = types.SimpleNamespace()
    mx.default_stream = lambda *a: None
    mx.default_device = lambda: None
    return mx


def load_reference(ref_root: Path):
    mlx = types.ModuleType("mlx")
    core = _stand_in_mlx()
    mlx.core = core
    # mlx.nn only provides base classes for the module definitions; the functional entry points
    # recorded below (gqa_attention, mqa_attention) do not touch it.
    nn = types.ModuleType("mlx.nn")
    nn.Module = type("Module", (), {"__init__": lambda self, *a, **k: None})
    nn.Linear = lambda *a, **k: None
    mlx.nn = nn
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = core
    sys.modules["mlx.nn"] = nn
    pkg_dir = ref_root / "mlx_primitives"
    for name, sub in [("mlx_primitives", ""), ("mlx_primitives.attention", "attention"),
                      ("mlx_primitives.kernels", "kernels"), ("mlx_primitives.utils", "utils"),
                      ("mlx_primitives.cache", "cache")]:
        m = types.ModuleType(name)
        m.__path__ = [str(pkg_dir / sub) if sub else str(pkg_dir)]
        sys.modules[name] = m
    hw = types.ModuleType("mlx_primitives.hardware")
    hw.get_chip_info = lambda *a, **k: None
    hw.get_optimal_attention_config = lambda *a, **k: None
    sys.modules["mlx_primitives.hardware"] = hw
    mods = {}
    for n in ["_online_softmax", "flash", "sliding_window", "chunked"]:
        mods[n] = importlib.import_module(f"mlx_primitives.attention.{n}")
    mods["masking"] = importlib.import_module("mlx_primitives.utils.masking")
    mods["grouped_query"] = importlib.import_module("mlx_primitives.attention.grouped_query")
    mods["multi_query"] = importlib.import_module("mlx_primitives.attention.multi_query")
    mods["rope"] = importlib.import_module("mlx_primitives.kernels.rope")
    mods["fused_rope"] = importlib.import_module("mlx_primitives.kernels.fused_rope_attention")
    mods["paged"] = importlib.import_module("mlx_primitives.cache.paged_attention")
    for n in ["rope", "fused_rope"]:
        setattr(mods[n], "_USE_METAL_KERNELS", False)
    setattr(mods["fused_rope"], "_HAS_SDPA", False)
    for n in ["flash", "sliding_window", "chunked"]:
        setattr(mods[n], "_HAS_SDPA", False)
        setattr(mods[n], "_HAS_METAL", False)
    return mods


def digest(*arrs) -> str:
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()[:16]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the zakkeown/mlx-primitives checkout (read only)")
    args = ap.parse_args()
    mods = load_reference(Path(args.reference))
    fl, sw, ch, osm, mk = (mods[n] for n in ["flash", "sliding_window", "chunked", "_online_softmax", "masking"])
    out = {}

    def case(name, seed, shape_q, shape_kv, fn, std=1.0):
        q, k, v = make_qkv(shape_q, shape_kv, seed=seed, std=std)
        res = np.asarray(fn(q, k, v), dtype=np.float32)
        out[f"{name}__out"] = res
        out[f"{name}__meta"] = np.array([seed, std] + list(shape_q) + list(shape_kv), dtype=np.float64)
        out[f"{name}__digest"] = np.array(digest(q, k, v))
        print(f"{name:34s} q{shape_q} kv{shape_kv} -> {res.shape}")

    # flash_attention, BSHD, tiled path (S > 512): flash.py:257-316
    case("flash_bshd_tiled_causal_d64", 101, (1, 520, 2, 64), (1, 520, 2, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False))
    case("flash_bshd_tiled_noncausal_d64", 102, (1, 530, 1, 64), (1, 530, 1, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=False, use_metal=False))
    case("flash_bshd_tiled_causal_d128_b16", 103, (1, 600, 1, 128), (1, 600, 1, 128),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, block_q=16, block_kv=16,
                                            use_metal=False))
    case("flash_bshd_tiled_causal_d32_ragged", 104, (6, 300, 1, 32), (6, 300, 1, 32),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False))
    # flash_attention, BSHD, dense reference path (short S): flash.py:479-525
    case("flash_bshd_dense_causal_d64", 105, (2, 64, 3, 64), (2, 64, 3, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False))
    case("flash_bshd_dense_scale_d64", 106, (1, 100, 2, 64), (1, 100, 2, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, scale=0.3, causal=False, use_metal=False))
    case("flash_bshd_single_token", 107, (1, 1, 1, 64), (1, 1, 1, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False))
    case("flash_bshd_large_values", 108, (1, 130, 1, 64), (1, 130, 1, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False), std=10.0)
    # flash_attention, BHSD branch (dense fallback with create_causal_mask): flash.py:172-192
    case("flash_bhsd_causal_d128", 109, (2, 2, 200, 128), (2, 2, 200, 128),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=True, use_metal=False, layout="BHSD"))
    case("flash_bhsd_noncausal_d64", 110, (1, 3, 150, 64), (1, 3, 150, 64),
         lambda q, k, v: fl.flash_attention(q, k, v, causal=False, use_metal=False, layout="BHSD"))
    # sliding window: sliding_window.py:363-511 (tiled) and 514-560 (dense)
    case("swa_tiled_causal_w37", 111, (1, 300, 2, 64), (1, 300, 2, 64),
         lambda q, k, v: sw.sliding_window_attention(q, k, v, window_size=37, causal=True, use_metal=False))
    case("swa_tiled_bidir_w20", 112, (1, 200, 1, 64), (1, 200, 1, 64),
         lambda q, k, v: sw.sliding_window_attention(q, k, v, window_size=20, causal=False, use_metal=False))
    case("swa_tiled_causal_w130_d128", 113, (1, 400, 1, 128), (1, 400, 1, 128),
         lambda q, k, v: sw.sliding_window_attention(q, k, v, window_size=130, causal=True, use_metal=False))
    case("swa_dense_causal_w5", 114, (1, 40, 1, 64), (1, 40, 1, 64),
         lambda q, k, v: sw._reference_sliding_window_attention(q, k, v, 5, 0.125, True))
    # chunked cross attention: chunked.py:129-169 and 172-203
    case("chunked_loop_noncausal", 115, (2, 50, 2, 64), (2, 700, 2, 64),
         lambda q, k, v: ch.chunked_cross_attention(q, k, v, chunk_size=128, use_metal=False),
         std=0.5)
    case("chunked_loop_causal", 116, (1, 300, 1, 64), (1, 300, 1, 64),
         lambda q, k, v: ch.chunked_cross_attention(q, k, v, chunk_size=64, causal=True, use_metal=False))
    case("chunked_loop_q_longer_causal", 117, (1, 260, 1, 64), (1, 200, 1, 64),
         lambda q, k, v: ch.chunked_cross_attention(q, k, v, chunk_size=64, causal=True, use_metal=False))
    case("chunked_dense_short_kv", 118, (1, 30, 2, 128), (1, 100, 2, 128),
         lambda q, k, v: ch.chunked_cross_attention(q, k, v, chunk_size=1024, use_metal=False))

    # grouped-query / multi-query functional forms: grouped_query.py:195-261, multi_query.py:161-225
    gq, mq = mods["grouped_query"], mods["multi_query"]
    case("gqa_g4_causal_d64", 120, (2, 96, 8, 64), (2, 96, 2, 64),
         lambda q, k, v: gq.gqa_attention(q, k, v, num_kv_groups=4, causal=True))
    case("gqa_g2_noncausal_d128", 121, (1, 70, 4, 128), (1, 90, 2, 128),
         lambda q, k, v: gq.gqa_attention(q, k, v, num_kv_groups=2, causal=False))
    case("gqa_g2_causal_kv_longer_d64", 122, (1, 40, 6, 64), (1, 130, 3, 64),
         lambda q, k, v: gq.gqa_attention(q, k, v, num_kv_groups=2, scale=0.2, causal=True))
    case("mqa_causal_d64", 123, (2, 80, 4, 64), (2, 80, 1, 64),
         lambda q, k, v: mq.mqa_attention(q, k, v, causal=True))
    case("mqa_3d_kv_noncausal_d128", 124, (1, 50, 3, 128), (1, 75, 1, 128),
         lambda q, k, v: mq.mqa_attention(q, k[:, :, 0], v[:, :, 0], causal=False))
    # custom additive masks (grouped_query.py:253-254, multi_query.py:218-219), stored with the
    # case as "<case>__mask": a (seq_q, seq_kv) bias, a (batch, 1, seq_q, seq_kv) exclusion mask
    # (-inf entries, every row keeps a key) with causal masking, a per-head bias for mqa
    rs = np.random.RandomState(7)
    m1 = (rs.standard_normal((60, 90)) * 2.0).astype(np.float32)
    out["gqa_mask_bias_g2_d64__mask"] = m1
    case("gqa_mask_bias_g2_d64", 140, (2, 60, 4, 64), (2, 90, 2, 64),
         lambda q, k, v: gq.gqa_attention(q, k, v, num_kv_groups=2, mask=m1))
    m2 = np.where(rs.rand(2, 1, 48, 48) < 0.3, -np.inf, 0.0).astype(np.float32)
    m2[..., np.arange(48), np.arange(48)] = 0.0  # the diagonal stays: no empty row under causal
    out["gqa_mask_exclude_causal_d128__mask"] = m2
    case("gqa_mask_exclude_causal_d128", 141, (2, 48, 6, 128), (2, 48, 3, 128),
         lambda q, k, v: gq.gqa_attention(q, k, v, num_kv_groups=2, mask=m2, causal=True))
    m3 = (rs.standard_normal((1, 3, 33, 70)) * 0.5).astype(np.float32)
    out["mqa_mask_head_bias_d64__mask"] = m3
    case("mqa_mask_head_bias_d64", 142, (1, 33, 3, 64), (1, 70, 1, 64),
         lambda q, k, v: mq.mqa_attention(q, k, v, mask=m3))

    # RoPE (kernels/rope.py:223-255, 451-496) and RoPE + attention
    # (kernels/fused_rope_attention.py:766-800 via fused_rope_attention(use_metal=False))
    ro, fr = mods["rope"], mods["fused_rope"]
    cos, sin = ro.precompute_rope_cache(80, 64, base=10000.0)
    out["rope__cos_80x64"] = np.asarray(cos, dtype=np.float32)
    out["rope__sin_80x64"] = np.asarray(sin, dtype=np.float32)
    case("rope_only_offset7_d64", 125, (1, 50, 2, 64), (1, 50, 2, 64),
         lambda q, k, v: ro.rope(q, cos, sin, 7))
    case("fused_rope_causal_d64", 126, (1, 96, 2, 64), (1, 96, 2, 64),
         lambda q, k, v: fr.fused_rope_attention(q, k, v, causal=True, use_metal=False))
    case("fused_rope_offsets_noncausal_d128", 127, (1, 40, 2, 128), (1, 70, 2, 128),
         lambda q, k, v: fr.fused_rope_attention(q, k, v, q_offset=30, kv_offset=0,
                                                 causal=False, use_metal=False))
    case("fused_rope_decode_causal_base500", 128, (2, 1, 4, 64), (2, 33, 4, 64),
         lambda q, k, v: fr.fused_rope_attention(q, k, v, rope_base=500.0, q_offset=32,
                                                 causal=True, use_metal=False))

    # paged attention (cache/paged_attention.py): q from make_qkv's q, the pools from its k/v
    # (shape_kv = (num_blocks, block_size, heads, dim)); tables, lengths and slopes are stored.
    pa = mods["paged"]

    def paged_case(name, seed, B, Sq, H, D, num_blocks, bs, tables, lens, causal=True,
                   alibi=False, scale=None):
        bt = np.asarray(tables, dtype=np.int32)
        cl = np.asarray(lens, dtype=np.int32)
        slopes = pa.get_alibi_slopes(H) if alibi else None
        out[f"{name}__bt"] = bt
        out[f"{name}__ctx"] = cl
        out[f"{name}__opts"] = np.array([bs, int(causal), int(alibi),
                                         -1.0 if scale is None else scale], dtype=np.float64)
        case(name, seed, (B, Sq, H, D), (num_blocks, bs, H, D),
             lambda q, k, v: pa.paged_attention(q, k, v, bt, cl, scale=scale, block_size=bs,
                                                causal=causal, alibi_slopes=slopes))

    # decode, the reference test's tables (tests/cache/test_paged_attention.py:164-196)
    paged_case("paged_decode_batch_d64", 130, 4, 1, 8, 64, 20, 16,
               [[0, -1, -1], [1, 2, -1], [3, 4, 5], [6, 7, -1]], [16, 32, 48, 25])
    # decode with ALiBi, permuted blocks, a one-token context and an empty one (NaN row)
    paged_case("paged_decode_alibi_d128", 131, 4, 1, 4, 128, 12, 16,
               [[7, 2, 9, 0], [5, -1, -1, -1], [11, 3, 1, 4], [6, -1, -1, -1]],
               [40, 1, 64, 0], alibi=True)
    # decode, head_dim 32, block 8: a missing block inside the context, a length past the
    # table's capacity, and an explicit scale
    paged_case("paged_decode_hole_d32", 132, 3, 1, 2, 32, 16, 8,
               [[0, 1, -1, 2, 3], [4, 5, 6, 7, 8], [9, 10, -1, -1, -1]], [37, 90, 11],
               scale=0.3)
    # prefill, causal (query i sees positions <= i), contexts longer and shorter than seq_q
    paged_case("paged_prefill_causal_d64", 133, 2, 20, 8, 64, 10, 16,
               [[0, 1, 2], [3, 4, -1]], [45, 13])
    # prefill, ALiBi, bidirectional, block 32
    paged_case("paged_prefill_alibi_noncausal_d64", 134, 1, 16, 4, 64, 4, 32,
               [[2, 0]], [40], causal=False, alibi=True)
    # prefill, ALiBi and causal, head_dim 128
    paged_case("paged_prefill_alibi_causal_d128", 135, 2, 12, 2, 128, 6, 16,
               [[5, 1], [0, -1]], [20, 5], alibi=True)
    out["paged__alibi_8"] = np.asarray(pa.get_alibi_slopes(8), dtype=np.float32)
    out["paged__alibi_12"] = np.asarray(pa.get_alibi_slopes(12), dtype=np.float32)
    out["paged__table_16_33_5"] = np.asarray(
        pa.create_block_table_from_lengths(np.array([16, 33, 5], dtype=np.int32), 16))
    out["paged__table_7_0_64_b8_max10"] = np.asarray(
        pa.create_block_table_from_lengths(np.array([7, 0, 64], dtype=np.int32), 8, max_blocks=10))

    # _online_softmax: merge and chunk helpers
    q, k, v = make_qkv((1, 16, 2, 64), (1, 48, 2, 64), seed=119)
    o1, m1, l1 = osm.compute_chunk_attention(q, k[:, :24], v[:, :24], 0.125, causal=True,
                                             q_offset=30, kv_offset=0)
    o2, m2, l2 = osm.compute_chunk_attention(q, k[:, 24:], v[:, 24:], 0.125, causal=True,
                                             q_offset=30, kv_offset=24)
    om, mm, lm = osm.online_softmax_merge(o1, m1, l1, o2, m2, l2)
    for nm, a in dict(o1=o1, m1=m1, l1=l1, o2=o2, m2=m2, l2=l2, om=om, mm=mm, lm=lm).items():
        out[f"merge__{nm}"] = np.asarray(a, dtype=np.float32)
    out["merge__digest"] = np.array(digest(q, k, v))

    # masks
    out["mask__causal_4x7"] = np.asarray(mk.create_causal_mask(4, 7), dtype=np.float32)
    out["mask__causal_5x5"] = np.asarray(mk.create_causal_mask(5, 5), dtype=np.float32)
    out["mask__window_causal_8_2"] = np.asarray(sw.create_sliding_window_mask(8, 2, causal=True))
    out["mask__window_bidir_8_2"] = np.asarray(sw.create_sliding_window_mask(8, 2, causal=False))
    out["api__flash_config"] = np.array([fl.get_optimal_flash_config(s, d, 8)
                                         for s in (4, 64, 4096) for d in (32, 64, 128, 256)])
    out["api__memory_savings"] = np.array(ch.estimate_memory_savings(512, 65536, 16, 64, 4096),
                                          dtype=np.float64)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
