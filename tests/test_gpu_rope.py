"""RoPE (mlxp_rope / mlxp_rope_qk) and RoPE + attention on the GPU against the oracle
restatement of the reference's rope / fused_rope_attention (pinned to the reference's own
outputs in tests/golden).  Tolerances: fp32 <= 1e-4 (the fp32 gate; the cos/sin of large
angles carry the fp32 rounding of the angle itself, a few 1e-6 relative, here and in the
reference); bf16/fp16 rotations <= one ulp of the value (1e-2 relative); attention outputs
bf16 <= 2e-2."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _x(shape, dtype, seed):
    a = np.random.RandomState(seed).standard_normal(shape).astype(np.float32)
    t = torch.from_numpy(a).cuda().to(dtype)
    return t, t.float().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128, 36])  # 36: half 18, the unvectorised path
@pytest.mark.parametrize("offset", [0, 5])
def test_rope_matches_oracle(dtype, D, offset):
    from mlx_primitives.kernels import precompute_rope_cache, rope

    x, nx = _x((2, 77, 3, D), dtype, seed=D + offset)
    cos, sin = precompute_rope_cache(100, D)
    y = rope(x, cos, sin, offset)
    ncos, nsin = O.precompute_rope_cache(100, D)
    want = O.rope(nx, ncos, nsin, offset)
    got = y.float().cpu().numpy()
    if dtype == torch.float32:
        assert np.max(np.abs(got - want)) <= 1e-4
    else:
        assert np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-2)) <= 1e-2


def test_rope_strided_input_and_out_of_range_positions():
    from mlx_primitives.kernels import precompute_rope_cache, rope

    x, nx = _x((2, 4, 64, 128), torch.bfloat16, seed=1)  # BHSD storage
    xv = x.transpose(1, 2)                                # BSHD view with strides
    cos, sin = precompute_rope_cache(64, 128)
    y = rope(xv, cos, sin, 0)
    want = O.rope(nx.transpose(0, 2, 1, 3), *O.precompute_rope_cache(64, 128), 0)
    assert np.max(np.abs(y.float().cpu().numpy() - want) / np.maximum(np.abs(want), 1e-2)) <= 1e-2
    with pytest.raises(ValueError, match="exceed"):
        rope(xv, cos, sin, 1)  # positions 1..64 need 65 cache rows


def test_rope_qk_grouped_heads_and_offsets():
    from mlx_primitives.kernels import fast_rope_qk, precompute_rope_cache

    q, nq = _x((2, 20, 8, 64), torch.bfloat16, seed=3)
    k, nk = _x((2, 50, 2, 64), torch.bfloat16, seed=4)
    cos, sin = precompute_rope_cache(64, 64)
    qo, ko = fast_rope_qk(q, k, cos, sin, 30, k_offset=0)
    ncos, nsin = O.precompute_rope_cache(64, 64)
    for got, want in ((qo, O.rope(nq, ncos, nsin, 30)), (ko, O.rope(nk, ncos, nsin, 0))):
        got = got.float().cpu().numpy()
        assert np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-2)) <= 1e-2


@pytest.mark.parametrize("causal", [True, False])
def test_fused_rope_attention_bf16(causal):
    from mlx_primitives.kernels import fused_rope_attention

    q, nq = _x((2, 600, 4, 128), torch.bfloat16, seed=11)
    k, nk = _x((2, 600, 4, 128), torch.bfloat16, seed=12)
    v, nv = _x((2, 600, 4, 128), torch.bfloat16, seed=13)
    out = fused_rope_attention(q, k, v, causal=causal)
    # the kernel rotates in fp32 and rounds Q/K to bf16 before the bf16 attention: the oracle
    # sees the same rounding
    ncos, nsin = O.precompute_rope_cache(600, 128)
    qr = O.round_bf16(O.rope(nq, ncos, nsin, 0).astype(np.float32))
    kr = O.round_bf16(O.rope(nk, ncos, nsin, 0).astype(np.float32))
    want = O.flash_attention(qr, kr, nv, causal=causal)
    assert np.max(np.abs(out.float().cpu().numpy() - want)) <= 2e-2


def test_fused_rope_module_with_cache():
    from mlx_primitives.kernels import FusedRoPEFlashAttention

    torch.manual_seed(0)
    mod = FusedRoPEFlashAttention(256, 4, causal=True).cuda()
    x = torch.randn(2, 40, 256, device="cuda")
    out, cache = mod(x)
    with torch.no_grad():
        q = mod.q_proj(x).reshape(2, 40, 4, 64).cpu().numpy()
        k = mod.k_proj(x).reshape(2, 40, 4, 64).cpu().numpy()
        v = mod.v_proj(x).reshape(2, 40, 4, 64).cpu().numpy()
        att = O.fused_rope_attention(q, k, v, causal=True).astype(np.float32)
        want = mod.out_proj(torch.from_numpy(att.reshape(2, 40, -1)).cuda())
    assert float((out - want).abs().max().detach()) <= 1e-3
    x1 = torch.randn(2, 1, 256, device="cuda")
    out1, cache1 = mod(x1, cache=cache, offset=40)
    assert cache1[0].shape == (2, 41, 4, 64) and out1.shape == (2, 1, 256)


def _two_launch(q, k, v, cos, sin, q_off, k_off, causal):
    """mlxp_rope_qk, then attention on the rotated tensors (the path the single launch replaces)."""
    from mlx_primitives.attention._core import attention_forward
    from mlx_primitives.kernels import fast_rope_qk

    qr, kr = fast_rope_qk(q, k, cos, sin, q_off, k_offset=k_off)
    Sq, Skv = q.shape[1], k.shape[1]
    return attention_forward(qr, kr, v, layout="BSHD", scale=q.shape[-1] ** -0.5, causal=causal,
                             q_offset=(Skv - Sq) if causal else 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("shape,causal,offsets", [
    ((2, 1000, 4), True, (0, 0)),       # S not a multiple of the 256-row rotation chunk
    ((1, 300, 3, 700), True, (400, 0)),  # cached keys: Sq < Skv, query positions after them
    ((3, 257, 2, 257), False, (7, 7)),
])
def test_rope_attention_single_launch_is_the_two_launch_result(dtype, D, shape, causal, offsets):
    """mlxp_rope_attn_fwd (rotation items inside the attention launch) against mlxp_rope_qk +
    attention: bit-identical (same rotation arithmetic and rounding, same attention kernel),
    and within the bf16/fp16 tolerance of the oracle's rope + attention."""
    import importlib

    from mlx_primitives.kernels import fused_rope_attention, precompute_rope_cache
    M = importlib.import_module("mlx_primitives.kernels.fused_rope_attention")

    B, Sq, H = shape[:3]
    Skv = shape[3] if len(shape) > 3 else Sq
    q, nq = _x((B, Sq, H, D), dtype, seed=D + Sq)
    k, nk = _x((B, Skv, H, D), dtype, seed=D + Skv + 1)
    v, nv = _x((B, Skv, H, D), dtype, seed=D + 2)
    q_off, k_off = offsets
    n_pos = max(Sq + q_off, Skv + k_off)
    cos, sin = precompute_rope_cache(n_pos, D)
    assert M._single_launch_applies(q, k, v, cos, sin)
    got = fused_rope_attention(q, k, v, cos_cache=cos, sin_cache=sin, q_offset=q_off,
                               kv_offset=k_off, causal=causal)
    want2 = _two_launch(q, k, v, cos, sin, q_off, k_off, causal)
    torch.cuda.synchronize()
    assert torch.equal(got, want2)
    ncos, nsin = O.precompute_rope_cache(n_pos, D)
    want = O.fused_rope_attention(nq, nk, nv, cos_cache=ncos, sin_cache=nsin, q_offset=q_off,
                                  kv_offset=k_off, causal=causal)
    assert np.max(np.abs(got.float().cpu().numpy() - want)) <= 2e-2


def test_rope_attention_single_launch_config2_shape_and_repeat():
    """The config-2 shape (B4 S4096 H32 D128, BSHD, causal) twice in a row: bit-identical to
    the two-launch path each time (the workspace counters are cleared per launch)."""
    from mlx_primitives.kernels import fused_rope_attention, precompute_rope_cache

    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    q, k, v = (torch.randn((4, 4096, 32, 128), generator=g, device="cuda").bfloat16()
               for _ in range(3))
    cos, sin = precompute_rope_cache(4096, 128)
    want = _two_launch(q, k, v, cos, sin, 0, 0, True)
    for _ in range(2):
        got = fused_rope_attention(q, k, v, cos_cache=cos, sin_cache=sin, causal=True)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
