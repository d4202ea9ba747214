"""Attention backward on the GPU (mlxp_attn_bwd through torch autograd of the public API)
against the oracle's backward (oracle.attention_bwd_bhsd, pinned to fp64 autodiff in
tests/test_oracle_backward.py).  Tolerances, max-abs against fp64 on the same inputs:
fp32 <= 1e-4 * (1 + max|grad|); bf16/fp16 <= 2e-2 * (1 + max|grad|) (outputs rounded to
the input type)."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _make(shape_q, shape_kv, dtype, seed, std=1.0):
    rs = np.random.RandomState(seed)
    arrs = [rs.standard_normal(s).astype(np.float32) * std
            for s in (shape_q, shape_kv, shape_kv, shape_q)]
    ts = [torch.from_numpy(a).cuda().to(dtype) for a in arrs]
    for t in ts[:3]:
        t.requires_grad_(True)
    return ts, [t.detach().float().cpu().numpy() for t in ts]


def _check(grads, want, dtype, what=""):
    for name, g, w in zip("qkv", grads, want):
        err = float(np.max(np.abs(g.detach().float().cpu().numpy().astype(np.float64) - w)))
        bound = TOL[dtype] * (1.0 + float(np.max(np.abs(w))))
        assert err <= bound, f"d{name} {what}: max-abs {err:.3g} > {bound:.3g}"


def _bhsd(a, layout):
    return a if layout == "BHSD" else np.ascontiguousarray(np.swapaxes(a, 1, 2))


def _from_bhsd(a, layout):
    return a if layout == "BHSD" else np.swapaxes(a, 1, 2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_attention_gradients(dtype, D, causal):
    import mlx_primitives as mp
    (q, k, v, do), (nq, nk, nv, ndo) = _make((2, 200, 3, D), (2, 200, 3, D), dtype, seed=D)
    out = mp.flash_attention(q, k, v, causal=causal)
    out.backward(do)
    want = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, nk, nv, ndo)), D ** -0.5,
                                causal=causal)
    _check((q.grad, k.grad, v.grad), [_from_bhsd(w, "BSHD") for w in want], dtype)


@pytest.mark.parametrize("Sq,Skv", [(100, 260), (257, 70)])
def test_bhsd_cross_lengths_bottom_right_causal(Sq, Skv):
    import mlx_primitives as mp
    (q, k, v, do), (nq, nk, nv, ndo) = _make((1, 2, Sq, 64), (1, 2, Skv, 64), torch.bfloat16, 3)
    out = mp.flash_attention(q, k, v, causal=True, layout="BHSD")
    out.backward(do)
    want = O.attention_bwd_bhsd(nq, nk, nv, ndo, 0.125, causal=True, q_offset=Skv - Sq)
    _check((q.grad, k.grad, v.grad), want, torch.bfloat16)


@pytest.mark.parametrize("causal", [True, False])
def test_sliding_window_gradients(causal):
    import mlx_primitives as mp
    W = 37
    (q, k, v, do), (nq, nk, nv, ndo) = _make((1, 300, 2, 64), (1, 300, 2, 64), torch.float32, 5)
    out = mp.sliding_window_attention(q, k, v, window_size=W, causal=causal)
    out.backward(do)
    want = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, nk, nv, ndo)), 0.125,
                                causal=causal, window_left=W, window_right=-1 if causal else W)
    _check((q.grad, k.grad, v.grad), [_from_bhsd(w, "BSHD") for w in want], torch.float32)


def test_chunked_cross_attention_gradients():
    import mlx_primitives as mp
    (q, k, v, do), (nq, nk, nv, ndo) = _make((2, 50, 2, 64), (2, 700, 2, 64), torch.bfloat16, 7)
    out = mp.chunked_cross_attention(q, k, v, chunk_size=128)
    out.backward(do)
    want = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, nk, nv, ndo)), 0.125)
    _check((q.grad, k.grad, v.grad), [_from_bhsd(w, "BSHD") for w in want], torch.bfloat16)


@pytest.mark.parametrize("H,Hkv", [(8, 2), (6, 1)])
def test_grouped_query_gradients(H, Hkv):
    from mlx_primitives.attention import gqa_attention
    (q, k, v, do), (nq, nk, nv, ndo) = _make((2, 150, H, 64), (2, 150, Hkv, 64),
                                             torch.bfloat16, H)
    out = gqa_attention(q, k, v, num_kv_groups=H // Hkv, causal=True)
    out.backward(do)
    want = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, nk, nv, ndo)), 0.125,
                                causal=True)
    _check((q.grad, k.grad, v.grad), [_from_bhsd(w, "BSHD") for w in want], torch.bfloat16)


@pytest.mark.parametrize("D", [8, 16, 48, 80])
def test_padded_head_dims_and_reference_gradient_shapes(D):
    """The reference's gradient tests use head_dim 8 and 16 at sequence 8-32 with inputs
    scaled by 0.1 (tests/gradients/test_numerical_gradients.py:27-75)."""
    import mlx_primitives as mp
    for S, causal in ((8, True), (16, False), (32, True)):
        (q, k, v, do), (nq, nk, nv, ndo) = _make((1, S, 2, D), (1, S, 2, D), torch.float32,
                                                 S + D, std=0.1)
        out = mp.flash_attention(q, k, v, causal=causal, scale=0.5 if S == 16 else None)
        out.backward(do)
        scale = 0.5 if S == 16 else D ** -0.5
        want = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, nk, nv, ndo)), scale,
                                    causal=causal)
        _check((q.grad, k.grad, v.grad), [_from_bhsd(w, "BSHD") for w in want], torch.float32,
               f"S={S}")


def test_loss_through_sum_and_broadcast_kv():
    """dO with zero strides (loss = out.sum()) and K/V broadcast over the batch by expand."""
    import mlx_primitives as mp
    (q, k, v, _), (nq, nk, nv, _) = _make((3, 64, 2, 64), (1, 64, 2, 64), torch.float32, 9)
    out = mp.flash_attention(q, k.expand(3, -1, -1, -1), v.expand(3, -1, -1, -1), causal=True)
    out.sum().backward()
    ndo = np.ones(q.shape, dtype=np.float64)
    kb, vb = np.repeat(nk, 3, axis=0), np.repeat(nv, 3, axis=0)
    dq, dk, dv = O.attention_bwd_bhsd(*(_bhsd(a, "BSHD") for a in (nq, kb, vb, ndo)), 0.125,
                                      causal=True)
    want = (_from_bhsd(dq, "BSHD"), _from_bhsd(dk, "BSHD").sum(0, keepdims=True),
            _from_bhsd(dv, "BSHD").sum(0, keepdims=True))
    _check((q.grad, k.grad, v.grad), want, torch.float32)


def _cuda_core_backward(on: bool):
    from mlx_primitives import _lib
    assert _lib.lib().mlxp_set_backward_path(1 if on else 0) == 0


def test_cuda_core_backward_is_deterministic():
    """The CUDA-core backward has one writer per output element: bit-identical reruns.  (The
    tensor-core path accumulates dQ by TMA reduce-add, whose order of additions varies.)"""
    import mlx_primitives as mp
    _cuda_core_backward(True)
    try:
        grads = []
        for _ in range(2):
            (q, k, v, do), _ = _make((1, 300, 2, 128), (1, 300, 2, 128), torch.bfloat16, 13)
            mp.flash_attention(q, k, v, causal=True).backward(do)
            grads.append([t.grad.clone() for t in (q, k, v)])
        for a, b in zip(*grads):
            assert torch.equal(a, b)
    finally:
        _cuda_core_backward(False)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", ["causal", "noncausal", "gqa", "window", "cross", "ragged"])
def test_tensor_core_backward_matches_oracle(dtype, case, D):
    """head_dim 64 and 128 in bf16/fp16 take the tensor-core kernel; every mask form, grouped
    heads, lengths that are not multiples of the 64-query / 128-key tiles."""
    from mlx_primitives.attention._core import _forward_impl, attention_backward
    B, H, Hkv, Sq, Skv, kw = 2, 4, 4, 320, 320, dict(causal=True)
    if case == "noncausal":
        kw = dict(causal=False)
    elif case == "gqa":
        Hkv = 1
    elif case == "window":
        kw = dict(causal=True, window_left=70)
    elif case == "cross":
        Sq, Skv, kw = 100, 333, dict(causal=True, q_offset=233)
    elif case == "ragged":
        Sq, Skv = 77, 201
    (q, k, v, do), (nq, nk, nv, ndo) = _make((B, H, Sq, D), (B, Hkv, Skv, D), dtype, 29 + D)
    args = dict(layout="BHSD", scale=D ** -0.5, **kw)
    with torch.no_grad():
        out, lse = _forward_impl(q, k, v, return_lse=True, **args)
        grads = attention_backward(q, k, v, out, lse, do, **args)
    want = O.attention_bwd_bhsd(nq, nk, nv, ndo, D ** -0.5, causal=kw["causal"],
                                window_left=kw.get("window_left", -1),
                                q_offset=kw.get("q_offset", 0))
    _check(grads, want, dtype, case)
    # and the CUDA-core path on the same inputs agrees with it
    _cuda_core_backward(True)
    try:
        with torch.no_grad():
            ref = attention_backward(q, k, v, out, lse, do, **args)
    finally:
        _cuda_core_backward(False)
    _check(grads, [r.float().cpu().numpy().astype(np.float64) for r in ref], dtype, case + " vs cuda cores")


def test_no_grad_path_unchanged():
    import mlx_primitives as mp
    (q, k, v, _), _ = _make((1, 128, 2, 64), (1, 128, 2, 64), torch.bfloat16, 17)
    with torch.no_grad():
        o1 = mp.flash_attention(q, k, v, causal=True)
    o2 = mp.flash_attention(q.detach(), k.detach(), v.detach(), causal=True)
    assert o1.grad_fn is None and torch.equal(o1, o2)


def _rope_t(x, cos, sin, off):
    h = x.shape[-1] // 2
    c = cos[off:off + x.shape[1]][None, :, None, :]
    s = sin[off:off + x.shape[1]][None, :, None, :]
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)


def test_fused_rope_attention_gradients():
    """RoPE (orthogonal: its gradient is the inverse rotation) then attention, against fp64
    torch autograd of the same composition."""
    from mlx_primitives.kernels import fused_rope_attention, precompute_rope_cache
    (q, k, v, do), (nq, nk, nv, ndo) = _make((1, 90, 2, 64), (1, 120, 2, 64), torch.float32, 19)
    out = fused_rope_attention(q, k, v, q_offset=30, kv_offset=0, causal=True)
    out.backward(do)
    cos, sin = (t.double().cpu() for t in precompute_rope_cache(150, 64))
    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (nq, nk, nv))
    qr, kr = _rope_t(tq, cos, sin, 30), _rope_t(tk, cos, sin, 0)
    s = torch.einsum("bqhd,bkhd->bhqk", qr, kr) * 0.125
    ok = torch.from_numpy(O.admissible(90, 120, True, q_offset=30))
    p = torch.softmax(s.masked_fill(~ok, float("-inf")), dim=-1)
    ref = torch.einsum("bhqk,bkhd->bqhd", p, tv)
    (ref * torch.tensor(ndo, dtype=torch.float64)).sum().backward()
    _check((q.grad, k.grad, v.grad), (tq.grad.numpy(), tk.grad.numpy(), tv.grad.numpy()),
           torch.float32)


def test_rope_gradient_is_inverse_rotation():
    from mlx_primitives.kernels import precompute_rope_cache, rope
    (x, _, _, g), (nx, _, _, ng) = _make((2, 40, 3, 64), (2, 40, 3, 64), torch.float32, 23)
    cos, sin = precompute_rope_cache(64, 64)
    rope(x, cos, sin, 7).backward(g)
    tx = torch.tensor(nx, dtype=torch.float64, requires_grad=True)
    _rope_t(tx, cos.double().cpu(), sin.double().cpu(), 7).backward(
        torch.tensor(ng, dtype=torch.float64))
    err = float((x.grad.double().cpu() - tx.grad).abs().max())
    assert err <= 1e-5
