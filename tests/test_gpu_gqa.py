"""Grouped-query and multi-query attention on the GPU (K/V head h // groups for query head h,
read in place by both kernels) against the oracle restatement of the reference's
gqa_attention / mqa_attention (oracle.gqa_attention, pinned to the reference's own outputs in
tests/golden).  Tolerances: fp32 <= 1e-4 max-abs; bf16 <= 2e-2 against the fp64 oracle fed the
same bf16-rounded inputs."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _inputs(shape_q, shape_kv, dtype, seed):
    q, k, v = O.make_qkv(shape_q, shape_kv, seed=seed)
    t = [torch.from_numpy(a).cuda().to(dtype) for a in (q, k, v)]
    return t, [x.float().cpu().numpy() for x in t]


def _maxabs(got, want):
    return float(np.max(np.abs(got.float().cpu().numpy().astype(np.float64) - want)))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("H,Hkv", [(8, 1), (8, 2), (8, 4), (6, 3)])
@pytest.mark.parametrize("Sq,Skv,causal", [(300, 300, True), (257, 700, True), (300, 513, False)])
def test_gqa_matches_oracle(dtype, D, H, Hkv, Sq, Skv, causal):
    from mlx_primitives.attention import gqa_attention

    (q, k, v), (nq, nk, nv) = _inputs((2, Sq, H, D), (2, Skv, Hkv, D), dtype, seed=H * 10 + Hkv)
    out = gqa_attention(q, k, v, num_kv_groups=H // Hkv, causal=causal)
    want = O.gqa_attention(nq, nk, nv, H // Hkv, causal=causal)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert _maxabs(out, want) <= TOL[dtype]


def test_gqa_bhsd_split_kv_and_lse():
    """BHSD, long keys with a forced key split (partials merged by LSE) and the LSE output."""
    from mlx_primitives.attention._core import attention_forward

    B, H, Hkv, Sq, Skv, D = 2, 8, 2, 200, 3000, 128
    (q, k, v), (nq, nk, nv) = _inputs((B, H, Sq, D), (B, Hkv, Skv, D), torch.bfloat16, seed=3)
    out, lse = attention_forward(q, k, v, layout="BHSD", scale=D ** -0.5, causal=False,
                                 kv_splits=4, return_lse=True)
    to_bshd = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3))
    want = O.gqa_attention(to_bshd(nq), to_bshd(nk), to_bshd(nv), H // Hkv, causal=False)
    assert _maxabs(out.transpose(1, 2), want) <= 2e-2
    # LSE against the dense log-sum-exp on the repeated heads
    kr = np.repeat(nk, H // Hkv, axis=1).astype(np.float64)
    s = np.einsum("bhqd,bhkd->bhqk", nq.astype(np.float64), kr) * D ** -0.5
    m = s.max(-1)
    want_lse = m + np.log(np.exp(s - m[..., None]).sum(-1))
    assert float(np.max(np.abs(lse.cpu().numpy() - want_lse))) <= 1e-2


@pytest.mark.parametrize("kv3d", [False, True])
def test_mqa_matches_oracle(kv3d):
    from mlx_primitives.attention import mqa_attention

    (q, k, v), (nq, nk, nv) = _inputs((2, 333, 6, 64), (2, 333, 1, 64), torch.bfloat16, seed=8)
    if kv3d:
        k, v, nk, nv = k[:, :, 0], v[:, :, 0], nk[:, :, 0], nv[:, :, 0]
    out = mqa_attention(q, k, v, causal=True)
    assert _maxabs(out, O.mqa_attention(nq, nk, nv, causal=True)) <= 2e-2


@pytest.mark.parametrize("cls", ["gqa", "mqa"])
def test_modules_match_projection_plus_oracle(cls):
    from mlx_primitives.attention import GroupedQueryAttention, MultiQueryAttention

    torch.manual_seed(0)
    dims, H = 256, 4
    if cls == "gqa":
        mod = GroupedQueryAttention(dims, H, num_kv_heads=2, causal=True)
        Hkv = 2
    else:
        mod = MultiQueryAttention(dims, H, causal=True)
        Hkv = 1
    mod = mod.cuda()
    x = torch.randn(2, 150, dims, device="cuda")
    out, cache = mod(x)
    hd = dims // H
    with torch.no_grad():
        qp = mod.q_proj(x).reshape(2, 150, H, hd).cpu().numpy()
        kp = mod.k_proj(x).reshape(2, 150, Hkv, hd).cpu().numpy()
        vp = mod.v_proj(x).reshape(2, 150, Hkv, hd).cpu().numpy()
        att = O.gqa_attention(qp, kp, vp, H // Hkv, causal=True).astype(np.float32)
        want = mod.out_proj(torch.from_numpy(att.reshape(2, 150, -1)).cuda())
    assert out.shape == x.shape
    assert float((out - want).abs().max().detach()) <= 1e-3
    assert cache[0].shape == (2, 150, Hkv, hd)
    # one more token against the cache: the new query attends to all 151 keys
    x1 = torch.randn(2, 1, dims, device="cuda")
    out1, cache1 = mod(x1, cache=cache)
    assert cache1[0].shape == (2, 151, Hkv, hd) and out1.shape == (2, 1, dims)
    assert torch.isfinite(out1).all()


# --------------------------------------------------------------------- custom additive masks
GOLDEN = np.load(__import__("pathlib").Path(__file__).parent / "golden" / "reference_outputs.npz")


@pytest.mark.parametrize("case", ["gqa_mask_bias_g2_d64", "gqa_mask_exclude_causal_d128",
                                  "mqa_mask_head_bias_d64"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_custom_mask_matches_reference_golden(case, dtype):
    """The reference's own gqa/mqa outputs with a custom mask (tests/golden): through the public
    API on the GPU (fp32: the CUDA-core kernel, <= 1e-4 against the golden; bf16: the
    tensor-core kernel's mask instantiation, <= 2e-2 against the oracle on the rounded inputs)."""
    from mlx_primitives.attention import gqa_attention, mqa_attention

    meta = GOLDEN[f"{case}__meta"]
    seed, std = int(meta[0]), float(meta[1])
    sq, skv = tuple(int(x) for x in meta[2:6]), tuple(int(x) for x in meta[6:10])
    (q, k, v), (nq, nk, nv) = _inputs(sq, skv, dtype, seed)
    mask = torch.from_numpy(GOLDEN[f"{case}__mask"]).cuda()
    groups = sq[2] // skv[2]
    causal = "causal" in case
    if case.startswith("mqa"):
        out = mqa_attention(q, k, v, mask=mask, causal=causal)
    else:
        out = gqa_attention(q, k, v, num_kv_groups=groups, mask=mask, causal=causal)
    want = O.gqa_attention(nq, nk, nv, groups, mask=GOLDEN[f"{case}__mask"], causal=causal)
    assert _maxabs(out, want) <= TOL[dtype]
    if dtype == torch.float32:
        assert _maxabs(out, GOLDEN[f"{case}__out"]) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("shape", ["SqSkv", "bhqk", "b1qk", "odd_keys"])
def test_custom_mask_broadcast_forms(dtype, D, shape):
    """Masks of every broadcast form, with key counts that are not multiples of 4 (rows padded
    by the wrapper) and of the 128-key tile (the partial last tile), causal and windowed by the
    kernel at the same time; -inf entries exclude keys; fully excluded rows give zeros."""
    from mlx_primitives.attention._core import attention_forward

    B, H, Hkv, Sq = 2, 4, 2, 200
    Skv = 301 if shape == "odd_keys" else 260
    (q, k, v), (nq, nk, nv) = _inputs((B, Sq, H, D), (B, Skv, Hkv, D), dtype, seed=D + Skv)
    rs = np.random.RandomState(D)
    mshape = {"SqSkv": (Sq, Skv), "bhqk": (B, H, Sq, Skv), "b1qk": (B, 1, Sq, Skv),
              "odd_keys": (1, H, Sq, Skv)}[shape]
    m = (rs.standard_normal(mshape) * 1.5).astype(np.float32)
    m[rs.rand(*mshape) < 0.2] = -np.inf
    m[..., 7, :] = -np.inf  # a row with no admissible key
    out = attention_forward(q, k, v, layout="BSHD", scale=D ** -0.5, causal=True,
                            q_offset=Skv - Sq, window_left=150, mask=torch.from_numpy(m).cuda())
    kr, vr = (np.repeat(t, H // Hkv, axis=2) for t in (nk, nv))
    want = O.from_bhsd(O.attention_bhsd(O.to_bhsd(nq, "BSHD"), O.to_bhsd(kr, "BSHD"),
                                        O.to_bhsd(vr, "BSHD"), D ** -0.5, causal=True,
                                        q_offset=Skv - Sq, window_left=150, bias=m), "BSHD")
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert _maxabs(out, want) <= tol
    assert torch.count_nonzero(out[:, 7]) == 0
