"""Paged-KV attention on the GPU (mlxp_paged_attn through mlx_primitives.cache) against the
oracle restatement of the reference's paged_attention (oracle.paged_attention, pinned to the
reference's own outputs in tests/golden).  Tolerances: fp32 <= 1e-4 max-abs; bf16/fp16
<= 2e-2 against the fp64 oracle fed the same rounded inputs.  Rows with no admissible key are
zeros here (NaN in the reference)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _case(B, Sq, H, D, Hkv, bs, lens, dtype, seed, max_blocks=None, holes=0, spare=3):
    """Pools holding every sequence's blocks at shuffled ids, tables padded with -1."""
    rs = np.random.RandomState(seed)
    need = [(int(n) + bs - 1) // bs for n in lens]
    mb = max(max(need), 1) if max_blocks is None else max_blocks
    nblk = sum(need) + spare
    ids = rs.permutation(nblk)
    bt = np.full((B, mb), -1, dtype=np.int32)
    pos = 0
    for b, n in enumerate(need):
        n = min(n, mb)
        bt[b, :n] = ids[pos:pos + n]
        pos += n
    for _ in range(holes):  # missing blocks inside contexts
        b = rs.randint(B)
        if need[b] > 1:
            bt[b, rs.randint(min(need[b], mb))] = -1
    q, kp, vp = O.make_qkv((B, Sq, H, D), (nblk, bs, Hkv, D), seed=seed)
    t = [torch.from_numpy(a).cuda().to(dtype) for a in (q, kp, vp)]
    n = [x.float().cpu().numpy() for x in t]
    return t, n, bt, np.asarray(lens, dtype=np.int32)


def _oracle(nq, nk, nv, bt, ctx, **kw):
    H, Hkv = nq.shape[2], nk.shape[2]
    if Hkv != H:
        nk, nv = (np.repeat(a, H // Hkv, axis=2) for a in (nk, nv))
    return np.nan_to_num(O.paged_attention(nq, nk, nv, bt, ctx, **kw), nan=0.0)


def _maxabs(got, want):
    return float(np.max(np.abs(got.float().cpu().numpy().astype(np.float64) - want)))


def _run(t, bt, ctx, kv_splits=0, **kw):
    from mlx_primitives.cache.paged_attention import _paged_forward
    q, kp, vp = t
    slopes = kw.pop("alibi_slopes", None)
    return _paged_forward(q, kp, vp, torch.from_numpy(bt).cuda(), torch.from_numpy(ctx).cuda(),
                          kw.get("scale"), kw["block_size"], kw.get("causal", True),
                          slopes, kv_splits=kv_splits)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("bs", [16, 32])
def test_decode_matches_oracle(dtype, D, bs):
    lens = [1, 17, 300, 1000, 64, 0, 555, 2048]
    t, n, bt, ctx = _case(8, 1, 8, D, 8, bs, lens, dtype, seed=D + bs, holes=2)
    out = _run(t, bt, ctx, block_size=bs)
    assert out.shape == t[0].shape and out.dtype == dtype
    assert _maxabs(out, _oracle(*n, bt, ctx, block_size=bs)) <= TOL[dtype]


@pytest.mark.parametrize("bs", [8, 24, 48, 64, 128])
@pytest.mark.parametrize("D", [64, 128])
def test_decode_block_sizes(bs, D):
    """Block sizes a multiple of 16 take the TMA kernel (16-row boxes), others the cp.async
    kernel; both against the oracle."""
    lens = [5, 130, 777, 2000]
    t, n, bt, ctx = _case(4, 1, 4, D, 4, bs, lens, torch.bfloat16, seed=bs + D, holes=1)
    out = _run(t, bt, ctx, block_size=bs)
    assert _maxabs(out, _oracle(*n, bt, ctx, block_size=bs)) <= 2e-2


@pytest.mark.parametrize("kv_splits", [1, 2, 7, 0])
def test_decode_forced_splits(kv_splits):
    lens = [4000, 123, 2500]
    t, n, bt, ctx = _case(3, 1, 4, 128, 4, 16, lens, torch.bfloat16, seed=5)
    out = _run(t, bt, ctx, kv_splits=kv_splits, block_size=16)
    assert _maxabs(out, _oracle(*n, bt, ctx, block_size=16)) <= 2e-2


@pytest.mark.parametrize("alibi", [False, True])
def test_decode_alibi_and_scale(alibi):
    from mlx_primitives.cache import get_alibi_slopes
    H = 12
    t, n, bt, ctx = _case(4, 1, H, 64, H, 16, [700, 33, 1500, 2], torch.bfloat16, seed=9)
    slopes = get_alibi_slopes(H, device="cuda") if alibi else None
    out = _run(t, bt, ctx, block_size=16, scale=0.2, alibi_slopes=slopes)
    want = _oracle(*n, bt, ctx, block_size=16, scale=0.2,
                   alibi_slopes=O.get_alibi_slopes(H) if alibi else None)
    assert _maxabs(out, want) <= 2e-2


@pytest.mark.parametrize("H,Hkv", [(8, 2), (32, 8), (6, 1)])
def test_decode_grouped_pool_heads(H, Hkv):
    t, n, bt, ctx = _case(3, 1, H, 128, Hkv, 16, [900, 65, 1700], torch.bfloat16, seed=H)
    out = _run(t, bt, ctx, block_size=16)
    assert _maxabs(out, _oracle(*n, bt, ctx, block_size=16)) <= 2e-2


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("alibi", [False, True])
def test_prefill_matches_oracle(causal, alibi):
    H = 4
    t, n, bt, ctx = _case(2, 70, H, 64, H, 16, [150, 40], torch.bfloat16, seed=11, holes=1)
    slopes = O.get_alibi_slopes(H) if alibi else None
    out = _run(t, bt, ctx, block_size=16, causal=causal,
               alibi_slopes=torch.from_numpy(slopes).cuda() if alibi else None)
    want = _oracle(*n, bt, ctx, block_size=16, causal=causal, alibi_slopes=slopes)
    assert _maxabs(out, want) <= 2e-2


def test_out_of_range_ids_count_as_missing():
    t, n, bt, ctx = _case(2, 1, 4, 64, 4, 16, [200, 300], torch.float32, seed=21)
    nblk = t[1].shape[0]
    bt2 = bt.copy()
    bt2[0, 3] = nblk + 5
    bt2[1, 1] = 1 << 30
    out = _run(t, bt2, ctx, block_size=16)
    bt_ref = np.where(bt2 >= nblk, -1, bt2).astype(np.int32)
    assert _maxabs(out, _oracle(*n, bt_ref, ctx, block_size=16)) <= 1e-4


def test_public_api_views_host_tensors_and_errors():
    from mlx_primitives.cache import paged_attention, paged_attention_with_bias
    t, n, bt, ctx = _case(2, 1, 4, 64, 4, 16, [100, 37], torch.bfloat16, seed=31)
    q, kp, vp = t
    btc, ctxc = torch.from_numpy(bt).cuda(), torch.from_numpy(ctx).cuda()
    want = _oracle(*n, bt, ctx, block_size=16)
    assert _maxabs(paged_attention(q, kp, vp, btc, ctxc), want) <= 2e-2
    # q as a strided view (BHSD storage seen as BSHD)
    qv = q.transpose(1, 2).contiguous().transpose(1, 2)
    assert _maxabs(paged_attention(qv, kp, vp, btc, ctxc), want) <= 2e-2
    # int64 tables / lengths and host tensors
    o_host = paged_attention(q.cpu(), kp.cpu(), vp.cpu(), torch.from_numpy(bt).long(),
                             torch.from_numpy(ctx).long())
    assert o_host.device.type == "cpu" and _maxabs(o_host, want) <= 2e-2
    assert _maxabs(paged_attention_with_bias(q, kp, vp, btc, ctxc), want) <= 2e-2
    with pytest.raises(NotImplementedError):
        paged_attention_with_bias(q, kp, vp, btc, ctxc, attention_bias=torch.zeros(1))
    with pytest.raises(ValueError):
        paged_attention_with_bias(q, kp, vp, btc, ctxc, attention_bias=torch.zeros(1),
                                  alibi_slopes=torch.ones(4))
    with pytest.raises(ValueError):
        paged_attention(q, kp, vp, btc, ctxc, block_size=32)  # pool blocks hold 16
    with pytest.raises(ValueError):
        paged_attention(q.float(), kp, vp, btc, ctxc)
    q96 = torch.zeros(2, 1, 4, 96, device="cuda", dtype=torch.bfloat16)
    p96 = torch.zeros(4, 16, 4, 96, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        paged_attention(q96, p96, p96, btc[:, :2], ctxc)


def test_c_abi_direct_and_workspace_errors():
    """mlxp_paged_attn called directly: BHSD q/o strides, the workspace contract."""
    from mlx_primitives import _lib
    L = _lib.lib()
    t, n, bt, ctx = _case(2, 1, 4, 128, 4, 16, [1500, 2000], torch.bfloat16, seed=41)
    q, kp, vp = t
    qb = q.permute(0, 2, 1, 3).contiguous()                  # (B, H, 1, D)
    o = torch.empty_like(qb)
    btc, ctxc = torch.from_numpy(bt).cuda(), torch.from_numpy(ctx).cuda()
    B, H, D, nblk, mb = 2, 4, 128, kp.shape[0], bt.shape[1]
    ws_bytes = L.mlxp_paged_attn_workspace_size(1, B, H, 1, D, H, nblk, 16, mb, 8)
    assert ws_bytes > 0
    st = lambda t4: (ctypes.c_int64 * 4)(*t4.stride())
    args = lambda ws, nbytes: (
        qb.data_ptr(), kp.data_ptr(), vp.data_ptr(), btc.data_ptr(), ctxc.data_ptr(), None,
        o.data_ptr(), 1, B, H, 1, D, H, nblk, 16, mb, st(qb), st(kp), btc.stride(0), st(o),
        ctypes.c_float(D ** -0.5), 1, 8, ws, nbytes, torch.cuda.current_stream().cuda_stream)
    assert L.mlxp_paged_attn(*args(None, 0)) == _lib.MLXP_ERR_WORKSPACE
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    assert L.mlxp_paged_attn(*args(ws.data_ptr(), ws_bytes - 1)) == _lib.MLXP_ERR_WORKSPACE
    assert L.mlxp_paged_attn(*args(ws.data_ptr(), ws_bytes)) == 0, _lib.last_error()
    want = _oracle(*n, bt, ctx, block_size=16)
    assert _maxabs(o.permute(0, 2, 1, 3), want) <= 2e-2


def test_deterministic_and_large_decode():
    """The reference benchmark's largest decode shape (batch 8, 4096 cached tokens, 32 heads,
    head_dim 128, block 16), checked on sampled sequences and run twice for determinism."""
    lens = [4096] * 8
    t, n, bt, ctx = _case(8, 1, 32, 128, 32, 16, lens, torch.bfloat16, seed=51, spare=0)
    o1 = _run(t, bt, ctx, block_size=16)
    o2 = _run(t, bt, ctx, block_size=16)
    assert torch.equal(o1, o2)
    nq, nk, nv = n
    for b in (0, 5):
        ids = bt[b]  # the oracle gets only this sequence's blocks, renumbered 0..n-1
        sub_bt = np.arange(len(ids), dtype=np.int32)[None]
        want = _oracle(nq[b:b + 1], nk[ids], nv[ids], sub_bt, ctx[b:b + 1], block_size=16)
        assert _maxabs(o1[b:b + 1], want) <= 2e-2


@pytest.mark.parametrize("seed", list(range(2000, 2040)))
def test_paged_random(seed):
    """Seeded random sweep: dtype, head_dim, block size (TMA and cp.async kernels), pool head
    groups, decode and short prefill, causal, ALiBi, holes in the tables, empty and
    over-long contexts, automatic and forced splits."""
    rs = np.random.RandomState(seed)
    dtype = [torch.bfloat16, torch.float16, torch.float32][rs.randint(3)]
    D = int(rs.choice([32, 64, 128]))
    bs = int(rs.choice([8, 16, 24, 32, 64]))
    Hkv = int(rs.choice([1, 2, 4]))
    H = Hkv * int(rs.choice([1, 2, 4]))
    B = int(rs.randint(1, 5))
    Sq = int(rs.choice([1, 1, 1, 3, 17]))
    lens = [int(rs.choice([0, rs.randint(1, 40), rs.randint(40, 900)])) for _ in range(B)]
    t, n, bt, ctx = _case(B, Sq, H, D, Hkv, bs, lens, dtype, seed=seed, holes=int(rs.randint(3)))
    if rs.randint(4) == 0:  # a context longer than the table holds
        ctx = ctx + bs * bt.shape[1]
    causal = bool(rs.randint(2))
    alibi = bool(rs.randint(2))
    slopes = O.get_alibi_slopes(H) if alibi else None
    splits = int(rs.choice([0, 0, 1, 5]))
    out = _run(t, bt, ctx, kv_splits=splits, block_size=bs, causal=causal,
               alibi_slopes=torch.from_numpy(slopes).cuda() if alibi else None)
    want = _oracle(*n, bt, ctx, block_size=bs, causal=causal, alibi_slopes=slopes)
    assert _maxabs(out, want) <= TOL[dtype], (seed, dtype, D, bs, H, Hkv, B, Sq, lens)
