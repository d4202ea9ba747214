"""The (batch, head) split of one call across ranks (mlx_primitives.attention.partition) on one
GPU: every rank's share is run in turn into one output, which must equal the whole call — bit
for bit where the launch has no key splits (each unit's rows are computed by the same kernel
code whatever other units share the launch), within the bf16 tolerance (2e-2 max-abs) where
the split-KV heuristic picks a different split count for a smaller launch — and sampled rows
of every unit must match the fp64 oracle."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-2


def seeded(shape, seed, std=1.0, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * std).to(dtype)


def all_ranks(fn, world, q):
    out = torch.full(q.shape, float("nan"), dtype=q.dtype, device=q.device)
    for r in range(world):
        fn(r, out)
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any(), "a unit was not computed by any rank"
    return out


def rows_vs_oracle(o_bhsd, q, k, v, rows, scale, group=1, **mask):
    B, H = q.shape[:2]
    for b in range(B):
        for h in range(H):
            kh = h // group
            want = O.attention_rows_bhsd(q[b:b + 1, h:h + 1].float().cpu().numpy(),
                                         k[b:b + 1, kh:kh + 1].float().cpu().numpy(),
                                         v[b:b + 1, kh:kh + 1].float().cpu().numpy(),
                                         rows, scale, **mask)[0]
            got = o_bhsd[b, h, torch.as_tensor(rows, device=o_bhsd.device)].float().cpu().numpy()
            err = np.abs(got - want).max()
            assert err <= TOL, f"(b={b}, h={h}) max-abs {err}"


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("layout", ["BHSD", "BSHD"])
def test_flash_shards_reassemble_the_whole_call(world, layout):
    import mlx_primitives as mp
    from mlx_primitives.attention import flash_attention_shard

    B, H, S, D = 2, 12, 1280, 128
    q, k, v = (seeded((B, H, S, D), 900 + i) for i in range(3))
    if layout == "BSHD":
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    whole = mp.flash_attention(q, k, v, causal=True, layout=layout)
    got = all_ranks(lambda r, out: flash_attention_shard(q, k, v, world, r, causal=True,
                                                         layout=layout, out=out), world, q)
    assert torch.equal(got, whole)
    bhsd = (lambda t: t) if layout == "BHSD" else (lambda t: t.transpose(1, 2))
    rows = np.array([0, 1, 127, 128, 255, 256, 640, 1023, 1024, S - 1])
    rows_vs_oracle(bhsd(got), bhsd(q), bhsd(k), bhsd(v), rows, D ** -0.5, causal=True)


def test_sliding_window_shards_reassemble_the_whole_call():
    import mlx_primitives as mp
    from mlx_primitives.attention import sliding_window_attention_shard

    B, S, H, D, W = 2, 2048, 6, 64, 300
    q, k, v = (seeded((B, S, H, D), 910 + i) for i in range(3))
    whole = mp.sliding_window_attention(q, k, v, window_size=W, causal=True)
    got = all_ranks(lambda r, out: sliding_window_attention_shard(q, k, v, W, 4, r, out=out), 4, q)
    assert torch.equal(got, whole)
    t = lambda x: x.transpose(1, 2)
    rows_vs_oracle(t(got), t(q), t(k), t(v), np.array([0, 299, 300, 301, 1024, S - 1]),
                   D ** -0.5, causal=True, window_left=W)


def test_chunked_shards_match_the_whole_call_and_the_oracle():
    import mlx_primitives as mp
    from mlx_primitives.attention import chunked_cross_attention_shard

    B, Sq, Skv, H, D = 4, 256, 8192, 4, 64
    q = seeded((B, Sq, H, D), 920, std=0.5)
    k = seeded((B, Skv, H, D), 921, std=0.5)
    v = seeded((B, Skv, H, D), 922, std=0.5)
    whole = mp.chunked_cross_attention(q, k, v, chunk_size=4096)
    got = all_ranks(lambda r, out: chunked_cross_attention_shard(q, k, v, 8, r, out=out), 8, q)
    assert (got.float() - whole.float()).abs().max().item() <= TOL
    t = lambda x: x.transpose(1, 2)
    rows_vs_oracle(t(got), t(q), t(k), t(v), np.array([0, 1, 127, 128, Sq - 1]), D ** -0.5,
                   causal=False)


@pytest.mark.parametrize("world", [3, 5])
def test_grouped_heads_split_mid_group(world):
    """Rank ranges that start and end inside a K/V head group (6 query heads per K/V head)."""
    from mlx_primitives.attention import attention_units, gqa_attention, shard_units

    B, S, H, Hkv, D = 2, 512, 12, 2, 128
    q = seeded((B, S, H, D), 930)
    k, v = (seeded((B, S, Hkv, D), 931 + i) for i in range(2))
    whole = gqa_attention(q, k, v, num_kv_groups=H // Hkv, causal=True)
    got = all_ranks(lambda r, out: attention_units(q, k, v, shard_units(B, H, world, r),
                                                   layout="BSHD", scale=D ** -0.5, causal=True,
                                                   out=out), world, q)
    assert torch.equal(got, whole)
    t = lambda x: x.transpose(1, 2)
    rows_vs_oracle(t(got), t(q), t(k), t(v), np.array([0, 255, 256, S - 1]), D ** -0.5,
                   group=H // Hkv, causal=True)


def test_fp32_config1_split_over_8_ranks():
    """Config 1 (fp32, BSHD, 24 units) over 8 ranks: 3 units each, some ranks straddling a
    batch boundary (two pieces)."""
    import mlx_primitives as mp
    from mlx_primitives.attention import flash_attention_shard

    B, S, H, D = 2, 1024, 12, 64
    q, k, v = (seeded((B, S, H, D), 940 + i, dtype=torch.float32) for i in range(3))
    whole = mp.flash_attention(q, k, v, causal=True)
    got = all_ranks(lambda r, out: flash_attention_shard(q, k, v, 8, r, out=out), 8, q)
    assert (got - whole).abs().max().item() <= 1e-5
    t = lambda x: x.transpose(1, 2)
    want = O.attention_bhsd(t(q).double().cpu().numpy(), t(k).double().cpu().numpy(),
                            t(v).double().cpu().numpy(), D ** -0.5, causal=True)
    assert np.abs(t(got).cpu().numpy() - want).max() <= 1e-4
