"""GPU parity at BASELINE.json's full sizes.  A full CPU oracle of every config is out of reach
(up to 140 TFLOP), so each test checks (a) sampled query rows of EVERY (batch, head) unit —
including the first and last rows, tile and window boundaries — against the exact fp64 row
oracle on the same bf16 inputs, (b) whole heads of configs 2 and 3 (every row, computed by the
oracle in row blocks over each block's admissible keys), and (c) size-independent properties:
layout invariance (BSHD and BHSD views give bit-identical results), determinism, split
invariance and finiteness.  Tolerance: 2e-2 max-abs (bf16)."""

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


def sample_rows(S, extra=(), n_random=12, seed=0):
    rng = np.random.RandomState(seed)
    rows = {0, 1, 127, 128, 255, 256, S // 2, S - 257, S - 256, S - 129, S - 128, S - 1, *extra}
    rows |= set(rng.randint(0, S, n_random).tolist())
    return np.array(sorted(r for r in rows if 0 <= r < S))


def all_units(B, H):
    return [(b, h) for b in range(B) for h in range(H)]


def check_whole_heads(o_bhsd, q, k, v, pairs, scale, window_left=-1, block=512):
    """Every row of the given (b, h) units against the fp64 oracle, a row block at a time over
    the block's admissible (causal, optionally windowed) keys."""
    S = q.shape[2]
    for b, h in pairs:
        qn, kn, vn = (t[b, h].float().cpu().numpy()[None, None] for t in (q, k, v))
        got_all = o_bhsd[b, h].float().cpu().numpy()
        for r0 in range(0, S, block):
            r1 = min(S, r0 + block)
            lo = max(0, r0 - window_left) if window_left >= 0 else 0
            want = O.attention_rows_bhsd(qn, kn[:, :, lo:r1], vn[:, :, lo:r1],
                                         np.arange(r0, r1), scale, causal=True,
                                         window_left=window_left, kv_offset=lo)[0]
            err = np.abs(got_all[r0:r1] - want).max()
            assert err <= TOL, f"(b={b}, h={h}) rows [{r0}, {r1}): max-abs {err}"


def check_rows(o_bhsd, q, k, v, pairs, rows, scale, **mask):
    for b, h in pairs:
        qn = q[b, h].float().cpu().numpy()[None, None]
        kn = k[b, h].float().cpu().numpy()[None, None]
        vn = v[b, h].float().cpu().numpy()[None, None]
        want = O.attention_rows_bhsd(qn, kn, vn, rows, scale, **mask)[0]
        got = o_bhsd[b, h, torch.as_tensor(rows, device=o_bhsd.device)].float().cpu().numpy()
        err = np.max(np.abs(got - want))
        assert err <= TOL, f"(b={b}, h={h}) max-abs {err}"


def test_config2_flash_bhsd_causal_4x32x4096x128():
    import mlx_primitives as mp
    B, H, S, D = 4, 32, 4096, 128
    q, k, v = (seeded((B, H, S, D), 42 + i) for i in range(3))
    o = mp.flash_attention(q, k, v, causal=True, layout="BHSD")
    assert torch.isfinite(o.float()).all()
    check_rows(o, q, k, v, all_units(B, H), sample_rows(S), D ** -0.5, causal=True)
    check_whole_heads(o, q, k, v, [(0, 0), (1, 17), (2, 5), (3, 31)], D ** -0.5)
    # determinism and layout invariance
    assert torch.equal(o, mp.flash_attention(q, k, v, causal=True, layout="BHSD"))
    t = lambda x: x.transpose(1, 2)  # BSHD view of the same storage
    o_bshd = mp.flash_attention(t(q), t(k), t(v), causal=True, layout="BSHD")
    assert torch.equal(t(o_bshd), o)
    qc, kc, vc = (t(x).contiguous() for x in (q, k, v))  # genuinely BSHD-contiguous copies
    assert torch.equal(t(mp.flash_attention(qc, kc, vc, causal=True)), o)


def test_config3_sliding_window_bshd_2x16384x32x128_w4096():
    import mlx_primitives as mp
    B, S, H, D, W = 2, 16384, 32, 128, 4096
    q, k, v = (seeded((B, S, H, D), 142 + i) for i in range(3))
    o = mp.SlidingWindowAttention(num_heads=H, head_dim=D, window_size=W, causal=True)(q, k, v)
    assert torch.isfinite(o.float()).all()
    t = lambda x: x.transpose(1, 2)
    rows = sample_rows(S, extra=(W - 1, W, W + 1, 8191, 8192, 12288))
    check_rows(t(o), t(q), t(k), t(v), all_units(B, H), rows, D ** -0.5, causal=True,
               window_left=W)
    check_whole_heads(t(o), t(q), t(k), t(v), [(0, 0), (0, 21), (1, 9), (1, 31)], D ** -0.5,
                      window_left=W)
    # rows whose window does not bind equal plain causal attention
    o_causal = mp.flash_attention(q[:, :W], k[:, :W], v[:, :W], causal=True)
    assert (o[:, :W].float() - o_causal.float()).abs().max().item() <= 1e-2


def test_config4_chunked_cross_8x512_65536_16x64():
    import mlx_primitives as mp
    B, Sq, Skv, H, D = 8, 512, 65536, 16, 64
    q = seeded((B, Sq, H, D), 242, std=0.5)
    k = seeded((B, Skv, H, D), 243, std=0.5)
    v = seeded((B, Skv, H, D), 244, std=0.5)
    o = mp.ChunkedCrossAttention(num_heads=H, head_dim=D, chunk_size=4096)(q, k, v)
    assert torch.isfinite(o.float()).all()
    t = lambda x: x.transpose(1, 2)
    check_rows(t(o), t(q), t(k), t(v), all_units(B, H), sample_rows(Sq), D ** -0.5, causal=False)
    # split invariance: one CTA per query block over the whole key range vs the split-KV path
    from mlx_primitives.attention._core import attention_forward
    o1 = attention_forward(q, k, v, layout="BSHD", scale=D ** -0.5, causal=False, kv_splits=1)
    assert (o1.float() - o.float()).abs().max().item() <= TOL


def test_config5_long_context_single_gpu_1x32x131072x128():
    import mlx_primitives as mp
    B, H, S, D = 1, 32, 131072, 128
    q, k, v = (seeded((B, H, S, D), 342 + i) for i in range(3))
    o = mp.flash_attention(q, k, v, causal=True, layout="BHSD")
    assert torch.isfinite(o.float()).all()
    rows = sample_rows(S, extra=(8191, 8192, 16383, 16384, 65535, 65536), n_random=8)
    check_rows(o, q, k, v, all_units(B, H), rows, D ** -0.5, causal=True)
