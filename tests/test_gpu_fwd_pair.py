"""The CTA-pair forward (head_dim 128, 2-SM MMAs; opt-in through mlxp_set_forward_kernel(1))
against the fp64 oracle and against the default single-SM kernel: a seeded sweep over layouts,
grouped heads, mask forms with offsets, ragged lengths (rows of a pair past the end of the
sequence, key tiles past the end of K/V), key splits (fp32 partials + merge) and both 16-bit
dtypes.  Tolerances as everywhere: <= 2e-2 max-abs against fp64 for bf16/fp16, LSE <= 1e-2."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture
def pair_kernel():
    from mlx_primitives import _lib
    lib = _lib.lib()
    assert lib.mlxp_set_forward_kernel(1) == 0
    try:
        yield lib
    finally:
        lib.mlxp_set_forward_kernel(0)


def _status(lib):
    st = ctypes.c_int(0)
    assert lib.mlxp_device_status(ctypes.byref(st), 1) == 0
    return st.value


def _case(seed):
    rs = np.random.RandomState(seed)
    dtype = [torch.bfloat16, torch.float16][rs.randint(2)]
    B = int(rs.randint(1, 3))
    Hkv = int(rs.choice([1, 2, 3]))
    H = Hkv * int(rs.choice([1, 2, 4]))
    Sq = int(rs.randint(1, 700))
    Skv = int(rs.randint(1, 900))
    layout = ["BSHD", "BHSD"][rs.randint(2)]
    causal = bool(rs.randint(2))
    wl = int(rs.choice([-1, -1, rs.randint(0, 400)]))
    wr = -1 if causal else int(rs.choice([-1, -1, rs.randint(0, 400)]))
    q_off = int(rs.randint(-50, 400))
    kv_off = int(rs.randint(0, 100))
    splits = int(rs.choice([0, 1, 1, 2, 4]))
    return dict(dtype=dtype, B=B, H=H, Hkv=Hkv, Sq=Sq, Skv=Skv, layout=layout, causal=causal,
                wl=wl, wr=wr, q_off=q_off, kv_off=kv_off, splits=splits, seed=seed)


@pytest.mark.parametrize("seed", list(range(2000, 2040)))
def test_pair_kernel_random(pair_kernel, seed):
    from mlx_primitives.attention._core import _forward_impl
    c = _case(seed)
    D = 128
    q, k, v = O.make_qkv((c["B"], c["H"], c["Sq"], D), (c["B"], c["Hkv"], c["Skv"], D),
                         seed=seed)
    ts = [torch.from_numpy(a).cuda().to(c["dtype"]) for a in (q, k, v)]
    ns = [t.float().cpu().numpy().astype(np.float64) for t in ts]
    if c["layout"] == "BSHD":
        ts = [t.transpose(1, 2).contiguous() for t in ts]
    kw = dict(layout=c["layout"], scale=D ** -0.5, causal=c["causal"], window_left=c["wl"],
              window_right=c["wr"], q_offset=c["q_off"], kv_offset=c["kv_off"])
    with torch.no_grad():
        out, lse = _forward_impl(*ts, return_lse=True, kv_splits=c["splits"], **kw)
        torch.cuda.synchronize()
        assert _status(pair_kernel) == 0, c
        pair_kernel.mlxp_set_forward_kernel(0)
        ref_out = _forward_impl(*ts, kv_splits=c["splits"], **kw)
        pair_kernel.mlxp_set_forward_kernel(1)
    g = c["H"] // c["Hkv"]
    want, want_lse = O.attention_bhsd(ns[0], np.repeat(ns[1], g, axis=1),
                                      np.repeat(ns[2], g, axis=1), D ** -0.5,
                                      causal=c["causal"], window_left=c["wl"],
                                      window_right=c["wr"], q_offset=c["q_off"],
                                      kv_offset=c["kv_off"], return_lse=True)
    got = (out if c["layout"] == "BHSD" else out.transpose(1, 2)).float().cpu().numpy()
    err = float(np.abs(got - want).max()) if want.size else 0.0
    assert err <= 2e-2, (c, err)
    # the two tensor-core kernels differ only in the order of fp32 additions
    diff = float((out.float() - ref_out.float()).abs().max()) if out.numel() else 0.0
    assert diff <= 2e-2, (c, diff)
    fin = np.isfinite(want_lse)
    got_lse = lse.cpu().numpy()
    assert np.all(np.isneginf(got_lse[~fin])), c
    if fin.any():
        assert float(np.abs(got_lse[fin] - want_lse[fin]).max()) <= 1e-2, c


def test_pair_kernel_flash_api(pair_kernel):
    """The public flash_attention entry point routes through the pair kernel when selected."""
    import mlx_primitives as mp
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 4, 1000, 128, device="cuda", dtype=torch.bfloat16)
               for _ in range(3))
    out = mp.flash_attention(q, k, v, causal=True, layout="BHSD")
    torch.cuda.synchronize()
    assert _status(pair_kernel) == 0
    pair_kernel.mlxp_set_forward_kernel(0)
    ref = mp.flash_attention(q, k, v, causal=True, layout="BHSD")
    assert float((out.float() - ref.float()).abs().max()) <= 2e-2
