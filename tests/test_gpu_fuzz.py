"""Seeded random sweep of the attention entry points on the GPU against the oracle: shapes that
are not multiples of any tile, both layouts, grouped heads, every mask form with position
offsets, explicit key splits, forward and backward.  Each case is small enough for the fp64
oracle; the seed list is fixed so a failure reproduces.  Tolerances as everywhere: fp32
<= 1e-4, bf16/fp16 <= 2e-2 max-abs (gradients: relative to 1 + max |grad|)."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _case(seed):
    rs = np.random.RandomState(seed)
    dtype = [torch.bfloat16, torch.float16, torch.float32][rs.randint(3)]
    D = int(rs.choice([64, 128] if dtype != torch.float32 else [32, 64, 128]))
    B = int(rs.randint(1, 3))
    Hkv = int(rs.choice([1, 2, 3]))
    H = Hkv * int(rs.choice([1, 2, 4]))
    Sq = int(rs.randint(1, 400))
    Skv = int(rs.randint(1, 600))
    layout = ["BSHD", "BHSD"][rs.randint(2)]
    causal = bool(rs.randint(2))
    wl = int(rs.choice([-1, -1, rs.randint(0, 300)]))
    wr = -1 if causal else int(rs.choice([-1, -1, rs.randint(0, 300)]))
    q_off = int(rs.randint(-50, 300))
    kv_off = int(rs.randint(0, 100))
    splits = int(rs.choice([0, 1, 1, 3]))
    return dict(seed=seed, dtype=dtype, D=D, B=B, H=H, Hkv=Hkv, Sq=Sq, Skv=Skv, layout=layout,
                causal=causal, wl=wl, wr=wr, q_off=q_off, kv_off=kv_off, splits=splits)


def _tensors(c):
    shape_q = (c["B"], c["H"], c["Sq"], c["D"])
    shape_kv = (c["B"], c["Hkv"], c["Skv"], c["D"])
    q, k, v = O.make_qkv(shape_q, shape_kv, seed=c["seed"])
    do = O.make_qkv(shape_q, (1, 1, 1, 1), seed=c["seed"] + 7)[0]
    ts = [torch.from_numpy(a).cuda().to(c["dtype"]) for a in (q, k, v, do)]
    ns = [t.float().cpu().numpy().astype(np.float64) for t in ts]
    if c["layout"] == "BSHD":  # same values, other memory order
        ts = [t.transpose(1, 2).contiguous() for t in ts]
    return ts, ns


def _bhsd(t, layout):
    return t if layout == "BHSD" else t.transpose(1, 2)


TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


@pytest.mark.parametrize("seed", list(range(1000, 1120)))
def test_forward_and_backward_random(seed):
    from mlx_primitives.attention._core import _forward_impl, attention_backward
    c = _case(seed)
    (q, k, v, do), (nq, nk, nv, ndo) = _tensors(c)
    kw = dict(layout=c["layout"], scale=c["D"] ** -0.5, causal=c["causal"],
              window_left=c["wl"], window_right=c["wr"], q_offset=c["q_off"],
              kv_offset=c["kv_off"])
    with torch.no_grad():
        out, lse = _forward_impl(q, k, v, return_lse=True, kv_splits=c["splits"], **kw)
    g = c["H"] // c["Hkv"]
    kr, vr = np.repeat(nk, g, axis=1), np.repeat(nv, g, axis=1)
    want, want_lse = O.attention_bhsd(nq, kr, vr, c["D"] ** -0.5, causal=c["causal"],
                                      window_left=c["wl"], window_right=c["wr"],
                                      q_offset=c["q_off"], kv_offset=c["kv_off"],
                                      return_lse=True)
    got = _bhsd(out, c["layout"]).float().cpu().numpy()
    err = float(np.abs(got - want).max()) if want.size else 0.0
    assert err <= TOL[c["dtype"]], (c, err)
    fin = np.isfinite(want_lse)
    got_lse = lse.cpu().numpy()
    assert np.all(np.isneginf(got_lse[~fin])), c
    if fin.any():
        assert float(np.abs(got_lse[fin] - want_lse[fin]).max()) <= 1e-2, c
    if c["dtype"] == torch.float16 or c["Skv"] == 0:
        return
    with torch.no_grad():
        grads = attention_backward(q, k, v, out, lse, do, **kw)
    wants = O.attention_bwd_bhsd(nq, nk, nv, ndo, c["D"] ** -0.5, causal=c["causal"],
                                 window_left=c["wl"], window_right=c["wr"],
                                 q_offset=c["q_off"], kv_offset=c["kv_off"])
    for name, gt, w in zip("qkv", grads, wants):
        gt = _bhsd(gt, c["layout"]).float().cpu().numpy()
        e = float(np.abs(gt - w).max())
        assert e <= TOL[c["dtype"]] * (1.0 + float(np.abs(w).max())), (name, c, e)
