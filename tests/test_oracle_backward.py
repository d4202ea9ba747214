"""The oracle's backward (oracle.attention_bwd_bhsd, the chain rule written out) against
autodiff of the dense definition — the reference obtains its gradients by MLX autodiff through
its forward, so torch autograd in fp64 on the same function is the pin.  CPU only."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O


def _torch_ref(q, k, v, dout, scale, causal, wl, wr, qoff, kvoff):
    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    H, Hkv = q.shape[1], k.shape[1]
    kk = tk.repeat_interleave(H // Hkv, dim=1)
    vv = tv.repeat_interleave(H // Hkv, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", tq, kk) * scale
    ok = torch.from_numpy(O.admissible(q.shape[2], k.shape[2], causal, wl, wr, qoff, kvoff))
    s = s.masked_fill(~ok, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # rows with no admissible key
    o = p @ vv
    (o * torch.tensor(dout)).sum().backward()
    return tq.grad.numpy(), tk.grad.numpy(), tv.grad.numpy()


CASES = [
    # (B, H, Hkv, Sq, Skv, D, causal, wl, wr, qoff, kvoff)
    (1, 2, 2, 17, 17, 8, True, -1, -1, 0, 0),
    (2, 2, 2, 12, 20, 16, False, -1, -1, 0, 0),
    (1, 4, 2, 9, 30, 8, True, -1, -1, 21, 0),     # bottom-right causal, grouped heads
    (1, 2, 1, 25, 25, 8, True, 5, -1, 0, 0),      # sliding window
    (1, 1, 1, 16, 16, 8, False, 3, 3, 0, 0),      # bidirectional window
    (1, 2, 2, 10, 6, 8, True, -1, -1, 0, 0),      # rows without keys
]


@pytest.mark.parametrize("case", CASES)
def test_oracle_backward_matches_autodiff(case):
    B, H, Hkv, Sq, Skv, D, causal, wl, wr, qoff, kvoff = case
    rs = np.random.RandomState(sum(case[:6]))
    q = rs.standard_normal((B, H, Sq, D))
    k = rs.standard_normal((B, Hkv, Skv, D))
    v = rs.standard_normal((B, Hkv, Skv, D))
    dout = rs.standard_normal((B, H, Sq, D))
    scale = D ** -0.5
    got = O.attention_bwd_bhsd(q, k, v, dout, scale, causal, wl, wr, qoff, kvoff)
    want = _torch_ref(q, k, v, dout, scale, causal, wl, wr, qoff, kvoff)
    for g, w in zip(got, want):
        np.testing.assert_allclose(g, w, rtol=1e-10, atol=1e-10)
