"""The FMA-pipe exp2 used for part of each softmax row (exp2_poly2 in csrc/sm100_ptx.cuh),
replayed step by step in numpy float32: Cody-Waite reduction with the 1.5*2^23 rounding
constant, the degree-3 Remez polynomial, and the exponent-field injection.  Its relative error
must stay within 1e-4 over the whole range the kernel feeds it (x <= 0), far below bf16's
2^-8, and it must never produce a negative, infinite or NaN value."""

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "mlx-primitives_b200" / "csrc" / "sm100_ptx.cuh"


def coefficients():
    text = SRC.read_text()
    vals = {}
    for name in ("kC0", "kC1", "kC2", "kC3"):
        m = re.search(rf"{name} = ([0-9.]+)f;\s*//\s*0x([0-9a-f]+)", text)
        vals[name] = (np.float32(float(m.group(1))), int(m.group(2), 16))
    return vals


def exp2_poly(x):
    c = coefficients()
    f32 = np.float32
    x = np.maximum(x.astype(f32), f32(-125.0))
    rnd = f32(12582912.0)
    t = (x + rnd).astype(f32)
    j = (t - rnd).astype(f32)
    f = (x - j).astype(f32)
    p = (c["kC3"][0] * f + c["kC2"][0]).astype(f32)
    p = (p * f + c["kC1"][0]).astype(f32)
    p = (p * f + c["kC0"][0]).astype(f32)
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_decimal_and_hex_coefficients_agree():
    for name, (val, hx) in coefficients().items():
        assert val.view(np.uint32) == hx, name


def test_relative_error_bound():
    x = np.concatenate([np.linspace(-124.9, 0.0, 2_000_001, dtype=np.float32),
                        np.float32(-np.arange(0, 125, 0.25))])
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1e-4, rel.max()


def test_masked_and_underflowing_inputs_are_tiny_and_finite():
    x = np.array([-np.inf, -1e30, -500.0, -126.0, -125.0], dtype=np.float32)
    y = exp2_poly(x)
    assert np.all(np.isfinite(y)) and np.all(y > 0) and np.all(y < 3e-38)
