"""The quantise pass's f32 fast path, restated in numpy and checked against
the oracle's DynamicQuantizeLinear (src/operators/dynamic_quantize_linear.rs:
32-112) on the CPU.

The GPU kernel (iconnx_b200/csrc/dql.cu, quant4) rounds
u = fma(x, f32(1/scale), zp) to the nearest integer and clamps it, except
for elements whose u lies within 1e-4 of a half-integer, which take an f64
division.  The claim that makes this bit-exact is |u - (x/scale + zp)| <
4.6e-5: outside the band, rounding u and rounding the reference's f64
quotient give the same integer.  These tests exercise that claim directly:
every element the model sends down the fast path must equal the oracle,
including elements built to sit just outside and inside the band.

The fma is modelled as the f64 value of x * inv32 + zp rounded once to f32:
the 48-bit product is exact in f64, and so is the sum whenever the product
is not far below 2^-45 (for such tiny products u is the integer zp either
way).
"""
import numpy as np
import pytest

from iconnx_b200 import synth
from oracle import oracle


def _params(x):
    """Scale / zero point as the kernel's dql_params (min, max seeded with 0)."""
    fin = x[~np.isnan(x)]
    mn = float(min(0.0, fin.min())) if fin.size else 0.0
    mx = float(max(0.0, fin.max())) if fin.size else 0.0
    scale = (mx - mn) / 255.0
    zp = min(255.0, max(0.0, float(np.rint(0.0 - mn / scale))))
    inv32 = np.float32(1.0 / scale)
    return scale, np.float32(zp), inv32


def _fast_path(x):
    """(q, near) of the vector path: q is what the fast path would write,
    near marks the elements that take the exact f64 division instead."""
    _, zpf, inv32 = _params(x)
    u = (x.astype(np.float64) * np.float64(inv32) + np.float64(zpf)).astype(np.float32)
    r = np.rint(u)
    near = np.abs(np.abs(u - r) - np.float32(0.5)) <= np.float32(1e-4)
    q = np.clip(r, 0.0, 255.0)
    q = np.where(np.isnan(q), 0.0, q).astype(np.uint8)
    return q, near


@pytest.mark.parametrize("make", [
    lambda: synth.normal((1 << 21,), 1.0, 31),
    lambda: synth.outlier_mix((1 << 21,), 32),
    lambda: synth.uniform_f32((1 << 21,), -3.0, 7.0, 33),
    lambda: synth.uniform_f32((1 << 21,), 0.0, 5.0, 34),    # min = 0: zero point 0
    lambda: synth.uniform_f32((1 << 21,), -9.0, -1.0, 35),  # max = 0: zero point 255
])
def test_fast_path_equals_oracle(make):
    x = make()
    q, near = _fast_path(x)
    y, _, _ = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(q[~near], y[~near])
    assert near.mean() < 1e-3  # the f64 path stays rare


def test_fast_path_at_the_band_edge():
    """Elements placed at half-integer quotients offset by -3e-4 .. +3e-4, on
    both sides of the 1e-4 band: every one the fast path keeps is exact,
    every exact tie is sent to the f64 path."""
    scale = 6.0 / 255.0
    rng = np.random.default_rng(36)
    # min -2, max 4: zero point 85, u = x / scale + 85 = k + 0.5 + delta
    k = rng.integers(0, 254, size=200_000).astype(np.float64)
    delta = rng.uniform(-3e-4, 3e-4, size=k.size)
    body = ((k + 0.5 + delta) * scale - 2.0).astype(np.float32)
    ties = ((np.arange(-80, 160) + 0.5) * scale).astype(np.float32)
    x = np.concatenate([np.array([-2.0, 4.0], np.float32), body, ties])
    x = np.clip(x, np.float32(-2.0), np.float32(4.0))  # keep min / max (and the scale) fixed
    q, near = _fast_path(x)
    y, s, _ = oracle.dynamic_quantize_linear(x)
    assert s == np.float32(scale)
    np.testing.assert_array_equal(q[~near], y[~near])
    # both sides of the band are populated: about a third of the body is near
    body_near = near[2:2 + k.size]
    assert 0.2 < body_near.mean() < 0.5
    assert (~body_near & (np.abs(delta) < 1.5e-4)).any()
    # exact ties of the f64 quotient must not be decided by the fast path
    _, zpf, _ = _params(x)
    qexact = x.astype(np.float64) / scale + float(zpf)
    tie = np.abs(qexact - np.floor(qexact) - 0.5) < 1e-9
    assert tie.any() and near[tie].all()
