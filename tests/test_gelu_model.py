"""The GEMM epilogue's erf-GELU, restated in numpy and checked on the CPU
against the oracle's op-by-op GELU subgraph (Div(sqrt2) -> Erf -> Add(1) ->
Mul(x) -> Mul(0.5), with the reference's Abramowitz & Stegun 7.1.26 erf,
src/operators/erf.rs:30-40).

The kernel (iconnx_b200/csrc/qgemm.cu, gelu_erf / gelu_erf2) rewrites
0.5 x (1 + erf(x / sqrt2)) as x - x Q/2 (x >= 0) or x Q/2 (x < 0), where
Q = t P(t) exp(-d^2), t = 1 / (1 + p |d|), d = x / sqrt2.  With
u = d sqrt(log2 e), exp(-d^2) = 2^(-u^2) and p |d| = (p / sqrt(log2 e)) |u|;
the 1/2 is folded into P's coefficients.  This restatement uses the kernel's
constants with exact reciprocal and exp2, so it pins the algebra and the
constants; the hardware rcp / ex2 approximations add a few ulps on top,
which the GPU tests bound (1e-5).
"""
import numpy as np

from iconnx_b200 import synth
from oracle import oracle

# the kernel's constants
K_U = 0.8493217825889587      # sqrt(log2 e) / sqrt2
K_P = 0.2727374732494354      # A&S p / sqrt(log2 e)
HALF_A = (0.5307027, -0.72657605, 0.7107069, -0.14224836, 0.1274148)  # A&S a5..a1, halved


def _gelu_model(x):
    x = x.astype(np.float64)
    u = x * K_U
    t = 1.0 / (1.0 + K_P * np.abs(u))
    e = np.exp2(-(u * u))
    p = HALF_A[0]
    for c in HALF_A[1:]:
        p = p * t + c
    hq = p * t * e
    return np.where(u >= 0.0, x - x * hq, x * hq)


def test_constants_restate_the_published_ones():
    a = (1.061405429, -1.453152027, 1.421413741, -0.284496736, 0.254829592)  # A&S a5..a1
    p = 0.3275911
    log2e = 1.0 / np.log(2.0)
    # the kernel's f32 literals are the nearest f32 values of the exact ones
    assert np.float32(K_U) == np.float32(np.sqrt(log2e) / np.sqrt(2.0))
    assert np.float32(K_P) == np.float32(p / np.sqrt(log2e))
    for h, full in zip(HALF_A, a):
        assert np.float32(h) == np.float32(0.5 * full)


def test_model_matches_oracle_gelu():
    x = np.concatenate([
        np.linspace(-12.0, 12.0, 200_001, dtype=np.float32),
        synth.normal((200_000,), 3.0, 51),
        np.array([0.0, -0.0, 1e-30, -1e-30, 40.0, -40.0], np.float32),
    ])
    ref = oracle.gelu(x).astype(np.float64)
    got = _gelu_model(x)
    # the oracle rounds every op in f32; the model is f64 with the same
    # formula, so they agree to a few f32 ulps of max(1, |x|)
    assert np.max(np.abs(got - ref) / np.maximum(1.0, np.abs(x))) < 1e-6
