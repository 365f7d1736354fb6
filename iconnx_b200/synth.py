"""Seeded synthetic inputs for the benchmark configurations.

The generator is the reference test-suite's ``seeded(n, seed)``
(tests/common/ort_parity.rs:141-170): a SplitMix64 stream feeding
Box-Muller, vectorised here with numpy.  Derived draws:

* N(0, sigma):           sigma * seeded(n, seed)
* int8 uniform [-127,127]: (splitmix64() % 255) - 127
* uniform f32 [a, b]:    a + (b - a) * unit()
* int8 uniform [-8, 8]:  (splitmix64() % 17) - 8
* outlier mix:           per element, unit() < 0.001 -> 20*N(0,1) else N(0,1)

Seeds: x=0, W=1, bias=2, W2=3, w_scale=4, b_zp=5, token ids=6; layer l adds
100*l.
"""

from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(n: int, seed: int) -> np.ndarray:
    """The first n outputs of SplitMix64 started at `seed`."""
    with np.errstate(over="ignore"):
        state = np.uint64(seed) + _GOLDEN * np.arange(1, n + 1, dtype=np.uint64)
        z = state
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def unit(n: int, seed: int) -> np.ndarray:
    """Open-interval uniforms in (0, 1], as f64."""
    bits = splitmix64(n, seed) >> np.uint64(11)
    return (bits.astype(np.float64) + 1.0) / (float(1 << 53) + 1.0)


def seeded(n: int, seed: int) -> np.ndarray:
    """n deterministic N(0,1) samples as f32 (Box-Muller on unit pairs)."""
    pairs = (n + 1) // 2
    u = unit(2 * pairs, seed)
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    ang = 2.0 * np.pi * u2
    out = np.empty(2 * pairs, dtype=np.float64)
    out[0::2] = r * np.cos(ang)
    out[1::2] = r * np.sin(ang)
    return out[:n].astype(np.float32)


def normal(shape, sigma: float, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    return (seeded(n, seed) * np.float32(sigma)).reshape(shape)


def int8_uniform(shape, seed: int, lo: int = -127, hi: int = 127) -> np.ndarray:
    n = int(np.prod(shape))
    span = np.uint64(hi - lo + 1)
    return ((splitmix64(n, seed) % span).astype(np.int64) + lo).astype(np.int8).reshape(shape)


def uniform_f32(shape, lo: float, hi: float, seed: int) -> np.ndarray:
    n = int(np.prod(shape))
    return (lo + (hi - lo) * unit(n, seed)).astype(np.float32).reshape(shape)


def outlier_mix(shape, seed: int) -> np.ndarray:
    """99.9% N(0,1), 0.1% N(0,20)."""
    n = int(np.prod(shape))
    base = seeded(n, seed)
    pick = unit(n, seed + 7919) < 0.001
    base[pick] *= np.float32(20.0)
    return base.reshape(shape)


def token_ids(shape, seed: int, vocab: int = 30522) -> np.ndarray:
    n = int(np.prod(shape))
    return (splitmix64(n, seed) % np.uint64(vocab)).astype(np.int64).reshape(shape)
