"""The attention kernel's exact-integer QK^T, restated in numpy and checked on
the CPU against float64 (iconnx_b200/csrc/attention.cu: slice_row_store and
the score combine of attention_tc_kernel).

Each Q / K row (64 values, max magnitude m with biased exponent E) is scaled
by 2^(25-n), n = max(-101, E - 132), and rounded to an integer T with
|T| < 2^31.  T's four bytes are the int8 slices (the most significant one
signed).  The kernel accumulates the ten slice products with i + j <= 3, one
s32 tensor-memory level per i + j, then combines the levels in fp32 as
(((acc3 / 2^24 + acc2 / 2^16) + acc1 / 2^8) + acc0) and multiplies by
2^(nq-1) 2^(nk-1).  Two facts make that exact enough:
  * every level stays below 2^24 in magnitude, so its s32 -> f32
    conversion is exact;
  * the combined score is within 2^-20 max|q| max|k| + 4 2^-24 |q|.|k| of
    the float64 dot product: for rows without outliers a few 2^-24 of
    |q|.|k|, tighter than an fp32 dot product of the same rows.
"""
import numpy as np
import pytest


def _slices(v):
    """Rows v [R, 64] f32 -> (four slices [R, 64] int64, most significant
    first, and the per-row exponent n)."""
    m = np.abs(v).max(axis=1).astype(np.float32)
    e = ((m.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    n = np.maximum(-101, e - 132)
    sc = np.ldexp(np.float32(1.0), 25 - n).astype(np.float32)
    t = np.rint((v * sc[:, None]).astype(np.float32)).astype(np.int64)
    assert np.abs(t).max(initial=0) < 2 ** 31
    u = t & 0xFFFFFFFF
    b3 = (u >> 24) & 0xFF
    b3 = np.where(b3 >= 128, b3 - 256, b3)
    return [b3, (u >> 16) & 0xFF, (u >> 8) & 0xFF, u & 0xFF], n


def _f32(a):
    return np.asarray(a, np.float64).astype(np.float32)


def _scores(q, k):
    """(scores [Rq, Rk] f32, the four s32 levels) as the kernel computes them."""
    sq, nq = _slices(q)
    sk, nk = _slices(k)
    acc = [sum(sq[i] @ sk[lvl - i].T for i in range(lvl + 1)) for lvl in range(4)]
    # fp32 combine, one rounding per step (the f64 sums are exact here)
    f = _f32(acc[3] * 2.0 ** -24)
    f = _f32(acc[2] * 2.0 ** -16 + f)
    f = _f32(acc[1] * 2.0 ** -8 + f)
    f = _f32(acc[0] + f.astype(np.float64))
    pq = np.ldexp(np.float32(1.0), nq - 1).astype(np.float32)
    pk = np.ldexp(np.float32(1.0), nk - 1).astype(np.float32)
    return (f * pq[:, None]).astype(np.float32) * pk[None, :], acc


def test_levels_fit_f32_exactly():
    """The worst case by bytes (64 products per term, |signed byte| <= 128,
    |unsigned byte| <= 255) stays below 2^24, and so do rows at the extremes
    of the integer range."""
    hi, lo = 128, 255
    for lvl in range(4):
        terms = [(hi if i == 0 else lo) * (hi if lvl - i == 0 else lo) for i in range(lvl + 1)]
        assert 64 * sum(terms) < 2 ** 24
    # rows at the largest integer magnitude, 2^31 - 128 (bytes 7f ff ff 80,
    # the largest f32 below 2^31), of both signs and alternating signs, and
    # rows of random 24-bit integers spread over the full range
    big = np.float32(2.0 ** 31 - 128)
    rng = np.random.default_rng(40)
    rows = [np.full(64, big, np.float32), np.full(64, -big, np.float32),
            big * np.where(np.arange(64) % 2, -1, 1).astype(np.float32)]
    for _ in range(8):
        rows.append((rng.integers(-(2 ** 23), 2 ** 23, 64) * 2.0 ** 8).astype(np.float32))
    r = np.stack(rows)
    _, acc = _scores(r, r)
    assert max(int(np.abs(a).max()) for a in acc) < 2 ** 24


@pytest.mark.parametrize("scale", [1.0, 12.0, 1e-3, 1e3, 1e-15])
def test_scores_within_a_few_ulps_of_float64(scale):
    """Rows without outliers (plus a zero row and a row 10^6 smaller): within
    4 units of 2^-24 |q|.|k| of float64, and no worse than numpy's fp32 dot
    product of the same rows."""
    rng = np.random.default_rng(int(abs(np.log10(scale))) + 7)
    q = (rng.standard_normal((128, 64)) * scale).astype(np.float32)
    k = (rng.standard_normal((192, 64)) * scale).astype(np.float32)
    q[0, :] = 0.0
    k[2, :] *= np.float32(1e-6)
    s, _ = _scores(q, k)
    qd, kd = q.astype(np.float64), k.astype(np.float64)
    exact = qd @ kd.T
    mag = np.abs(qd) @ np.abs(kd).T
    err = np.abs(s.astype(np.float64) - exact)
    ok = mag > 0
    assert np.all(err[~ok] == 0.0)
    assert (err[ok] / mag[ok]).max() < 4 * 2.0 ** -24
    e32 = np.abs((q @ k.T).astype(np.float64) - exact)
    assert err.max() <= max(e32.max(), 4 * 2.0 ** -24 * mag.max())


def test_scores_with_outlier_rows_bounded_by_row_maxima():
    """A row whose largest element dwarfs the others keeps the others'
    significant bits in its low slices, whose cross products (i + j >= 4)
    are not computed: the error is bounded by the row maxima,
    2^-20 max|q| max|k| + 4 2^-24 |q|.|k|, rather than by |q|.|k| alone."""
    rng = np.random.default_rng(41)
    for _ in range(20):
        q = rng.standard_normal((64, 64)).astype(np.float32)
        k = rng.standard_normal((96, 64)).astype(np.float32)
        f = np.float32(10.0 ** rng.uniform(0, 5))
        q[::3, rng.integers(64)] *= f
        k[::5, rng.integers(64)] *= f
        s, _ = _scores(q, k)
        qd, kd = q.astype(np.float64), k.astype(np.float64)
        err = np.abs(s.astype(np.float64) - qd @ kd.T)
        bound = (2.0 ** -20 * np.outer(np.abs(qd).max(1), np.abs(kd).max(1))
                 + 4 * 2.0 ** -24 * (np.abs(qd) @ np.abs(kd).T))
        assert np.all(err <= bound)
