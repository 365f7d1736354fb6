"""Integer algebra of the fused GEMM, restated in numpy and checked on the CPU
against the oracle's MatMulInteger (src/operators/matmul_integer.rs:239-267).

The tensor cores compute acc = sum_k a*b on the raw operands; the epilogue
of iconnx_b200/csrc/qgemm.cu applies the zero points afterwards, modulo 2^32
(the reference's checked i32 arithmetic panics where this wraps; the oracle
wraps like the kernel, and the configs never get there):
    sum_k (a - za)(b - zb[n]) = acc - za * colsum[n] + zb[n] * (K * za - rowsum[m])
with colsum[n] = sum_k b[k, n] (prepared once per weight) and
rowsum[m] = sum_k a[m, k] (from the quantise pass).  Quantised exports that
store u8 weights with a u8 zero point are converted once to s8 by w ^ 0x80
and zw ^ 0x80, which leaves every (w - zw) unchanged.
"""
import numpy as np
import pytest

from iconnx_b200 import synth
from oracle import oracle


def _wrap32(v):
    return ((np.asarray(v, np.int64) + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int32)


def _epilogue(a, b, za, zb):
    """The kernel's correction on the raw product, in 32-bit wraparound."""
    a64, b64 = a.astype(np.int64), b.astype(np.int64)
    K = a.shape[1]
    acc = a64 @ b64
    colsum = b64.sum(axis=0)
    rowsum = a64.sum(axis=1)
    zb = np.broadcast_to(np.asarray(zb, np.int64), (b.shape[1],))
    v = acc - za * colsum[None, :] + zb[None, :] * (K * za - rowsum[:, None])
    return _wrap32(v)


@pytest.mark.parametrize("a_signed,b_signed", [(False, True), (False, False), (True, True), (True, False)])
@pytest.mark.parametrize("per_col", [False, True])
def test_zero_point_correction_equals_oracle(a_signed, b_signed, per_col):
    rng = np.random.default_rng(61 + 2 * a_signed + b_signed + 4 * per_col)
    M, K, N = 37, 203, 29
    at = np.int8 if a_signed else np.uint8
    bt = np.int8 if b_signed else np.uint8
    lo_a, hi_a = (-128, 128) if a_signed else (0, 256)
    lo_b, hi_b = (-128, 128) if b_signed else (0, 256)
    a = rng.integers(lo_a, hi_a, (M, K)).astype(at)
    b = rng.integers(lo_b, hi_b, (K, N)).astype(bt)
    za = int(rng.integers(lo_a, hi_a))
    zb = rng.integers(lo_b, hi_b, N if per_col else 1).astype(bt)
    got = _epilogue(a, b, za, zb.astype(np.int64) if per_col else int(zb[0]))
    ref = oracle.matmul_integer(a, b, np.array(za, at), zb if per_col else zb[0])
    np.testing.assert_array_equal(got, ref)


def test_zero_point_correction_wraps_like_i32():
    """Long K with extreme operands: the true sums leave the i32 range (where
    the reference would panic) and the kernel's algebra wraps exactly as the
    oracle does."""
    K = 70_000
    a = np.full((2, K), 255, np.uint8)
    b = np.full((K, 3), -128, np.int8)
    got = _epilogue(a, b, 0, 127)
    ref = oracle.matmul_integer(a, b, np.uint8(0), np.int8(127))
    np.testing.assert_array_equal(got, ref)


def test_u8_weights_convert_exactly_to_s8():
    rng = np.random.default_rng(62)
    M, K, N = 16, 96, 24
    a = synth.int8_uniform((M, K), 63).astype(np.int16)
    a = (a + 128).astype(np.uint8)
    w = rng.integers(0, 256, (K, N)).astype(np.uint8)
    zw = rng.integers(0, 256, N).astype(np.uint8)
    za = np.uint8(113)
    ref = oracle.matmul_integer(a, w, za, zw)
    ws = (w ^ 0x80).view(np.int8)
    zs = (zw ^ 0x80).view(np.int8)
    np.testing.assert_array_equal(oracle.matmul_integer(a, ws, za, zs), ref)
    np.testing.assert_array_equal(_epilogue(a, ws, int(za), zs.astype(np.int64)), ref)
