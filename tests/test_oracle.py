"""Pins the CPU oracle against the reference's own known-answer tests and the
ONNX 1.18 node-test vectors the reference vendors.

Known answers restated from (reference paths):
  src/operators/dynamic_quantize_linear.rs:119-169
  src/operators/matmul_integer.rs:273-382
  src/operators/dequantize_linear.rs:216-297
  src/operators/erf.rs:42-171
  tests/operators/layer_norm_test.rs, softmax_test.rs, matmul_test.rs (the
  fp32 glue of the encoder, restated from src/operators/
  layer_normalization.rs:25-80, softmax.rs:21-56, matmul.rs:27-186)
"""
import numpy as np
import pytest

from oracle import oracle
from tests.golden_io import attributes, load


# --- DynamicQuantizeLinear KATs (dynamic_quantize_linear.rs:119-169) -------
def test_dql_simple_positive():
    y, s, z = oracle.dynamic_quantize_linear(np.array([0.0, 2.0, 4.0], np.float32))
    assert y.tolist() == [0, 128, 255]
    assert abs(s - 4.0 / 255.0) < 1e-6
    assert z == 0


def test_dql_negative_tie_rounds_to_even():
    _, _, z = oracle.dynamic_quantize_linear(np.array([-1.0, 0.0, 1.0], np.float32))
    assert z == 128


def test_dql_constant_zero_range():
    y, s, z = oracle.dynamic_quantize_linear(np.zeros(5, np.float32))
    assert y.tolist() == [0] * 5 and s == 0.0 and z == 0


def test_dql_nan_skipped_and_zero():
    x = np.array([np.nan, -2.0, 3.0, np.nan], np.float32)
    y, s, z = oracle.dynamic_quantize_linear(x)
    assert y[0] == 0 and y[3] == 0
    assert s == np.float32(5.0 / 255.0)


@pytest.mark.parametrize("case", ["test_dynamicquantizelinear",
                                  "test_dynamicquantizelinear_max_adjusted",
                                  "test_dynamicquantizelinear_min_adjusted"])
def test_dql_onnx_golden(case):
    (x,), (y, s, z) = load(case)
    gy, gs, gz = oracle.dynamic_quantize_linear(x)
    y = y.copy()
    if case == "test_dynamicquantizelinear":
        # The reference quantises with an f64 scale (dynamic_quantize_linear.rs:
        # 89-103): -2.5 / (5/255) is exactly -127.5 in f64 and rounds to even
        # (-128, +153 -> 25).  The ONNX vector divides by an f32 scale and gets
        # -127.49999 -> 26.  Parity follows the reference, so that one element
        # is pinned to the reference's value.
        assert x.ravel()[3] == np.float32(-2.5) and y.ravel()[3] == 26
        y.ravel()[3] = 25
    np.testing.assert_array_equal(gy, y)
    assert gs == s
    assert gz == z


# --- MatMulInteger KATs (matmul_integer.rs:273-382) ------------------------
def test_mmi_u8_s8_no_zp():
    a = np.array([[1, 2, 3], [4, 5, 6]], np.uint8)
    b = np.array([[1, 2], [3, 4], [5, 6]], np.int8)
    assert oracle.matmul_integer(a, b).reshape(-1).tolist() == [22, 28, 49, 64]


def test_mmi_s8_s8_with_zp():
    a = np.array([[10, 20], [30, 40]], np.int8)
    b = np.array([[1, 2], [3, 4]], np.int8)
    out = oracle.matmul_integer(a, b, np.int8(5), np.int8(1))
    assert out.reshape(-1).tolist() == [30, 50, 70, 130]


def test_mmi_k768_ones():
    out = oracle.matmul_integer(np.ones((4, 768), np.uint8), np.ones((768, 4), np.int8))
    assert (out == 768).all()


def test_mmi_k3072_overflow_safety():
    out = oracle.matmul_integer(np.full((1, 3072), 100, np.uint8), np.full((3072, 1), 100, np.int8))
    assert out[0, 0] == 30_720_000


def test_mmi_onnx_golden():
    (a, b, az, bz), (y,) = load("test_matmulinteger")
    np.testing.assert_array_equal(oracle.matmul_integer(a, b, az, bz), y)


def test_mmi_per_column_zp_matches_spec():
    rng = np.random.default_rng(0)
    a = rng.integers(0, 256, (5, 7), dtype=np.uint8)
    b = rng.integers(-127, 128, (7, 3), dtype=np.int8)
    bz = np.array([-3, 0, 8], np.int8)
    ref = (a.astype(np.int64) - 9) @ (b.astype(np.int64) - bz.astype(np.int64)[None, :])
    np.testing.assert_array_equal(oracle.matmul_integer(a, b, np.uint8(9), bz), ref)


def test_mmi_threads_agree():
    rng = np.random.default_rng(1)
    a = rng.integers(0, 256, (37, 64), dtype=np.uint8)
    b = rng.integers(-127, 128, (64, 19), dtype=np.int8)
    np.testing.assert_array_equal(oracle.matmul_integer(a, b, threads=1),
                                  oracle.matmul_integer(a, b, threads=4))


# --- DequantizeLinear KATs (dequantize_linear.rs:216-297) ------------------
def test_deq_kats():
    np.testing.assert_allclose(oracle.dequantize_linear(np.array([-128, 0, 127], np.int8), 0.5),
                               [-64, 0, 63.5], atol=1e-6)
    np.testing.assert_allclose(
        oracle.dequantize_linear(np.array([[1, 2], [3, 4]], np.int8), np.array([0.1, 0.2]), axis=0).ravel(),
        [0.1, 0.2, 0.6, 0.8], atol=1e-6)
    np.testing.assert_allclose(
        oracle.dequantize_linear(np.array([0, 128, 255], np.uint8), 0.5, np.uint8(128)),
        [-64, 0, 63.5], atol=1e-6)
    np.testing.assert_allclose(
        oracle.dequantize_linear(np.array([100, -50, 200], np.int32), 0.01), [1, -0.5, 2], atol=1e-6)


@pytest.mark.parametrize("case", ["test_dequantizelinear", "test_dequantizelinear_axis"])
def test_deq_onnx_golden(case):
    (x, s, z), (y,) = load(case)
    np.testing.assert_array_equal(oracle.dequantize_linear(x, s, z, axis=1), y)


# --- Erf / GELU (erf.rs:42-171) --------------------------------------------
def test_erf_spot_and_bounds():
    assert oracle.erf(np.array([0.0], np.float32))[0] == 0.0
    assert abs(oracle.erf(np.array([1.0], np.float32))[0] - 0.8427008) < 1e-6
    assert abs(oracle.erf(np.array([-1.0], np.float32))[0] + 0.8427008) < 1e-6
    g = np.linspace(-6, 6, 12001).astype(np.float32)
    e = oracle.erf(g)
    assert np.all(np.abs(e) <= 1.0)
    np.testing.assert_array_equal(oracle.erf(-g), -e)
    assert np.all(np.diff(e) >= 0)


def test_erf_onnx_golden():
    (x,), (y,) = load("test_erf")
    # A&S 7.1.26 is a 1.5e-7 approximation; f32 evaluation adds a few ulp.
    np.testing.assert_allclose(oracle.erf(x), y, atol=1e-6)


@pytest.mark.parametrize("case", ["test_gelu_default_1", "test_gelu_default_2"])
def test_gelu_onnx_golden(case):
    (x,), (y,) = load(case)
    np.testing.assert_allclose(oracle.gelu(x), y, atol=1e-6)


def test_quant_linear_chain_composes_ops():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((9, 32)).astype(np.float32)
    w = rng.integers(-127, 128, (32, 5), dtype=np.int8)
    bias = (rng.standard_normal(5) * 0.02).astype(np.float32)
    out, q, s, z, acc = oracle.quant_linear(x, w, np.float32(0.01), bias, gelu=True)
    q2, s2, z2 = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(q, q2)
    acc2 = oracle.matmul_integer(q2, w, z2)
    np.testing.assert_array_equal(acc, acc2)
    sc = np.float32(s2) * np.float32(0.01)
    ref = oracle.gelu(oracle.cast_i32_f32(acc2) * sc + bias)
    np.testing.assert_array_equal(out, ref)



# --- fp32 glue: reference KATs and ONNX node vectors -------------------------
def test_layer_norm_reference_kats():
    # tests/operators/layer_norm_test.rs: rows normalise to mean ~0; with
    # scale 2 and bias 1 the mean is ~1
    y = oracle.layer_normalization(np.array([[1, 2, 3, 4]], np.float32), np.ones(4, np.float32),
                                   np.zeros(4, np.float32))
    assert abs(y.mean()) < 0.01
    y = oracle.layer_normalization(np.array([[1, 2, 3], [4, 5, 6]], np.float32),
                                   np.ones(3, np.float32), np.zeros(3, np.float32))
    assert np.all(np.abs(y.mean(-1)) < 0.01)
    y = oracle.layer_normalization(np.array([[1, 2, 3]], np.float32), np.full(3, 2, np.float32),
                                   np.ones(3, np.float32))
    assert abs(y.mean() - 1.0) < 0.1


def test_layer_norm_op_order_is_the_references():
    """mean -> centered -> variance -> sqrt(var + eps) -> divide -> scale ->
    bias, each rounded once, sums in ndarray's 8-accumulator order."""
    x = (np.arange(19, dtype=np.float32) * np.float32(0.37) - np.float32(2.1)).reshape(1, 19)
    g = np.linspace(0.5, 1.5, 19).astype(np.float32)
    b = np.linspace(-0.1, 0.1, 19).astype(np.float32)
    f32 = np.float32

    def s8(v):
        p = [f32(0)] * 8
        n8 = len(v) // 8 * 8
        for i in range(0, n8, 8):
            for u in range(8):
                p[u] = f32(p[u] + v[i + u])
        acc = f32(0)
        for u in range(4):
            acc = f32(acc + f32(p[u] + p[u + 4]))
        for t in v[n8:]:
            acc = f32(acc + t)
        return acc

    r = x[0]
    mean = f32(s8(r) / f32(19))
    c = (r - mean).astype(f32)
    var = f32(s8((c * c).astype(f32)) / f32(19))
    sd = f32(np.sqrt(f32(var + f32(1e-5))))
    want = (((c / sd).astype(f32) * g).astype(f32) + b).astype(f32)
    got = oracle.layer_normalization(x, g, b, 1e-5)[0]
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("case", ["test_layer_normalization_2d_axis_negative_1",
                                  "test_layer_normalization_3d_axis_negative_1_epsilon",
                                  "test_layer_normalization_4d_axis_negative_1"])
def test_layer_norm_onnx_golden(case):
    (x, scale, bias), (y, *_) = load(case)
    eps = attributes(case).get("epsilon", 1e-5)
    np.testing.assert_allclose(oracle.layer_normalization(x, scale, bias, eps), y,
                               rtol=1e-5, atol=1e-6)


def test_softmax_reference_kats():
    # tests/operators/softmax_test.rs: [1, 2, 3] -> ~[0.090, 0.245, 0.665]
    y = oracle.softmax(np.array([1, 2, 3], np.float32))
    assert abs(y.sum() - 1.0) < 1e-3
    np.testing.assert_allclose(y, [0.090, 0.245, 0.665], atol=0.01)


@pytest.mark.parametrize("case", ["test_softmax_axis_2", "test_softmax_default_axis",
                                  "test_softmax_example", "test_softmax_large_number",
                                  "test_softmax_negative_axis"])
def test_softmax_onnx_golden(case):
    (x,), (y,) = load(case)
    np.testing.assert_allclose(oracle.softmax(x), y, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("case", ["test_matmul_2d", "test_matmul_3d", "test_matmul_4d"])
def test_matmul_onnx_golden(case):
    (a, b), (y,) = load(case)
    np.testing.assert_allclose(oracle.matmul(a, b), y, rtol=1e-6, atol=1e-6)


def test_matmul_blocks_of_256_fused_steps():
    """matrixmultiply's FMA kernel: one fused multiply-add per k, blocks of
    kc = 256 summed in order (restated, not numpy's BLAS order)."""
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 600)).astype(np.float32)
    b = rng.standard_normal((600, 2)).astype(np.float32)
    want = np.empty((3, 2), np.float32)
    for i in range(3):
        for j in range(2):
            out = None
            for k0 in range(0, 600, 256):
                acc = np.float64(0)
                for k in range(k0, min(k0 + 256, 600)):
                    # one rounding per fused step: exact product + acc, then f32
                    acc = np.float64(np.float32(np.float64(a[i, k]) * np.float64(b[k, j]) + acc))
                out = np.float32(acc) if out is None else np.float32(out + np.float32(acc))
            want[i, j] = out
    np.testing.assert_array_equal(oracle.matmul(a, b).view(np.uint32), want.view(np.uint32))
