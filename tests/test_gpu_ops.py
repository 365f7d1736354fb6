"""GPU parity tests: the sm_100a kernels (through the C ABI) against the CPU
oracle on identical seeded inputs.

Contract (restating the reference's GPU==CPU tests,
tests/dynamic_quantize_linear_test.rs:28-136, tests/matmul_integer_test.rs:
170-307, tests/dequantize_linear_test.rs:20-186):
  * u8 quantised values, scale, zero-point and s32 accumulators: bit-exact;
  * f32 dequantised output (Cast -> Mul -> Add): bit-exact (tolerance 0 ulp,
    within the 1-ulp bar);
  * output after erf-GELU: within 1e-5 absolute.
"""
import numpy as np
import pytest
import torch

from iconnx_b200 import IcxError, ops, synth
from oracle import oracle
from tests.golden_io import load

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GELU_ATOL = 1e-5


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    return t.cpu().numpy()


def dql_both(x):
    gy, gs, gz = ops.gpu_dynamic_quantize_linear(cu(x))
    oy, os_, oz = oracle.dynamic_quantize_linear(x)
    return (host(gy), host(gs).item(), host(gz).item()), (oy, float(os_), int(oz))


# ------------------------------------------------------ DynamicQuantizeLinear
def test_dql_simple_positive():
    (y, s, z), (oy, os_, oz) = dql_both(np.array([0.0, 2.0, 4.0], np.float32))
    assert y.tolist() == [0, 128, 255] == oy.tolist()
    assert s == os_ and z == oz == 0


def test_dql_negative_tie():
    (_, _, z), (_, _, oz) = dql_both(np.array([-1.0, 0.0, 1.0], np.float32))
    assert z == oz == 128


def test_dql_constant_zero_range():
    (y, s, z), _ = dql_both(np.zeros(5, np.float32))
    assert y.tolist() == [0] * 5 and s == 0.0 and z == 0


def test_dql_3d_shape_preserved():
    x = (np.arange(24, dtype=np.float32) * np.float32(0.1)).reshape(2, 3, 4)
    gy, gs, gz = ops.gpu_dynamic_quantize_linear(cu(x))
    assert list(gy.shape) == [2, 3, 4] and gs.dim() == 0 and gz.dim() == 0
    np.testing.assert_array_equal(host(gy), oracle.dynamic_quantize_linear(x)[0])


def test_dql_rejects_non_float():
    with pytest.raises(IcxError, match="must be Float32"):
        ops.gpu_dynamic_quantize_linear(torch.tensor([1, 2, 3], dtype=torch.int32, device=DEV))


@pytest.mark.parametrize("case", ["test_dynamicquantizelinear",
                                  "test_dynamicquantizelinear_max_adjusted",
                                  "test_dynamicquantizelinear_min_adjusted"])
def test_dql_onnx_golden_matches_oracle(case):
    (x,), _ = load(case)
    (y, s, z), (oy, os_, oz) = dql_both(x)
    np.testing.assert_array_equal(y, oy)
    assert s == os_ and z == oz


@pytest.mark.parametrize("shape,kind", [((1, 128, 768), "normal"), ((4096, 768), "normal"),
                                        ((4096, 3072), "normal"), ((1024, 1024), "outlier"),
                                        ((333, 77), "normal"), ((1,), "normal"), ((17,), "outlier")])
def test_dql_random_bit_exact(shape, kind):
    x = synth.normal(shape, 1.0, 0) if kind == "normal" else synth.outlier_mix(shape, 0)
    (y, s, z), (oy, os_, oz) = dql_both(x)
    assert s == os_ and z == oz
    np.testing.assert_array_equal(y, oy)


def test_dql_special_values():
    x = np.array([np.nan, -3.0, 1e-30, -0.0, 7.5, np.nan, 2.5, -1.25] * 37, np.float32)
    (y, s, z), (oy, os_, oz) = dql_both(x)
    assert s == os_ and z == oz
    np.testing.assert_array_equal(y, oy)


def test_dql_infinite_and_tiny_ranges():
    for x in (np.array([1.0, np.inf, -2.0, 3.0], np.float32),
              np.array([1e-40, -3e-41, 0.0, 2e-42] * 5, np.float32),
              np.array([-np.inf, 1.0, 2.0], np.float32)):
        (y, s, z), (oy, os_, oz) = dql_both(x)
        assert (s == os_ or (np.isnan(s) and np.isnan(os_))) and z == oz
        np.testing.assert_array_equal(y, oy)


def test_dql_exact_ties_everywhere():
    # integers scaled so that many x/scale land exactly on .5
    x = (np.arange(-255, 256, dtype=np.float32) * np.float32(0.5))
    (y, s, z), (oy, os_, oz) = dql_both(x)
    assert s == os_ and z == oz
    np.testing.assert_array_equal(y, oy)


def test_dql_misaligned_view():
    base = synth.normal((4097,), 1.0, 3)
    t = cu(base)[1:]  # 4-byte offset: scalar path
    gy, gs, gz = ops.gpu_dynamic_quantize_linear(t)
    oy, os_, oz = oracle.dynamic_quantize_linear(base[1:])
    np.testing.assert_array_equal(host(gy), oy)
    assert host(gs).item() == os_


@pytest.mark.parametrize("M,K", [(64, 768), (5, 40), (3, 7)])
def test_dql_rowsum(M, K):
    x = synth.normal((M, K), 1.0, 4)
    y, s, z, rows = ops.gpu_dynamic_quantize_linear(cu(x), row_len=K)
    np.testing.assert_array_equal(host(rows), oracle.rowsum_u8(host(y)))


# -------------------------------------------------------------- MatMulInteger
def test_mmi_u8_s8_kat():
    a = np.array([[1, 2, 3], [4, 5, 6]], np.uint8)
    b = np.array([[1, 2], [3, 4], [5, 6]], np.int8)
    assert host(ops.gpu_matmul_integer(cu(a), cu(b))).ravel().tolist() == [22, 28, 49, 64]


def test_mmi_s8_s8_zp_kat():
    a = np.array([[10, 20], [30, 40]], np.int8)
    b = np.array([[1, 2], [3, 4]], np.int8)
    out = ops.gpu_matmul_integer(cu(a), cu(b), cu(np.array(5, np.int8)), cu(np.array(1, np.int8)))
    assert host(out).ravel().tolist() == [30, 50, 70, 130]


def test_mmi_k768_ones_and_k3072_overflow_safety():
    out = ops.gpu_matmul_integer(cu(np.ones((4, 768), np.uint8)), cu(np.ones((768, 4), np.int8)))
    assert (host(out) == 768).all()
    out = ops.gpu_matmul_integer(cu(np.full((1, 3072), 100, np.uint8)),
                                 cu(np.full((3072, 1), 100, np.int8)))
    assert host(out)[0, 0] == 30_720_000


def test_mmi_onnx_golden_u8u8():
    (a, b, az, bz), (y,) = load("test_matmulinteger")
    out = ops.gpu_matmul_integer(cu(a), cu(b), cu(az), cu(bz))
    np.testing.assert_array_equal(host(out), y)


@pytest.mark.parametrize("M,K,N", [(128, 768, 768), (1, 16, 8), (129, 48, 5), (300, 256, 300),
                                   (513, 3072, 768), (64, 1024, 1024), (7, 3, 9), (1000, 4096, 256)])
@pytest.mark.parametrize("signs", ["u8s8", "s8s8", "u8u8", "s8u8"])
def test_mmi_random_bit_exact(M, K, N, signs):
    if signs != "u8s8" and M * N * K > 50_000_000:
        pytest.skip("large shapes run for u8s8 only")
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    adt = np.uint8 if signs[:2] == "u8" else np.int8
    bdt = np.uint8 if signs[2:] == "u8" else np.int8
    a = rng.integers(np.iinfo(adt).min, np.iinfo(adt).max + 1, (M, K)).astype(adt)
    b = rng.integers(np.iinfo(bdt).min, np.iinfo(bdt).max + 1, (K, N)).astype(bdt)
    az = np.array(rng.integers(0, 100), adt)
    bz = np.array(rng.integers(0, 100), bdt)
    out = ops.gpu_matmul_integer(cu(a), cu(b), cu(az), cu(bz))
    np.testing.assert_array_equal(host(out), oracle.matmul_integer(a, b, az, bz))


def test_mmi_per_column_b_zero_point():
    rng = np.random.default_rng(11)
    a = rng.integers(0, 256, (200, 768), dtype=np.uint8)
    b = synth.int8_uniform((768, 384), 1)
    bz = synth.int8_uniform((384,), 5, -8, 8)
    out = ops.gpu_matmul_integer(cu(a), cu(b), cu(np.array(131, np.uint8)), cu(bz))
    np.testing.assert_array_equal(host(out), oracle.matmul_integer(a, b, np.uint8(131), bz))


def test_mmi_rank3_flattening():
    rng = np.random.default_rng(12)
    a = rng.integers(0, 256, (2, 64, 128), dtype=np.uint8)
    b = synth.int8_uniform((128, 96), 2)
    out = ops.gpu_matmul_integer(cu(a), cu(b))
    assert list(out.shape) == [2, 64, 96]
    np.testing.assert_array_equal(host(out), oracle.matmul_integer(a, b))


def test_mmi_rejections():
    f = cu(np.ones((2, 2), np.float32))
    i8 = cu(np.ones((2, 2), np.int8))
    with pytest.raises(IcxError, match="must be Int8 or UInt8"):
        ops.gpu_matmul_integer(f, i8)
    with pytest.raises(IcxError, match="K mismatch"):
        ops.gpu_matmul_integer(cu(np.ones((2, 3), np.int8)), cu(np.ones((4, 2), np.int8)))
    with pytest.raises(IcxError, match="dtype"):
        ops.gpu_matmul_integer(i8, i8, cu(np.array(0, np.uint8)))


# ----------------------------------------------------------- DequantizeLinear
def test_deq_kats_exact():
    cases = [
        (np.array([-128, 0, 127], np.int8), np.array(0.5, np.float32), None, 1),
        (np.array([[1, 2], [3, 4]], np.int8), np.array([0.1, 0.2], np.float32), None, 0),
        (np.array([0, 128, 255], np.uint8), np.array(0.5, np.float32), np.array(128, np.uint8), 1),
        (np.array([100, -50, 200], np.int32), np.array(0.01, np.float32), None, 1),
        (np.array([[10, 20, 30], [40, 50, 60]], np.uint8), np.array([1.0, 0.5, 0.25], np.float32),
         np.array([0, 10, 20], np.uint8), 1),
    ]
    for x, s, z, ax in cases:
        g = ops.gpu_dequantize_linear(cu(x), cu(s), None if z is None else cu(z), axis=ax)
        np.testing.assert_array_equal(host(g), oracle.dequantize_linear(x, s, z, axis=ax))


@pytest.mark.parametrize("case", ["test_dequantizelinear", "test_dequantizelinear_axis"])
def test_deq_onnx_golden(case):
    (x, s, z), (y,) = load(case)
    np.testing.assert_array_equal(host(ops.gpu_dequantize_linear(cu(x), cu(s), cu(z))), y)


def test_deq_rejections():
    x = cu(np.ones(3, np.int8))
    with pytest.raises(IcxError, match="zero_point dtype"):
        ops.gpu_dequantize_linear(x, cu(np.array(0.1, np.float32)), cu(np.array(5, np.uint8)))
    with pytest.raises(IcxError, match="zero_point shape"):
        ops.gpu_dequantize_linear(cu(np.ones(4, np.int8)), cu(np.array(0.1, np.float32)),
                                  cu(np.zeros(2, np.int8)))


# ------------------------------------------------------ fused quantised Linear
def _chain(M, K, N, gelu, per_col=False, kind="normal", seed=0):
    x = synth.normal((M, K), 1.0, seed) if kind == "normal" else synth.outlier_mix((M, K), seed)
    w = synth.int8_uniform((K, N), 1 + seed)
    bias = synth.normal((N,), 0.02, 2 + seed)
    if per_col:
        ws = synth.uniform_f32((N,), 0.005, 0.02, 4 + seed)
        bz = synth.int8_uniform((N,), 5 + seed, -8, 8)
    else:
        ws = np.array([0.01], np.float32)
        bz = None
    pw = ops.prepare_weight(cu(w))
    out, y, s, z = ops.dynamic_quant_linear(cu(x), pw, cu(ws), cu(bias),
                                            None if bz is None else cu(bz), gelu)
    ref = oracle.quant_linear(x, w, ws, bias, bz, gelu)
    return host(out), host(y), host(s).item(), host(z).item(), ref


@pytest.mark.parametrize("M,K,N", [(128, 768, 768), (4096, 768, 3072), (4096, 3072, 768),
                                   (100, 64, 40), (1, 32, 16), (257, 1024, 1024)])
def test_quant_linear_bit_exact(M, K, N):
    out, y, s, z, (rout, ry, rs, rz, racc) = _chain(M, K, N, gelu=False)
    np.testing.assert_array_equal(y, ry)
    assert s == rs and z == rz
    np.testing.assert_array_equal(out.view(np.uint32), rout.view(np.uint32))


@pytest.mark.parametrize("M,K,N", [(4096, 768, 3072), (130, 96, 200)])
def test_quant_linear_gelu(M, K, N):
    out, y, s, z, (rout, ry, rs, rz, _) = _chain(M, K, N, gelu=True)
    np.testing.assert_array_equal(y, ry)
    np.testing.assert_allclose(out, rout, atol=GELU_ATOL, rtol=0)


def test_quant_linear_per_column_scale_and_zero_point():
    out, y, s, z, (rout, ry, rs, rz, _) = _chain(512, 768, 768, gelu=False, per_col=True)
    np.testing.assert_array_equal(y, ry)
    np.testing.assert_array_equal(out.view(np.uint32), rout.view(np.uint32))


def test_quant_linear_outliers_large_m():
    out, y, s, z, (rout, ry, rs, rz, _) = _chain(8192, 1024, 1024, gelu=False, kind="outlier")
    np.testing.assert_array_equal(y, ry)
    np.testing.assert_array_equal(out.view(np.uint32), rout.view(np.uint32))


def test_ffn_block_stagewise():
    """Config 2: DQL -> GEMM1 (+bias, GELU) -> DQL -> GEMM2 (+bias), checked
    stage by stage (each GPU stage against the oracle fed the same input)."""
    M = 4096
    x = synth.normal((M, 768), 1.0, 0)
    w1, w2 = synth.int8_uniform((768, 3072), 1), synth.int8_uniform((3072, 768), 3)
    b1, b2 = synth.normal((3072,), 0.02, 2), synth.normal((768,), 0.02, 102)
    ws = np.array([0.01], np.float32)
    p1, p2 = ops.prepare_weight(cu(w1)), ops.prepare_weight(cu(w2))
    h, *_ = ops.dynamic_quant_linear(cu(x), p1, cu(ws), cu(b1), gelu=True)
    out, y2, s2, z2 = ops.dynamic_quant_linear(h, p2, cu(ws), cu(b2))
    rh = oracle.quant_linear(x, w1, ws, b1, None, True)[0]
    np.testing.assert_allclose(host(h), rh, atol=GELU_ATOL, rtol=0)
    rout, ry2, rs2, rz2, _ = oracle.quant_linear(host(h), w2, ws, b2, None, False, threads=8)
    np.testing.assert_array_equal(host(y2), ry2)
    assert host(s2).item() == rs2 and host(z2).item() == rz2
    np.testing.assert_array_equal(host(out).view(np.uint32), rout.view(np.uint32))


@pytest.mark.parametrize("M,K,N,gelu,per_col", [(4096, 768, 3072, True, False), (300, 64, 77, False, False),
                                                (512, 768, 768, False, True), (5, 3, 9, False, False)])
def test_producer_fused_minmax_then_quantize(M, K, N, gelu, per_col):
    """GEMM epilogue writes (min, max) partials; the next DQL's quantise pass
    alone must equal a full DQL of the same tensor (and the oracle)."""
    x = synth.normal((M, K), 1.0, 21)
    w = synth.int8_uniform((K, N), 22)
    bias = synth.normal((N,), 0.02, 23)
    ws = synth.uniform_f32((N,), 0.005, 0.02, 24) if per_col else np.array([0.01], np.float32)
    bz = synth.int8_uniform((N,), 25, -8, 8) if per_col else None
    pw = ops.prepare_weight(cu(w))
    mm = ops.MinMaxPartials(DEV)
    h, *_ = ops.dynamic_quant_linear(cu(x), pw, cu(ws), cu(bias), None if bz is None else cu(bz),
                                     gelu, out_minmax=mm)
    assert 1 <= mm.n <= 1184
    y1, s1, z1 = ops.gpu_dynamic_quantize_from_partials(h, mm)
    y2, s2, z2 = ops.gpu_dynamic_quantize_linear(h)
    oy, os_, oz = oracle.dynamic_quantize_linear(host(h))
    np.testing.assert_array_equal(host(y1), oy)
    np.testing.assert_array_equal(host(y2), oy)
    assert host(s1).item() == host(s2).item() == os_ and host(z1).item() == oz


def test_ffn_block_fused_chain_bit_exact():
    """Config 2 with the producer-fused DQL2: DQL2 and GEMM2 stages bit-exact."""
    M = 4096
    x = synth.normal((M, 768), 1.0, 0)
    w1, w2 = synth.int8_uniform((768, 3072), 1), synth.int8_uniform((3072, 768), 3)
    b1, b2 = synth.normal((3072,), 0.02, 2), synth.normal((768,), 0.02, 102)
    ws = np.array([0.01], np.float32)
    p1, p2 = ops.prepare_weight(cu(w1)), ops.prepare_weight(cu(w2))
    mm = ops.MinMaxPartials(DEV)
    h, *_ = ops.dynamic_quant_linear(cu(x), p1, cu(ws), cu(b1), gelu=True, out_minmax=mm)
    out, y2, s2, z2 = ops.dynamic_quant_linear(h, p2, cu(ws), cu(b2), x_minmax=mm)
    rout, ry2, rs2, rz2, _ = oracle.quant_linear(host(h), w2, ws, b2, None, False, threads=8)
    np.testing.assert_array_equal(host(y2), ry2)
    assert host(s2).item() == rs2 and host(z2).item() == rz2
    np.testing.assert_array_equal(host(out).view(np.uint32), rout.view(np.uint32))


def test_quant_linear_residual_epilogue_bit_exact():
    """Residual Add(out, r) fused in the epilogue == the separate f32 Add."""
    M, K, N = 1000, 768, 768
    x = synth.normal((M, K), 1.0, 41)
    r = synth.normal((M, N), 3.0, 42)
    w = synth.int8_uniform((K, N), 43)
    bias = synth.normal((N,), 0.02, 44)
    ws = np.array([0.01], np.float32)
    pw = ops.prepare_weight(cu(w))
    y, s, z = ops.gpu_dynamic_quantize_linear(cu(x))
    out = ops.quant_linear(y, s, z, pw, cu(ws), cu(bias), residual=cu(r))
    ref = oracle.quant_linear(x, w, ws, bias)[0] + r
    np.testing.assert_array_equal(host(out).view(np.uint32), ref.astype(np.float32).view(np.uint32))


# Large deep GEMMs (M >= 8192, K >= 1536) run as CTA pairs (tcgen05
# cta_group::2, 256-row tiles): ragged M and N, per-column scale / zero point,
# GELU, residual.
@pytest.mark.parametrize("M,K,N,gelu,per_col,residual", [
    (8192 + 77, 1536, 1000, False, True, False),
    (8192 + 200, 2048, 1000, True, False, False),
    (8192, 3072, 768, False, True, True),
    (16384 - 3, 1536, 2304, False, False, True),
])
def test_quant_linear_cta_pairs_bit_exact(M, K, N, gelu, per_col, residual):
    x = synth.normal((M, K), 1.0, 21)
    w = synth.int8_uniform((K, N), 22)
    bias = synth.normal((N,), 0.02, 23)
    if per_col:
        ws = synth.uniform_f32((N,), 0.005, 0.02, 24)
        bz = synth.int8_uniform((N,), 25, -8, 8)
    else:
        ws, bz = np.array([0.01], np.float32), None
    res = synth.normal((M, N), 1.0, 26) if residual else None
    pw = ops.prepare_weight(cu(w))
    outs = ops.gpu_dynamic_quantize_linear(cu(x), row_len=K if bz is not None else None)
    y, s, z = outs[:3]
    rows = outs[3] if bz is not None else None
    out = ops.quant_linear(y, s, z, pw, cu(ws), cu(bias), None if bz is None else cu(bz), rows,
                           gelu=gelu, residual=None if res is None else cu(res))
    ref = oracle.quant_linear_from_q(host(y), host(s).item(), host(z).item(), w, ws, bias, bz,
                                     gelu=gelu, residual=res, threads=8)
    ry, rs, rz = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(host(y), ry)
    if gelu:
        np.testing.assert_allclose(host(out), ref, atol=GELU_ATOL, rtol=0)
    else:
        np.testing.assert_array_equal(host(out).view(np.uint32), ref.view(np.uint32))


def test_s32_matmul_integer_cta_pairs_bit_exact():
    M, K, N = 8192 + 5, 2048, 520
    rng = np.random.default_rng(3)
    a = rng.integers(0, 256, (M, K)).astype(np.uint8)
    b = rng.integers(-127, 128, (K, N)).astype(np.int8)
    az = np.array(9, np.uint8)
    bz = rng.integers(-8, 9, (N,)).astype(np.int8)
    got = host(ops.gpu_matmul_integer(cu(a), cu(b), cu(az), cu(bz)))
    np.testing.assert_array_equal(got, oracle.matmul_integer(a, b, az, bz, threads=8))


# QuantLinear + residual Add + LayerNormalization in one launch: clusters of
# N / 192 CTAs hold whole rows and exchange the row statistics through
# distributed shared memory.  The residual sum before the LayerNorm is exact
# (the QuantLinear epilogue's arithmetic); the normalisation sums in another
# order than the reference (layer_normalization.rs:25-80), so y is compared
# with the restated operator within the LayerNorm kernel's 4e-6.
@pytest.mark.parametrize("M,K,N,per_col,beta", [
    (4096, 768, 768, False, True),      # DistilBERT O-proj
    (4096, 3072, 768, False, True),     # DistilBERT FFN2 (deep ring)
    (1000, 768, 768, True, True),       # per-column scale / zero point, ragged M
    (300, 768, 384, False, False),      # clusters of two, no beta
    (77, 1536, 576, True, True),        # clusters of three, deep
])
def test_quant_linear_layernorm(M, K, N, per_col, beta):
    x = synth.normal((M, K), 1.0, 51)
    w = synth.int8_uniform((K, N), 52)
    bias = synth.normal((N,), 0.02, 53)
    if per_col:
        ws = synth.uniform_f32((N,), 0.005, 0.02, 54)
        bz = synth.int8_uniform((N,), 55, -8, 8)
    else:
        ws, bz = np.array([0.01], np.float32), None
    res = synth.normal((M, N), 1.0, 56)
    gamma = (1.0 + synth.normal((N,), 0.05, 57)).astype(np.float32)
    bet = synth.normal((N,), 0.05, 58) if beta else None
    pw = ops.prepare_weight(cu(w))
    outs = ops.gpu_dynamic_quantize_linear(cu(x), row_len=K if bz is not None else None)
    y, s, z = outs[:3]
    rows = outs[3] if bz is not None else None
    mm = ops.MinMaxPartials(DEV)
    out = ops.quant_linear_layernorm(y, s, z, pw, cu(ws), cu(res), cu(gamma),
                                     None if bet is None else cu(bet), 1e-5, cu(bias),
                                     None if bz is None else cu(bz), rows, minmax=mm)
    zsum = oracle.quant_linear_from_q(host(y), host(s).item(), host(z).item(), w, ws, bias, bz,
                                      residual=res, threads=8)
    ref = oracle.layer_normalization(zsum, gamma, bet, 1e-5)
    got = host(out)
    assert np.abs(got.astype(np.float64) - ref).max() <= 4e-6
    # the (min, max) partials cover exactly the output (seeded with 0)
    parts = host(mm.buf)[:mm.n]
    assert mm.n >= N // 192
    assert parts[:, 0].min() == min(0.0, got.min()) and parts[:, 1].max() == max(0.0, got.max())


def test_quant_linear_layernorm_rejects_unsupported_widths():
    x = cu(np.zeros((4, 64), np.uint8))
    pw = ops.prepare_weight(cu(synth.int8_uniform((64, 200), 1)))
    one = cu(np.array(1.0, np.float32))
    with pytest.raises(IcxError, match="unsupported"):
        ops.quant_linear_layernorm(x, one, cu(np.array(0, np.uint8)), pw, cu(np.array([0.01], np.float32)),
                                   cu(np.zeros((4, 200), np.float32)), cu(np.ones(200, np.float32)))
