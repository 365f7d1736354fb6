"""Parity at the configurations' full sizes through sampled rows.

The oracle cannot run a 2.2 T-op GEMM in seconds, so at full size the whole
chain runs on the GPU and is checked where the oracle is cheap: the
DynamicQuantizeLinear of the full tensor (scale, zero point, every u8) and
the fused GEMM output on a random sample of rows, bit-exact.
"""
import numpy as np
import pytest
import torch

from iconnx_b200 import ops, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _sampled_rows_check(x, w, ws, bias, bz=None, rows=48, seed=0):
    M, K = x.shape
    N = w.shape[1]
    pw = ops.prepare_weight(torch.from_numpy(w).to(DEV))
    bzt = None if bz is None else torch.from_numpy(bz).to(DEV)
    out, y, s, z = ops.dynamic_quant_linear(torch.from_numpy(x).to(DEV), pw,
                                            torch.from_numpy(ws).to(DEV),
                                            torch.from_numpy(bias).to(DEV), bzt)
    oy, os_, oz = oracle.dynamic_quantize_linear(x)
    assert s.item() == os_ and z.item() == oz
    np.testing.assert_array_equal(y.cpu().numpy(), oy)          # every u8 of the full tensor
    pick = np.sort(np.random.default_rng(seed).choice(M, rows, replace=False))
    acc = oracle.matmul_integer(oy[pick], w, np.uint8(oz), bz, threads=8)
    sc = np.float32(os_) * ws.astype(np.float32)
    ref = oracle.cast_i32_f32(acc) * (sc if sc.size > 1 else sc[0])
    ref = (ref + bias).astype(np.float32)
    got = out[torch.from_numpy(pick).to(DEV)].cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_config5_largest_point_sampled():
    """M=65536, K=N=4096, outlier-skewed activations (config 5)."""
    M, K, N = 65536, 4096, 4096
    x = synth.outlier_mix((M, K), 0)
    _sampled_rows_check(x, synth.int8_uniform((K, N), 1), np.array([0.01], np.float32),
                        synth.normal((N,), 0.02, 2))


@pytest.mark.parametrize("M,KN", [(m, kn) for m in (128, 1024, 8192, 65536) for kn in (768, 1024, 4096)
                                  if (m, kn) != (65536, 4096)])
def test_config5_sweep_points_sampled(M, KN):
    """Every other point of config 5's grid (the largest one is the test above)."""
    x = synth.outlier_mix((M, KN), 3)
    _sampled_rows_check(x, synth.int8_uniform((KN, KN), 4), np.array([0.01], np.float32),
                        synth.normal((KN,), 0.02, 5), rows=min(M, 48))


def test_config4_linear_per_column_full_rows():
    """BERT-base Linear at config 4's M = 64 x 512, per-column w_scale and b_zp."""
    M, K, N = 32768, 768, 3072
    x = synth.normal((M, K), 1.0, 6)
    _sampled_rows_check(x, synth.int8_uniform((K, N), 7), synth.uniform_f32((N,), 0.005, 0.02, 8),
                        synth.normal((N,), 0.02, 9), bz=synth.int8_uniform((N,), 10, -8, 8))


@pytest.mark.parametrize("M,K,N,gelu", [
    (4096, 768, 3072, True),    # config 3 FFN1 (GELU epilogue)
    (4096, 768, 2304, False),   # config 3 merged Q/K/V
    (4261, 768, 3000, True),    # ragged M and N: the last tiles read past M / N
])
def test_wide_shallow_gemm_sampled(M, K, N, gelu):
    """Config 3's wide, shallow-K GEMMs at full size (and a ragged variant
    whose last tiles run past M and N): every u8 of the quantised input and a
    sample of output rows that includes the first and last ones, bit-exact
    (1e-5 after GELU)."""
    x = synth.normal((M, K), 1.0, 11)
    w = synth.int8_uniform((K, N), 12)
    ws = np.array([0.01], np.float32)
    bias = synth.normal((N,), 0.02, 13)
    pw = ops.prepare_weight(torch.from_numpy(w).to(DEV))
    out, y, s, z = ops.dynamic_quant_linear(torch.from_numpy(x).to(DEV), pw,
                                            torch.from_numpy(ws).to(DEV),
                                            torch.from_numpy(bias).to(DEV), None, gelu=gelu)
    oy, os_, oz = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(y.cpu().numpy(), oy)
    rng = np.random.default_rng(14)
    pick = np.unique(np.concatenate([rng.choice(M, 40, replace=False), np.arange(M - 8, M),
                                     np.arange(0, 8), np.arange(128, 136), np.arange(256, 260)]))
    acc = oracle.matmul_integer(oy[pick], w, np.uint8(oz), None, threads=8)
    ref = (oracle.cast_i32_f32(acc) * (np.float32(os_) * ws[0]) + bias).astype(np.float32)
    got = out[torch.from_numpy(pick).to(DEV)].cpu().numpy()
    if gelu:
        np.testing.assert_allclose(got, oracle.gelu(ref), rtol=0, atol=1e-5)
    else:
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("M,K,N,per_col,gelu", [
    (4000, 1552, 4064, True, False),   # ragged M / N / K, per-column scale and zero point
    (4096, 2048, 4096, False, True),   # GELU epilogue
])
def test_long_k_gemm_every_row(M, K, N, per_col, gelu):
    """Long-K (K >= 1536, deep stage ring) GEMMs with every output row
    checked: ragged M / N / K tails, per-column scale and zero point, and the
    GELU epilogue; bit-exact (1e-5 after GELU)."""
    x = synth.normal((M, K), 1.0, 21)
    w = synth.int8_uniform((K, N), 22)
    ws = synth.uniform_f32((N,), 0.005, 0.02, 23) if per_col else np.array([0.01], np.float32)
    bias = synth.normal((N,), 0.02, 24)
    bz = synth.int8_uniform((N,), 25, -8, 8) if per_col else None
    pw = ops.prepare_weight(torch.from_numpy(w).to(DEV))
    bzt = None if bz is None else torch.from_numpy(bz).to(DEV)
    out, y, s, z = ops.dynamic_quant_linear(torch.from_numpy(x).to(DEV), pw,
                                            torch.from_numpy(ws).to(DEV),
                                            torch.from_numpy(bias).to(DEV), bzt, gelu=gelu)
    oy, os_, oz = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(y.cpu().numpy(), oy)
    acc = oracle.matmul_integer(oy, w, np.uint8(oz), bz, threads=oracle.max_threads())
    sc = np.float32(os_) * ws.astype(np.float32)
    ref = (oracle.cast_i32_f32(acc) * (sc if sc.size > 1 else sc[0]) + bias).astype(np.float32)
    got = out.cpu().numpy()
    if gelu:
        np.testing.assert_allclose(got, oracle.gelu(ref), rtol=0, atol=1e-5)
    else:
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
