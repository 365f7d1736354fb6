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


@pytest.mark.parametrize("M,KN", [(128, 768), (1024, 1024), (8192, 4096)])
def test_config5_sweep_points_sampled(M, KN):
    x = synth.outlier_mix((M, KN), 3)
    _sampled_rows_check(x, synth.int8_uniform((KN, KN), 4), np.array([0.01], np.float32),
                        synth.normal((KN,), 0.02, 5), rows=min(M, 48))


def test_config4_linear_per_column_full_rows():
    """BERT-base Linear at config 4's M = 64 x 512, per-column w_scale and b_zp."""
    M, K, N = 32768, 768, 3072
    x = synth.normal((M, K), 1.0, 6)
    _sampled_rows_check(x, synth.int8_uniform((K, N), 7), synth.uniform_f32((N,), 0.005, 0.02, 8),
                        synth.normal((N,), 0.02, 9), bz=synth.int8_uniform((N,), 10, -8, 8))
