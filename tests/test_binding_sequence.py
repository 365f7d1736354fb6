"""The reference-side binding's call sequence for per-op MatMulInteger, through
the C ABI exactly as a Rust maintainer would issue it:

* once, at weight upload (src/ir/lowering.rs:159 upload_initializers):
  icx_prepare_b(B) -> bt [N, K], colsum [N];
* per call of the MatMulInteger arm (src/cuda/executor/layout.rs:1034-1097):
  icx_matmul_integer_rowsum(A) when B has a zero point, then
  icx_matmul_integer_prepared(A, bt, colsum, a_zp, b_zp, rowsum).

Checked bit-exactly against the oracle restatement of
src/operators/matmul_integer.rs:239-267, with a per-column B zero point and
with the rank-3 activation flattened like layout.rs:1058-1090, over several
calls that reuse the one prepared weight.
"""
import numpy as np
import pytest

from iconnx_b200 import _lib

gpu = pytest.mark.gpu
U8, S8 = 0, 1


@gpu
@pytest.mark.parametrize("b_signed,per_col", [(True, True), (True, False), (False, True)])
def test_prepare_once_then_rowsum_and_prepared_per_call(b_signed, per_col):
    import torch
    from oracle import oracle
    L = _lib.load()
    dev = "cuda:0"
    rng = np.random.default_rng(7)
    K, N = 768, 3072 if per_col else 768
    bt_np = np.int8 if b_signed else np.uint8
    b = rng.integers(-127 if b_signed else 0, 128 if b_signed else 256, (K, N)).astype(bt_np)
    if per_col:
        bz = rng.integers(-8 if b_signed else 120, 9 if b_signed else 137, (N,)).astype(bt_np)
    else:
        bz = np.array([3 if b_signed else 131], dtype=bt_np)
    b_type = S8 if b_signed else U8
    stream = torch.cuda.current_stream(dev).cuda_stream
    d_b = torch.from_numpy(b).to(dev)
    d_bz = torch.from_numpy(bz).to(dev)
    # one-time preparation at weight upload
    d_bt = torch.empty(N * K, dtype=torch.uint8, device=dev)
    d_colsum = torch.empty(N, dtype=torch.int32, device=dev)
    assert L.icx_prepare_b(stream, d_b.data_ptr(), b_type, K, N, d_bt.data_ptr(),
                           d_colsum.data_ptr()) == 0, L.icx_last_error()
    del d_b  # the arm never reads the original layout again
    for call, (batch, M) in enumerate([(2, 64), (1, 4096), (4, 37)]):
        a = rng.integers(0, 256, (batch, M, K)).astype(np.uint8)
        a_zp = np.array([rng.integers(0, 256)], dtype=np.uint8)
        d_a = torch.from_numpy(a).to(dev)
        d_azp = torch.from_numpy(a_zp).to(dev)
        rows = batch * M
        d_rowsum = torch.empty(rows, dtype=torch.int32, device=dev)
        d_out = torch.empty((rows, N), dtype=torch.int32, device=dev)
        assert L.icx_matmul_integer_rowsum(stream, d_a.data_ptr(), U8, rows, K,
                                           d_rowsum.data_ptr()) == 0, L.icx_last_error()
        assert L.icx_matmul_integer_prepared(
            stream, d_a.data_ptr(), U8, d_bt.data_ptr(), b_type, d_colsum.data_ptr(), rows, K, N,
            d_azp.data_ptr(), d_bz.data_ptr(), int(per_col), d_rowsum.data_ptr(),
            d_out.data_ptr()) == 0, L.icx_last_error()
        torch.cuda.synchronize()
        ref = oracle.matmul_integer(a, b, a_zp[0], bz if per_col else bz[0], threads=8)
        np.testing.assert_array_equal(d_out.cpu().numpy().reshape(batch, M, N), ref,
                                      err_msg=f"call {call}")
