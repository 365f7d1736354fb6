"""The allocation-free DynamicQuantizeLinear entry point.

icx_dql_f32_u8_noalloc serves callers that may not allocate device memory
while they run (a memory budget fixed at start-up, an allocator that cannot
be re-entered from the calling thread, a host that bans cudaMalloc because it
can synchronise the device).  It keeps its scratch in an array compiled into
the library.  These tests call it through the C ABI and check it, call after
call on the same array, against both the workspace-taking entry point and the
oracle restatement of the reference operator
(src/operators/dynamic_quantize_linear.rs:32-112): bit-exact u8 output,
scale, zero point and row sums.

This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

from iconnx_b200 import _lib, synth

NOALLOC_MAX_N = 1184 << 17   # ICX_DQL_NOALLOC_MAX_N


def test_noalloc_rejects_oversized_input_before_any_launch():
    L = _lib.load()
    rc = L.icx_dql_f32_u8_noalloc(None, None, NOALLOC_MAX_N + 1, None, None, None, None, 0)
    assert rc == -1  # ICX_ERR_INVALID
    assert b"exceeds the maximum" in L.icx_last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_and_oracle_call_after_call():
    import torch
    from oracle import oracle
    L = _lib.load()
    dev = "cuda:0"
    # large (1184 scratch pairs written), then mid-size (fewer pairs than the
    # previous call left in the array, different values), then small (one pair)
    cases = [(synth.normal((4096, 768), 1.0, 31), 768),
             (synth.outlier_mix((300, 768), 33) * np.float32(3.0), 768),
             (synth.outlier_mix((37, 20), 32), 20)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    for x_np, row_len in cases:
        x = torch.from_numpy(x_np).to(dev).reshape(-1)
        n = x.numel()
        ref = [torch.empty(n, dtype=torch.uint8, device=dev), torch.empty((), device=dev),
               torch.empty((), dtype=torch.uint8, device=dev),
               torch.empty(n // row_len, dtype=torch.int32, device=dev)]
        got = [torch.full((n,), 7, dtype=torch.uint8, device=dev), torch.empty((), device=dev),
               torch.empty((), dtype=torch.uint8, device=dev),
               torch.full((n // row_len,), -1, dtype=torch.int32, device=dev)]
        wsb = L.icx_dql_workspace_bytes(n)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = L.icx_dql_f32_u8(stream, x.data_ptr(), n, ref[0].data_ptr(), ref[1].data_ptr(),
                              ref[2].data_ptr(), ref[3].data_ptr(), row_len, ws.data_ptr(), wsb)
        assert rc == 0, L.icx_last_error()
        rc = L.icx_dql_f32_u8_noalloc(stream, x.data_ptr(), n, got[0].data_ptr(),
                                      got[1].data_ptr(), got[2].data_ptr(), got[3].data_ptr(),
                                      row_len)
        assert rc == 0, L.icx_last_error()
        torch.cuda.synchronize()
        for r, g in zip(ref, got):
            np.testing.assert_array_equal(g.cpu().numpy(), r.cpu().numpy())
        oy, os_, oz = oracle.dynamic_quantize_linear(x_np)
        np.testing.assert_array_equal(got[0].cpu().numpy(), oy.reshape(-1))
        assert got[1].item() == os_ and got[2].item() == oz
        np.testing.assert_array_equal(got[3].cpu().numpy(),
                                      oracle.rowsum_u8(oy.reshape(-1, row_len)))
