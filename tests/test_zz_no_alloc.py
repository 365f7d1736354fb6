"""The allocation-free DynamicQuantizeLinear entry point.

icx_dql_f32_u8_noalloc serves callers that may not allocate device memory
while they run (a memory budget fixed at start-up, an allocator that cannot
be re-entered from the calling thread, a host that bans cudaMalloc because it
can synchronise the device).  It keeps its scratch in an array compiled into
the library.  These tests call it through the C ABI and check that it gives
exactly what the workspace-taking entry point gives, on two calls in a row
(the second call reuses the array the first one left behind).

This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from iconnx_b200 import _lib, synth


def test_noalloc_rejects_oversized_input_before_any_launch():
    L = _lib.load()
    too_big = (1 << 32) + 1
    rc = L.icx_dql_f32_u8_noalloc(None, None, too_big, None, None, None, None, 0)
    assert rc == -1  # ICX_ERR_INVALID
    assert b"exceeds the maximum" in L.icx_last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    import torch
    L = _lib.load()
    dev = "cuda:0"
    cases = [(synth.normal((4096, 768), 1.0, 31), 768),     # large: many partials
             (synth.outlier_mix((37, 20), 32), 20)]          # small: one partial, odd rows
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
