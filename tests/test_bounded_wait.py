"""Failure handling of the kernels' bounded waits, without a GPU fault.

Every spin-wait in the tensor-core kernels (mbarrier phases fed by TMA, the
MMA warp or the epilogue) gives up after a wall-clock limit, records an
ICX_DEVICE_TIMEOUT_* code for icx_device_status and lets the kernel return.
icx_selftest_bounded_wait runs that wait on a barrier nothing arrives on,
with a 1 ms limit: the status must come back as ICX_DEVICE_TIMEOUT_SELFTEST
and the next kernels on the GPU must run normally.
"""
import ctypes

import numpy as np
import pytest

from iconnx_b200 import _lib, synth

TIMEOUT_SELFTEST = 0x1FF


def test_selftest_rejects_unbounded_limits():
    L = _lib.load()
    assert L.icx_selftest_bounded_wait(None, 0) == -1
    assert L.icx_selftest_bounded_wait(None, 10 ** 9) == -1
    assert b"outside" in L.icx_last_error()


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_stays_usable():
    import torch
    from iconnx_b200 import ops
    from oracle import oracle
    L = _lib.load()
    torch.cuda.init()
    status = ctypes.c_int(-1)
    assert L.icx_device_status(0, ctypes.byref(status)) == 0   # clear
    stream = torch.cuda.current_stream(0).cuda_stream
    assert L.icx_selftest_bounded_wait(stream, 1_000_000) == 0, L.icx_last_error()
    torch.cuda.synchronize()
    assert L.icx_device_status(0, ctypes.byref(status)) == 0
    assert status.value == TIMEOUT_SELFTEST
    assert L.icx_device_status(0, ctypes.byref(status)) == 0
    assert status.value == 0                                     # read clears it
    # the context still runs kernels: a DynamicQuantizeLinear, bit-exact
    x = synth.normal((64, 768), 1.0, 11)
    y, s, z = ops.gpu_dynamic_quantize_linear(torch.from_numpy(x).cuda())
    ry, rs, rz = oracle.dynamic_quantize_linear(x)
    np.testing.assert_array_equal(y.cpu().numpy(), ry)
    assert s.item() == rs and z.item() == rz
