"""CPU-side checks of the product library: it loads without a GPU, exports
every symbol the C header declares, and validates arguments before launching
(the reference's GPU ops return CudaError::Kernel for the same inputs)."""
import ctypes

from iconnx_b200 import _lib


def test_library_exports_every_header_symbol():
    L = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n


def test_version_and_errors_without_gpu():
    L = _lib.load()
    assert b"sm_100a" in L.icx_version()
    # null outputs are rejected before any CUDA call
    rc = L.icx_dql_f32_u8(None, None, 0, None, None, None, None, 0, None, 0)
    assert rc == -1
    assert b"null" in L.icx_last_error()
    rc = L.icx_matmul_integer(None, None, 3, None, 1, 1, 1, 1, None, None, 0, None, None, 0)
    assert rc == -1 and b"Int8 or UInt8" in L.icx_last_error()
    rc = L.icx_dequantize_linear(None, None, 7, 1, 1, 1, None, 1, None, None)
    assert rc == -1 and b"dtype" in L.icx_last_error()


def test_workspace_queries():
    L = _lib.load()
    assert L.icx_dql_workspace_bytes(10) >= 8
    assert L.icx_dql_workspace_bytes(1 << 30) <= 148 * 8 * 8
    assert L.icx_matmul_integer_workspace_bytes(4, 768, 768) >= 768 * 768
