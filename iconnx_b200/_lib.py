"""ctypes loader for libiconnx_b200.so (the in-tree sm_100a build).

There is no fallback: if the shared library is missing or fails to load,
every op raises.  Declared prototypes mirror include/iconnx_b200.h.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.environ.get("ICONNX_B200_LIB") or os.path.join(HERE, "libiconnx_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "iconnx_b200.h")

ICX_OK = 0
ICX_MAX_MINMAX_PARTIALS = 1184
ICX_U8, ICX_S8, ICX_S32, ICX_F32, ICX_S64, ICX_BOOL = 0, 1, 2, 3, 4, 5

_vp, _sz, _i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int

# name -> (restype, argtypes)
PROTOTYPES = {
    "icx_last_error": (ctypes.c_char_p, []),
    "icx_version": (ctypes.c_char_p, []),
    "icx_device_status": (_i, [_i, _vp]),
    "icx_selftest_bounded_wait": (_i, [_vp, ctypes.c_uint64]),
    "icx_dql_workspace_bytes": (_sz, [_sz]),
    "icx_dql_f32_u8": (_i, [_vp, _vp, _sz, _vp, _vp, _vp, _vp, _sz, _vp, _sz]),
    "icx_prepare_b": (_i, [_vp, _vp, _i, _sz, _sz, _vp, _vp]),
    "icx_matmul_integer_workspace_bytes": (_sz, [_sz, _sz, _sz]),
    "icx_matmul_integer": (_i, [_vp, _vp, _i, _vp, _i, _sz, _sz, _sz, _vp, _vp, _i, _vp, _vp, _sz]),
    "icx_matmul_integer_prepared": (_i, [_vp, _vp, _i, _vp, _i, _vp, _sz, _sz, _sz, _vp, _vp, _i,
                                         _vp, _vp]),
    "icx_quant_linear": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _i, _vp, _i,
                              _vp, _i, _vp, _vp, _vp, _vp]),
    "icx_quant_linear_layernorm": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp, _i,
                                        _vp, _i, _vp, _vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp]),
    "icx_dql_f32_u8_noalloc": (_i, [_vp, _vp, _sz, _vp, _vp, _vp, _vp, _sz]),
    "icx_dql_quantize_f32_u8": (_i, [_vp, _vp, _sz, _vp, _i, _vp, _vp, _vp, _vp, _sz]),
    "icx_dequantize_linear": (_i, [_vp, _vp, _i, _sz, _sz, _sz, _vp, _sz, _vp, _vp]),
    "icx_matmul_integer_rowsum": (_i, [_vp, _vp, _i, _sz, _sz, _vp]),
    "icx_engine_create": (_vp, [_i]),
    "icx_engine_destroy": (None, [_vp]),
    "icx_engine_add_input": (_i, [_vp, ctypes.c_char_p, _i, _i, _vp]),
    "icx_engine_add_initializer": (_i, [_vp, ctypes.c_char_p, _i, _i, _vp, _vp]),
    "icx_engine_add_node": (_i, [_vp, ctypes.c_char_p, ctypes.c_char_p, _i, _vp, _i, _vp, _i, _vp]),
    "icx_engine_run": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "icx_engine_submit": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp]),
    "icx_engine_wait": (_i, [_vp, ctypes.c_int64]),
    "icx_nccl_unique_id": (_i, [_vp, _sz]),
    "icx_engine_set_global_dql": (_i, [_vp, _vp, _i, _i]),
    "icx_engine_abort_global_dql": (_i, [_vp]),
    "icx_engine_output_info": (_i, [_vp, ctypes.c_char_p, _vp, _vp, _vp]),
    "icx_engine_output_copy": (_i, [_vp, ctypes.c_char_p, _vp, _sz]),
    "icx_engine_plan": (ctypes.c_char_p, [_vp]),
    "icx_engine_set_cuda_graphs": (_i, [_vp, _i]),
    "icx_engine_kernel_launches": (_i, [_vp]),
    "icx_engine_replay": (_i, [_vp]),
    "icx_engine_profile": (ctypes.c_char_p, [_vp]),
    "icx_engine_stream": (_vp, [_vp]),
    "icx_engine_step_count": (_i, [_vp]),
    "icx_engine_step_info": (ctypes.c_char_p, [_vp, _i]),
    "icx_engine_run_step": (_i, [_vp, _i]),
    "icx_engine_value_info": (_i, [_vp, ctypes.c_char_p, _vp, _vp, _vp]),
    "icx_engine_value_copy": (_i, [_vp, ctypes.c_char_p, _vp, _sz]),
}

_lib = None


class IcxError(RuntimeError):
    """A C-ABI call returned a non-zero status (the CudaError::Kernel analogue)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(SO_PATH):
        raise ImportError(
            f"{SO_PATH} is missing: build it with `python -m iconnx_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(SO_PATH)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != ICX_OK:
        msg = load().icx_last_error().decode(errors="replace")
        raise IcxError(status, msg)


def header_symbols() -> list[str]:
    """Function names declared with ICX_API in include/iconnx_b200.h."""
    import re
    text = open(HEADER).read()
    return re.findall(r"ICX_API\s+[\w\s\*]+?\b(icx_\w+)\s*\(", text)
