"""ctypes binding of the CPU oracle (oracle.cpp) — TEST INFRASTRUCTURE ONLY.

Loaded by the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py``; the product package never imports this module.  Every
function mirrors one reference CPU operator (file:line cited in oracle.cpp).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or (
                os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "oracle.cpp"))):
            build()
        L = ctypes.CDLL(_SO)
        vp, sz, i32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_float
        L.oracle_dql.argtypes = [vp, sz, vp, vp, vp]
        L.oracle_rowsum_u8.argtypes = [vp, sz, sz, vp]
        L.oracle_matmul_integer.argtypes = [vp, ctypes.c_int, vp, ctypes.c_int, sz, sz, sz,
                                            i32, vp, ctypes.c_int, vp, ctypes.c_int]
        L.oracle_cast_i32_f32.argtypes = [vp, sz, vp]
        L.oracle_mul_scalar_vec.argtypes = [f32, vp, sz, vp]
        L.oracle_mul_rows.argtypes = [vp, sz, sz, vp, sz, vp]
        L.oracle_add_bias.argtypes = [vp, sz, sz, vp, vp]
        L.oracle_erf.argtypes = [vp, sz, vp]
        L.oracle_gelu.argtypes = [vp, sz, vp]
        L.oracle_dequantize_linear.argtypes = [vp, ctypes.c_int, sz, sz, sz, vp, sz, vp, vp]
        L.oracle_quant_linear.argtypes = [vp, sz, sz, vp, sz, vp, ctypes.c_int, vp, ctypes.c_int,
                                          vp, ctypes.c_int, vp, vp, vp, vp, vp, ctypes.c_int]
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_sum_f32.argtypes = [vp, sz]
        L.oracle_sum_f32.restype = ctypes.c_float
        L.oracle_layernorm.argtypes = [vp, sz, sz, vp, vp, f32, vp]
        L.oracle_softmax.argtypes = [vp, sz, sz, vp]
        L.oracle_matmul.argtypes = [vp, vp, sz, sz, sz, sz, sz, sz, vp]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def dynamic_quantize_linear(x: np.ndarray):
    """DynamicQuantizeLinear (dynamic_quantize_linear.rs:32-112) -> (y, scale, zp)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint8)
    s = np.zeros(1, dtype=np.float32)
    z = np.zeros(1, dtype=np.uint8)
    lib().oracle_dql(_p(x), x.size, _p(y), _p(s), _p(z))
    return y, np.float32(s[0]), np.uint8(z[0])


def rowsum_u8(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint8)
    M, K = a.shape
    out = np.empty(M, dtype=np.int32)
    lib().oracle_rowsum_u8(_p(a), M, K, _p(out))
    return out


def matmul_integer(a: np.ndarray, b: np.ndarray, a_zp=None, b_zp=None, threads: int = 1):
    """MatMulInteger (matmul_integer.rs:52-179, 239-267).

    a: u8/i8 [M, K] (rank 3 is flattened as the GPU arm does, layout.rs:1058-1090),
    b: u8/i8 [K, N]; a_zp scalar; b_zp scalar or per-column [N] (spec extension).
    """
    lead = a.shape[:-1]
    a2 = np.ascontiguousarray(a.reshape(-1, a.shape[-1]))
    b = np.ascontiguousarray(b)
    M, K = a2.shape
    K2, N = b.shape
    assert K == K2, "K mismatch"
    out = np.empty((M, N), dtype=np.int32)
    bz = None
    per_col = 0
    if b_zp is not None:
        bz = np.ascontiguousarray(np.atleast_1d(np.asarray(b_zp)).astype(np.int32))
        per_col = int(bz.size > 1)
    az = 0 if a_zp is None else int(np.asarray(a_zp).reshape(-1)[0])
    lib().oracle_matmul_integer(_p(a2), int(a2.dtype == np.int8), _p(b), int(b.dtype == np.int8),
                                M, K, N, az, _p(bz), per_col, _p(out), threads)
    return out.reshape(*lead, N)


def cast_i32_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int32)
    y = np.empty(x.shape, dtype=np.float32)
    lib().oracle_cast_i32_f32(_p(x), x.size, _p(y))
    return y


def erf(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_erf(_p(x), x.size, _p(y))
    return y


def gelu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_gelu(_p(x), x.size, _p(y))
    return y


def dequantize_linear(x: np.ndarray, scale: np.ndarray, zp=None, axis: int = 1) -> np.ndarray:
    """DequantizeLinear (dequantize_linear.rs:32-179)."""
    x = np.ascontiguousarray(x)
    scale = np.ascontiguousarray(np.asarray(scale, dtype=np.float32).reshape(-1))
    code = {np.dtype(np.int8): 0, np.dtype(np.uint8): 1, np.dtype(np.int32): 2}[x.dtype]
    if scale.size == 1:
        outer, axis_len, inner = 1, 1, x.size
    else:
        ax = axis + x.ndim if axis < 0 else axis
        outer = int(np.prod(x.shape[:ax]))
        axis_len = x.shape[ax]
        inner = int(np.prod(x.shape[ax + 1:]))
    zpa = None if zp is None else np.ascontiguousarray(np.asarray(zp, dtype=x.dtype).reshape(-1))
    y = np.empty(x.shape, dtype=np.float32)
    if x.size == 0:
        return y
    lib().oracle_dequantize_linear(_p(x), code, outer, axis_len, inner, _p(scale), scale.size,
                                   _p(zpa), _p(y))
    return y


def quant_linear(x: np.ndarray, w: np.ndarray, w_scale, bias: np.ndarray, b_zp=None,
                 gelu: bool = False, threads: int = 1):
    """The whole DQL -> MatMulInteger -> Cast -> Mul -> Add [-> GELU] chain.

    Returns (out f32 [M, N], q u8 [M, K], scale f32, zp u8, acc i32 [M, N]).
    """
    x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]), dtype=np.float32)
    M, K = x2.shape
    w = np.ascontiguousarray(w, dtype=np.int8)
    N = w.shape[1]
    ws = np.ascontiguousarray(np.atleast_1d(np.asarray(w_scale, dtype=np.float32)))
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    bz = None
    bz_pc = 0
    if b_zp is not None:
        bz = np.ascontiguousarray(np.atleast_1d(np.asarray(b_zp)).astype(np.int32))
        bz_pc = int(bz.size > 1)
    out = np.empty((M, N), dtype=np.float32)
    q = np.empty((M, K), dtype=np.uint8)
    s = np.zeros(1, dtype=np.float32)
    z = np.zeros(1, dtype=np.uint8)
    acc = np.empty((M, N), dtype=np.int32)
    lib().oracle_quant_linear(_p(x2), M, K, _p(w), N, _p(ws), int(ws.size > 1), _p(bz), bz_pc,
                              _p(bias), int(gelu), _p(out), _p(q), _p(s), _p(z), _p(acc), threads)
    return out, q, np.float32(s[0]), np.uint8(z[0]), acc


def sum_f32(x: np.ndarray) -> np.float32:
    """ndarray's unrolled eight-accumulator sum of a contiguous f32 lane."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    return np.float32(lib().oracle_sum_f32(_p(x), x.size))


def layer_normalization(x: np.ndarray, scale: np.ndarray, bias=None, epsilon: float = 1e-5):
    """LayerNormalization over the last axis (layer_normalization.rs:25-80)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    D = x.shape[-1]
    y = np.empty_like(x)
    sc = np.ascontiguousarray(scale, dtype=np.float32).reshape(-1)
    bi = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
    lib().oracle_layernorm(_p(x), x.size // D if D else 0, D, _p(sc), _p(bi),
                           ctypes.c_float(float(np.float32(epsilon))), _p(y))
    return y


def softmax(x: np.ndarray) -> np.ndarray:
    """Softmax over the last axis (softmax.rs:21-56)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    D = x.shape[-1]
    y = np.empty_like(x)
    lib().oracle_softmax(_p(x), x.size // D if D else 0, D, _p(y))
    return y


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """MatMul of rank >= 2 operands with equal or absent batch dimensions
    (matmul.rs:27-186, ndarray / matrixmultiply arithmetic)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    assert K == K2, "inner dimensions must match"
    ab, bb = a.shape[:-2], b.shape[:-2]
    if ab and bb and ab != bb:
        raise ValueError(f"batch dimensions must match: {ab} vs {bb}")
    out_batch = ab if ab else bb
    batch = int(np.prod(out_batch)) if out_batch else 1
    c = np.empty((*out_batch, M, N), dtype=np.float32)
    lib().oracle_matmul(_p(a), _p(b), batch, M, K, N, M * K if ab else 0, K * N if bb else 0, _p(c))
    return c


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def quant_linear_from_q(q: np.ndarray, a_scale, a_zp, w: np.ndarray, w_scale, bias=None,
                        b_zp=None, gelu: bool = False, residual: np.ndarray | None = None,
                        threads: int = 1) -> np.ndarray:
    """The Linear chain after DynamicQuantizeLinear, on its outputs:
    MatMulInteger(q, w, a_zp, b_zp) (matmul_integer.rs:239-267) -> Cast
    (cast.rs:46-48) -> Mul(., Mul(a_scale, w_scale)) (mul.rs:26-58) ->
    [Add(bias) (add.rs:27-85)] [-> GELU subgraph (erf.rs:30-40)]
    [-> Add(residual)], each op rounded on its own as the reference's CPU
    GraphExecutor runs them one node at a time.  q u8 [M, K]; returns f32 [M, N]."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    M = q.shape[0]
    N = w.shape[1]
    acc = matmul_integer(q, np.ascontiguousarray(w), np.uint8(a_zp), b_zp, threads=threads)
    c = cast_i32_f32(acc)
    ws = np.ascontiguousarray(np.atleast_1d(np.asarray(w_scale, dtype=np.float32)))
    s = np.empty(ws.size, dtype=np.float32)
    L = lib()
    L.oracle_mul_scalar_vec(ctypes.c_float(float(np.float32(a_scale))), _p(ws), ws.size, _p(s))
    o = np.empty((M, N), dtype=np.float32)
    L.oracle_mul_rows(_p(c), M, N, _p(s), s.size, _p(o))
    if bias is not None:
        b = np.ascontiguousarray(bias, dtype=np.float32)
        o2 = np.empty_like(o)
        L.oracle_add_bias(_p(o), M, N, _p(b), _p(o2))
        o = o2
    if gelu:
        o = globals()["gelu"](o)
    if residual is not None:
        o = np.add(o, np.ascontiguousarray(residual, dtype=np.float32), dtype=np.float32)
    return o
