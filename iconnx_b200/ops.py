"""Per-op GPU entry points over torch CUDA tensors, through the C ABI.

These mirror the reference's op wrappers (src/cuda/ops/quantize.rs):

* ``gpu_dynamic_quantize_linear(x)``      -> [y u8, scale f32 [], zp u8 []]   (:296)
* ``gpu_matmul_integer(a, b, a_zp, b_zp)`` -> s32                           (:398)
* ``gpu_dequantize_linear(x, scale, zp, axis)`` -> f32                      (:24)

plus the fused chain this build adds (``quant_linear``).  Errors are raised
as :class:`IcxError` (the reference returns ``CudaError::Kernel``), before any
launch.  torch only supplies device memory and the current stream; every
computation runs in libiconnx_b200.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ICX_S8, ICX_S32, ICX_U8, IcxError, check

_TYPE = {torch.uint8: ICX_U8, torch.int8: ICX_S8, torch.int32: ICX_S32}
_DT_NAME = {torch.float32: "Float32", torch.uint8: "UInt8", torch.int8: "Int8",
            torch.int32: "Int32", torch.int64: "Int64", torch.float16: "Float16"}


def _name(dt) -> str:
    return _DT_NAME.get(dt, str(dt))


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _cuda(t: torch.Tensor, what: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise IcxError(-1, f"{what}: expected a CUDA tensor")
    return t.contiguous()


def gpu_dynamic_quantize_linear(x: torch.Tensor, row_len: int | None = None):
    """DynamicQuantizeLinear (quantize.rs:296-377 / dynamic_quantize_linear.rs:32-112).

    Returns ``[y, y_scale, y_zero_point]``; with ``row_len`` also the per-row
    sums of y (s32 [numel / row_len]).
    """
    x = _cuda(x, "DynamicQuantizeLinear")
    if x.dtype != torch.float32:
        raise IcxError(-1, f"DynamicQuantizeLinear: input must be Float32, got {_name(x.dtype)}")
    L = _lib.load()
    n = x.numel()
    y = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    zp = torch.empty((), dtype=torch.uint8, device=x.device)
    rows = None
    if row_len is not None:
        rows = torch.empty(n // row_len if row_len else 0, dtype=torch.int32, device=x.device)
    wsb = L.icx_dql_workspace_bytes(n)
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    check(L.icx_dql_f32_u8(_stream(x), _ptr(x), n, _ptr(y), _ptr(scale), _ptr(zp), _ptr(rows),
                           row_len or 0, _ptr(ws), wsb))
    out = [y, scale, zp]
    if rows is not None:
        out.append(rows)
    return out


def _check_zp(zp, operand_dtype, label, allow_per_col: bool, n: int):
    if zp is None:
        return None, 0
    zp = _cuda(zp, "MatMulInteger")
    if zp.dtype != operand_dtype:
        raise IcxError(-1, f"MatMulInteger: {label}_zero_point dtype {_name(zp.dtype)} must match "
                           f"operand dtype {_name(operand_dtype)}")
    if zp.numel() == 1:
        return zp, 0
    if allow_per_col and zp.dim() == 1 and zp.numel() == n:
        return zp, 1
    raise IcxError(-3, f"MatMulInteger: {label}_zero_point must be scalar or per-column "
                       f"(got shape {list(zp.shape)})")


def gpu_matmul_integer(a: torch.Tensor, b: torch.Tensor, a_zero_point=None, b_zero_point=None):
    """MatMulInteger (quantize.rs:398-615), output Int32.

    a: u8/i8 [M, K] or [B, M, K] (flattened like layout.rs:1058-1090);
    b: u8/i8 [K, N]; a_zero_point scalar; b_zero_point scalar or [N].
    """
    a = _cuda(a, "MatMulInteger")
    b = _cuda(b, "MatMulInteger")
    if a.dtype not in (torch.uint8, torch.int8):
        raise IcxError(-1, f"MatMulInteger: input a must be Int8 or UInt8, got {_name(a.dtype)}")
    if b.dtype not in (torch.uint8, torch.int8):
        raise IcxError(-1, f"MatMulInteger: input b must be Int8 or UInt8, got {_name(b.dtype)}")
    if b.dim() != 2 or a.dim() not in (2, 3):
        raise IcxError(-1, f"MatMulInteger: unsupported ranks a={a.dim()} b={b.dim()}")
    lead = a.shape[:-1]
    K = a.shape[-1]
    if b.shape[0] != K:
        raise IcxError(-1, f"MatMulInteger: K mismatch — a is {list(a.shape)}, b is {list(b.shape)}")
    N = b.shape[1]
    M = a.numel() // K if K else int(torch.tensor(lead).prod()) if len(lead) else 1
    azp, _ = _check_zp(a_zero_point, a.dtype, "a", False, N)
    bzp, per_col = _check_zp(b_zero_point, b.dtype, "b", True, N)
    L = _lib.load()
    out = torch.empty((*lead, N), dtype=torch.int32, device=a.device)
    wsb = L.icx_matmul_integer_workspace_bytes(M, K, N)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=a.device)
    check(L.icx_matmul_integer(_stream(a), _ptr(a), _TYPE[a.dtype], _ptr(b), _TYPE[b.dtype], M, K, N,
                               _ptr(azp), _ptr(bzp), per_col, _ptr(out), _ptr(ws), wsb))
    return out


def gpu_dequantize_linear(x: torch.Tensor, scale: torch.Tensor, zero_point=None, axis: int = 1):
    """DequantizeLinear (quantize.rs:24-267 / dequantize_linear.rs:32-179)."""
    x = _cuda(x, "DequantizeLinear")
    scale = _cuda(scale, "DequantizeLinear")
    if x.dtype not in _TYPE:
        raise IcxError(-1, f"DequantizeLinear: input dtype {_name(x.dtype)} unsupported "
                           "(must be Int8, UInt8, or Int32)")
    if scale.dtype != torch.float32:
        raise IcxError(-1, f"DequantizeLinear: scale must be Float32, got {_name(scale.dtype)}")
    per_tensor = scale.dim() == 0 or scale.numel() == 1
    outer, axis_len, inner = 1, 1, x.numel()
    if not per_tensor:
        ax = axis + x.dim() if axis < 0 else axis
        if not 0 <= ax < x.dim():
            raise IcxError(-1, f"DequantizeLinear: axis {axis} out of range for ndim {x.dim()}")
        if scale.numel() != x.shape[ax]:
            raise IcxError(-1, f"DequantizeLinear: per-axis scale length {scale.numel()} doesn't "
                               f"match input shape[{ax}] = {x.shape[ax]}")
        outer = int(torch.tensor(x.shape[:ax]).prod()) if ax else 1
        axis_len = x.shape[ax]
        inner = int(torch.tensor(x.shape[ax + 1:]).prod()) if ax + 1 < x.dim() else 1
    if zero_point is not None:
        zero_point = _cuda(zero_point, "DequantizeLinear")
        if zero_point.dtype != x.dtype:
            raise IcxError(-1, f"DequantizeLinear: zero_point dtype {_name(zero_point.dtype)} must "
                               f"match input dtype {_name(x.dtype)}")
        if list(zero_point.shape) != list(scale.shape):
            raise IcxError(-1, f"DequantizeLinear: zero_point shape {list(zero_point.shape)} must "
                               f"match scale shape {list(scale.shape)}")
    y = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    L = _lib.load()
    check(L.icx_dequantize_linear(_stream(x), _ptr(x), _TYPE[x.dtype], outer, axis_len, inner,
                                  _ptr(scale), scale.numel(), _ptr(zero_point), _ptr(y)))
    return y


@dataclass
class PreparedWeight:
    """An int8 weight in the tensor-core layout: bt [N, K] plus column sums."""
    bt: torch.Tensor
    colsum: torch.Tensor
    K: int
    N: int
    dtype: torch.dtype


def prepare_weight(b: torch.Tensor) -> PreparedWeight:
    b = _cuda(b, "MatMulInteger")
    if b.dtype not in (torch.uint8, torch.int8) or b.dim() != 2:
        raise IcxError(-1, "MatMulInteger: weight must be a 2-D Int8/UInt8 tensor")
    K, N = b.shape
    bt = torch.empty((N, K), dtype=b.dtype, device=b.device)
    colsum = torch.empty(N, dtype=torch.int32, device=b.device)
    check(_lib.load().icx_prepare_b(_stream(b), _ptr(b), _TYPE[b.dtype], K, N, _ptr(bt), _ptr(colsum)))
    return PreparedWeight(bt, colsum, K, N, b.dtype)


class MinMaxPartials:
    """(min, max) partials of a tensor written by its producer kernel."""

    def __init__(self, device):
        self.buf = torch.empty((_lib.ICX_MAX_MINMAX_PARTIALS, 2), dtype=torch.float32, device=device)
        self.count = ctypes.c_int(0)

    @property
    def n(self) -> int:
        return int(self.count.value)


def quant_linear(q: torch.Tensor, a_scale: torch.Tensor, a_zp: torch.Tensor, w: PreparedWeight,
                 w_scale: torch.Tensor, bias: torch.Tensor | None = None,
                 b_zp: torch.Tensor | None = None, rowsum: torch.Tensor | None = None,
                 gelu: bool = False, out: torch.Tensor | None = None,
                 minmax: "MinMaxPartials | None" = None,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """Fused MatMulInteger -> Cast -> Mul(a_scale*w_scale) -> Add(bias) [-> GELU].

    With ``minmax`` the kernel also records (min, max) partials of the output
    for a following :func:`gpu_dynamic_quantize_from_partials`.
    """
    K = q.shape[-1]
    M = q.numel() // K
    if K != w.K or w.dtype != torch.int8:
        raise IcxError(-1, "QuantLinear: weight must be Int8 with matching K")
    if out is None:
        out = torch.empty((*q.shape[:-1], w.N), dtype=torch.float32, device=q.device)
    per_col_s = int(w_scale.numel() > 1)
    per_col_z = int(b_zp is not None and b_zp.numel() > 1)
    check(_lib.load().icx_quant_linear(
        _stream(q), _ptr(q), _ptr(a_scale), _ptr(a_zp), _ptr(rowsum), _ptr(w.bt), _ptr(w.colsum),
        M, K, w.N, _ptr(w_scale), per_col_s, _ptr(b_zp), per_col_z, _ptr(bias), int(gelu), _ptr(residual), _ptr(out),
        None if minmax is None else minmax.buf.data_ptr(),
        None if minmax is None else ctypes.byref(minmax.count)))
    return out


def quant_linear_layernorm(q: torch.Tensor, a_scale: torch.Tensor, a_zp: torch.Tensor,
                           w: PreparedWeight, w_scale: torch.Tensor, residual: torch.Tensor,
                           gamma: torch.Tensor, beta: torch.Tensor | None = None,
                           epsilon: float = 1e-5, bias: torch.Tensor | None = None,
                           b_zp: torch.Tensor | None = None, rowsum: torch.Tensor | None = None,
                           out: torch.Tensor | None = None,
                           minmax: "MinMaxPartials | None" = None) -> torch.Tensor:
    """LayerNormalization(QuantLinear(q) + residual) over the last axis in one
    launch (N = 192 x 2..4); the residual sum itself is not written."""
    K = q.shape[-1]
    M = q.numel() // K
    if K != w.K or w.dtype != torch.int8:
        raise IcxError(-1, "QuantLinear+LayerNorm: weight must be Int8 with matching K")
    if out is None:
        out = torch.empty((*q.shape[:-1], w.N), dtype=torch.float32, device=q.device)
    per_col_s = int(w_scale.numel() > 1)
    per_col_z = int(b_zp is not None and b_zp.numel() > 1)
    check(_lib.load().icx_quant_linear_layernorm(
        _stream(q), _ptr(q), _ptr(a_scale), _ptr(a_zp), _ptr(rowsum), _ptr(w.bt), _ptr(w.colsum),
        M, K, w.N, _ptr(w_scale), per_col_s, _ptr(b_zp), per_col_z, _ptr(bias), _ptr(residual),
        _ptr(gamma), _ptr(beta), float(epsilon), _ptr(out),
        None if minmax is None else minmax.buf.data_ptr(),
        None if minmax is None else ctypes.byref(minmax.count)))
    return out


def gpu_dynamic_quantize_from_partials(x: torch.Tensor, minmax: MinMaxPartials,
                                       row_len: int | None = None):
    """DynamicQuantizeLinear whose min/max scan was done by x's producer."""
    x = _cuda(x, "DynamicQuantizeLinear")
    if x.dtype != torch.float32:
        raise IcxError(-1, f"DynamicQuantizeLinear: input must be Float32, got {_name(x.dtype)}")
    n = x.numel()
    y = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    zp = torch.empty((), dtype=torch.uint8, device=x.device)
    rows = None
    if row_len is not None:
        rows = torch.empty(n // row_len, dtype=torch.int32, device=x.device)
    check(_lib.load().icx_dql_quantize_f32_u8(_stream(x), _ptr(x), n, minmax.buf.data_ptr(), minmax.n,
                                              _ptr(y), _ptr(scale), _ptr(zp), _ptr(rows), row_len or 0))
    out = [y, scale, zp]
    if rows is not None:
        out.append(rows)
    return out


def dynamic_quant_linear(x: torch.Tensor, w: PreparedWeight, w_scale: torch.Tensor,
                         bias: torch.Tensor | None = None, b_zp: torch.Tensor | None = None,
                         gelu: bool = False, x_minmax: MinMaxPartials | None = None,
                         out_minmax: MinMaxPartials | None = None):
    """DQL(x) followed by the fused quantised Linear; returns (out, y, scale, zp).

    ``x_minmax``: partials of x from its producer (skips the min/max pass);
    ``out_minmax``: collect partials of the output for the next DQL.
    """
    K = x.shape[-1]
    if x_minmax is not None:
        outs = gpu_dynamic_quantize_from_partials(x, x_minmax, row_len=K if b_zp is not None else None)
    else:
        outs = gpu_dynamic_quantize_linear(x, row_len=K if b_zp is not None else None)
    y, s, z = outs[:3]
    rows = outs[3] if b_zp is not None else None
    out = quant_linear(y, s, z, w, w_scale, bias, b_zp, rows, gelu, minmax=out_minmax)
    return out, y, s, z
