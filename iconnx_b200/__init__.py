"""iconnx_b200: the int8 dynamic-quantization hot path of the iconnx ONNX
engine (DynamicQuantizeLinear -> MatMulInteger -> Cast -> Mul -> Add
[-> GELU]) as hand-written sm_100a CUDA kernels behind a C ABI
(include/iconnx_b200.h), with a host engine mirroring the reference's
GpuGraphExecutor API."""

from ._lib import IcxError, load as load_library  # noqa: F401

__all__ = ["IcxError", "load_library"]
