"""Generate the golden fixtures under tests/golden/ from the reference tree.

The reference engine vendors the ONNX 1.18 backend node tests under
``tests/conformance_data/onnx-1.18/node/`` (it only parses them; its harness
never checks their outputs, tests/onnx_conformance.rs:198-227).  This script
decodes the ``input_*.pb`` / ``output_*.pb`` TensorProto files of the node
tests that cover the int8 dynamic-quantization chain and writes them as small
JSON fixtures, so the test suite can run where the reference tree is absent.

Run once where the reference is mounted:

    python tests/golden/make_golden.py /path/to/iconnx

The TensorProto wire format is decoded by hand (the ``onnx`` package is not
installed): field 1 dims, 2 data_type, 4 float_data, 5 int32_data,
7 int64_data, 8 name, 9 raw_data.
"""

from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

CASES = [
    "test_dynamicquantizelinear",
    "test_dynamicquantizelinear_max_adjusted",
    "test_dynamicquantizelinear_min_adjusted",
    "test_matmulinteger",
    "test_dequantizelinear",
    "test_dequantizelinear_axis",
    "test_erf",
    "test_gelu_default_1",
    "test_gelu_default_2",
    # the fp32 glue of the encoder (last-axis forms, the ones the reference's
    # single-axis LayerNormalization / Softmax implement)
    "test_layer_normalization_2d_axis_negative_1",
    "test_layer_normalization_3d_axis_negative_1_epsilon",
    "test_layer_normalization_4d_axis_negative_1",
    "test_softmax_axis_2",
    "test_softmax_default_axis",
    "test_softmax_example",
    "test_softmax_large_number",
    "test_softmax_negative_axis",
    "test_matmul_2d",
    "test_matmul_3d",
    "test_matmul_4d",
]

# ONNX TensorProto.DataType -> numpy dtype
DTYPES = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64}


def _varint(buf: bytes, i: int) -> tuple[int, int]:
    shift = 0
    out = 0
    while True:
        b = buf[i]
        i += 1
        out |= (b & 0x7F) << shift
        if not b & 0x80:
            return out, i
        shift += 7


def decode_tensor(buf: bytes) -> dict:
    dims: list[int] = []
    dtype = 0
    name = ""
    raw = None
    floats: list[float] = []
    ints: list[int] = []
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        field, wire = key >> 3, key & 7
        if wire == 0:
            v, i = _varint(buf, i)
            if field == 1:
                dims.append(v)
            elif field == 2:
                dtype = v
            elif field in (5, 7):
                ints.append(v)
        elif wire == 2:
            ln, i = _varint(buf, i)
            chunk = buf[i:i + ln]
            i += ln
            if field == 1:
                j = 0
                while j < len(chunk):
                    v, j = _varint(chunk, j)
                    dims.append(v)
            elif field == 4:
                floats.extend(struct.unpack(f"<{len(chunk) // 4}f", chunk))
            elif field in (5, 7):
                j = 0
                while j < len(chunk):
                    v, j = _varint(chunk, j)
                    ints.append(v)
            elif field == 8:
                name = chunk.decode()
            elif field == 9:
                raw = chunk
        elif wire == 5:
            i += 4
        elif wire == 1:
            i += 8
        else:
            raise ValueError(f"unsupported wire type {wire}")
    np_dtype = DTYPES[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np_dtype)
    elif floats:
        arr = np.array(floats, dtype=np_dtype)
    else:
        # int32_data carries u8/i8/i32 as (possibly sign-extended) varints
        vals = [(v - (1 << 64)) if v >= (1 << 63) else v for v in ints]
        arr = np.array(vals, dtype=np.int64).astype(np_dtype)
    arr = arr.reshape(dims) if dims else arr.reshape(())
    return {"name": name, "dtype": np.dtype(np_dtype).name,
            "shape": list(arr.shape), "data": _jsonable(arr)}


def _fields(buf: bytes):
    """(field, wire, value) of one protobuf message; length-delimited values
    as bytes, fixed32 as raw 4 bytes."""
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        field, wire = key >> 3, key & 7
        if wire == 0:
            v, i = _varint(buf, i)
        elif wire == 2:
            ln, i = _varint(buf, i)
            v = buf[i:i + ln]
            i += ln
        elif wire == 5:
            v = buf[i:i + 4]
            i += 4
        elif wire == 1:
            v = buf[i:i + 8]
            i += 8
        else:
            raise ValueError(f"unsupported wire type {wire}")
        yield field, wire, v


def decode_attributes(model: bytes) -> dict:
    """Scalar attributes (int / float) of the model's nodes: ModelProto.graph
    (7) -> GraphProto.node (1) -> NodeProto.attribute (5) -> AttributeProto
    name (1), f (2), i (3)."""
    out = {}
    for f7, _, graph in _fields(model):
        if f7 != 7:
            continue
        for f1, _, node in _fields(graph):
            if f1 != 1:
                continue
            for f5, _, attr in _fields(node):
                if f5 != 5:
                    continue
                name, val = None, None
                for fa, wa, v in _fields(attr):
                    if fa == 1:
                        name = v.decode()
                    elif fa == 2 and wa == 5:
                        val = struct.unpack("<f", v)[0]
                    elif fa == 3 and wa == 0:
                        val = v - (1 << 64) if v >= (1 << 63) else v
                if name is not None and val is not None:
                    out[name] = val
    return out


def _jsonable(arr: np.ndarray) -> list:
    if arr.dtype == np.float32:
        # store exact bit patterns so the fixtures are lossless
        return [int(v) for v in arr.reshape(-1).view(np.uint32)]
    return [int(v) for v in arr.reshape(-1)]


def main(ref_root: str) -> None:
    node_dir = os.path.join(ref_root, "tests", "conformance_data",
                            "onnx-1.18", "node")
    out_dir = os.path.dirname(os.path.abspath(__file__))
    for case in CASES:
        ds = os.path.join(node_dir, case, "test_data_set_0")
        entry = {"case": case, "source": f"tests/conformance_data/onnx-1.18/node/{case}",
                 "float_encoding": "uint32 bit patterns",
                 "inputs": [], "outputs": []}
        for kind in ("input", "output"):
            idx = 0
            while os.path.exists(os.path.join(ds, f"{kind}_{idx}.pb")):
                with open(os.path.join(ds, f"{kind}_{idx}.pb"), "rb") as f:
                    entry[kind + "s"].append(decode_tensor(f.read()))
                idx += 1
        with open(os.path.join(node_dir, case, "model.onnx"), "rb") as f:
            attrs = decode_attributes(f.read())
        if attrs:
            entry["attributes"] = attrs
        with open(os.path.join(out_dir, case + ".json"), "w") as f:
            json.dump(entry, f, indent=1)
        print(case, [t["shape"] for t in entry["inputs"]],
              [t["shape"] for t in entry["outputs"]])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <iconnx crate root>")
    main(sys.argv[1])
