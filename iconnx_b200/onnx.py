"""Minimal ONNX model reader / writer (protobuf wire format, no `onnx` package).

``OnnxParser.parse_file(path) -> OnnxModel`` mirrors the reference's entry
point (src/onnx_parser.rs:138) with the accessors GpuGraphExecutor::from_model
uses: ``input_shapes()`` (:213), ``extract_weights()`` (:358, including INT8
and UINT8 initializers from raw_data / int32_data) and the node list
(``computation_graph`` :825).  Only what an int8 transformer graph needs is
decoded: ModelProto.graph with its nodes, initializers, inputs, outputs and
node attributes (int, float, string, ints, floats).

``save_model(path, builder)`` writes a graph recorded by :class:`GraphRecorder`
(the executor's builder protocol) as a .onnx file, so tests and users can
round-trip the synthetic configuration graphs through a real file.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# TensorProto.DataType <-> numpy
_ONNX2NP = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64, 9: np.bool_}
_NP2ONNX = {np.dtype(v): k for k, v in _ONNX2NP.items()}


# ---------------------------------------------------------------- decoding
def _varint(buf: bytes, i: int):
    shift = out = 0
    while True:
        b = buf[i]
        i += 1
        out |= (b & 0x7F) << shift
        if not b & 0x80:
            return out, i
        shift += 7


def _fields(buf: bytes):
    """Yields (field number, wire type, value) for a serialized message."""
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        f, w = key >> 3, key & 7
        if w == 0:
            v, i = _varint(buf, i)
        elif w == 1:
            v = buf[i:i + 8]
            i += 8
        elif w == 2:
            n, i = _varint(buf, i)
            v = buf[i:i + n]
            i += n
        elif w == 5:
            v = buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported protobuf wire type {w}")
        yield f, w, v


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _packed_varints(v, w):
    if w == 0:
        return [_signed(v)]
    out, j = [], 0
    while j < len(v):
        x, j = _varint(v, j)
        out.append(_signed(x))
    return out


def _tensor(buf: bytes):
    dims, dtype, name, raw, floats, ints = [], 1, "", None, [], []
    for f, w, v in _fields(buf):
        if f == 1:
            dims += _packed_varints(v, w)
        elif f == 2:
            dtype = v
        elif f == 4:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if w == 2 else [struct.unpack("<f", v)[0]]
        elif f in (5, 7):
            ints += _packed_varints(v, w)
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = bytes(v)
    if dtype not in _ONNX2NP:
        raise ValueError(f"tensor {name}: data type {dtype} unsupported")
    npdt = _ONNX2NP[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=npdt).copy()
    elif floats:
        arr = np.array(floats, dtype=npdt)
    else:
        arr = np.array(ints, dtype=np.int64).astype(npdt)
    return name, arr.reshape(dims) if dims else arr.reshape(())


def _attribute(buf: bytes):
    name, atype, val = "", 0, {}
    for f, w, v in _fields(buf):
        if f == 1:
            name = v.decode()
        elif f == 2:
            val["f"] = struct.unpack("<f", v)[0]
        elif f == 3:
            val["i"] = _signed(v)
        elif f == 4:
            val["s"] = bytes(v).decode(errors="replace")
        elif f == 7:
            val.setdefault("floats", []).extend(
                struct.unpack(f"<{len(v) // 4}f", v) if w == 2 else struct.unpack("<f", v))
        elif f == 8:
            val.setdefault("ints", []).extend(_packed_varints(v, w))
        elif f == 20:
            atype = v
    kind = {1: "f", 2: "i", 3: "s", 6: "floats", 7: "ints"}.get(atype)
    if kind is None:
        kind = next(iter(val), "i")
    return name, val.get(kind, [] if kind in ("floats", "ints") else 0)


def _value_info(buf: bytes):
    name, elem, shape = "", 1, []
    for f, _, v in _fields(buf):
        if f == 1:
            name = v.decode()
        elif f == 2:  # TypeProto
            for f2, _, v2 in _fields(v):
                if f2 == 1:  # tensor_type
                    for f3, _, v3 in _fields(v2):
                        if f3 == 1:
                            elem = v3
                        elif f3 == 2:  # TensorShapeProto
                            for f4, _, v4 in _fields(v3):
                                if f4 == 1:
                                    d = -1
                                    for f5, _, v5 in _fields(v4):
                                        if f5 == 1:
                                            d = _signed(v5)
                                    shape.append(d)
    return name, _ONNX2NP.get(elem, np.float32), shape


@dataclass
class OnnxNode:
    name: str
    op_type: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


@dataclass
class OnnxModel:
    nodes: list
    initializers: dict
    inputs: list          # (name, dtype, shape) excluding initializers
    outputs: list

    def input_shapes(self) -> dict:
        """name -> (dtype, shape) of the graph inputs (-1 = dynamic dim)."""
        return {n: (dt, shape) for n, dt, shape in self.inputs}

    def extract_weights(self) -> dict:
        return dict(self.initializers)

    def output_names(self) -> list:
        return list(self.outputs)


class OnnxParser:
    @staticmethod
    def parse_file(path) -> OnnxModel:
        with open(path, "rb") as f:
            return OnnxParser.parse_bytes(f.read())

    @staticmethod
    def parse_bytes(data: bytes) -> OnnxModel:
        graph = None
        for f, _, v in _fields(data):
            if f == 7:
                graph = v
        if graph is None:
            raise ValueError("ModelProto has no graph")
        nodes, inits, ins, outs = [], {}, [], []
        for f, _, v in _fields(graph):
            if f == 1:
                name, op, i_, o_, attrs = "", "", [], [], {}
                for f2, _, v2 in _fields(v):
                    if f2 == 1:
                        i_.append(v2.decode())
                    elif f2 == 2:
                        o_.append(v2.decode())
                    elif f2 == 3:
                        name = v2.decode()
                    elif f2 == 4:
                        op = v2.decode()
                    elif f2 == 5:
                        k, val = _attribute(v2)
                        attrs[k] = val
                nodes.append(OnnxNode(name, op, i_, o_, attrs))
            elif f == 5:
                n, arr = _tensor(v)
                inits[n] = arr
            elif f == 11:
                ins.append(_value_info(v))
            elif f == 12:
                outs.append(_value_info(v)[0])
        ins = [t for t in ins if t[0] not in inits]
        return OnnxModel(nodes, inits, ins, outs)


# ---------------------------------------------------------------- encoding
def _key(f, w):
    return _enc_varint((f << 3) | w)


def _enc_varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _ld(f, payload: bytes) -> bytes:
    return _key(f, 2) + _enc_varint(len(payload)) + payload


def _enc_tensor(name, arr) -> bytes:
    a = np.ascontiguousarray(arr)
    body = b"".join(_key(1, 0) + _enc_varint(d) for d in a.shape)
    body += _key(2, 0) + _enc_varint(_NP2ONNX[a.dtype])
    body += _ld(8, name.encode()) + _ld(9, a.tobytes())
    return body


def _enc_value_info(name, dtype, shape) -> bytes:
    dims = b"".join(_ld(1, (_key(1, 0) + _enc_varint(d)) if d is not None and d >= 0
                         else _ld(2, b"dyn")) for d in shape)
    tensor = _key(1, 0) + _enc_varint(_NP2ONNX[np.dtype(dtype)]) + _ld(2, dims)
    return _ld(1, name.encode()) + _ld(2, _ld(1, tensor))


def _enc_attr(name, v) -> bytes:
    body = _ld(1, name.encode())
    if isinstance(v, (bool, int, np.integer)):
        body += _key(3, 0) + _enc_varint(int(v)) + _key(20, 0) + _enc_varint(2)
    elif isinstance(v, (float, np.floating)):
        body += _key(2, 5) + struct.pack("<f", float(v)) + _key(20, 0) + _enc_varint(1)
    elif isinstance(v, str):
        body += _ld(4, v.encode()) + _key(20, 0) + _enc_varint(3)
    else:
        vals = list(v)
        if vals and isinstance(vals[0], (float, np.floating)):
            body += _ld(7, struct.pack(f"<{len(vals)}f", *vals)) + _key(20, 0) + _enc_varint(6)
        else:
            body += _ld(8, b"".join(_enc_varint(int(x)) for x in vals)) + _key(20, 0) + _enc_varint(7)
    return body


class GraphRecorder:
    """Records builder calls (add_input / add_initializer / add_node)."""

    def __init__(self):
        self.inputs, self.inits, self.nodes, self.outputs = [], {}, [], []

    def add_input(self, name, shape, dtype=np.float32):
        self.inputs.append((name, np.dtype(dtype), list(shape)))

    def add_initializer(self, name, array):
        self.inits[name] = np.ascontiguousarray(array)

    def add_node(self, name, op_type, inputs, outputs, attributes=None):
        self.nodes.append(OnnxNode(name, op_type, list(inputs), list(outputs), dict(attributes or {})))


def save_model(path, rec: GraphRecorder, outputs, opset: int = 17) -> None:
    g = b""
    for n in rec.nodes:
        body = b"".join(_ld(1, i.encode()) for i in n.inputs)
        body += b"".join(_ld(2, o.encode()) for o in n.outputs)
        body += _ld(3, n.name.encode()) + _ld(4, n.op_type.encode())
        body += b"".join(_ld(5, _enc_attr(k, v)) for k, v in n.attrs.items())
        g += _ld(1, body)
    g += _ld(2, b"iconnx_b200")
    for name, arr in rec.inits.items():
        g += _ld(5, _enc_tensor(name, arr))
    for name, dt, shape in rec.inputs:
        g += _ld(11, _enc_value_info(name, dt, shape))
    for o in outputs:
        g += _ld(12, _enc_value_info(o, np.float32, []))
    model = _key(1, 0) + _enc_varint(8) + _ld(8, _key(2, 0) + _enc_varint(opset)) + _ld(7, g)
    with open(path, "wb") as f:
        f.write(model)
