"""CPU graph interpreter — TEST INFRASTRUCTURE ONLY.

Restates the reference's legacy CPU GraphExecutor (src/graph_executor.rs:
92-278: topological order, DynamicQuantizeLinear as a multi-output node
:203-216, everything else through execute_operator :356-432).  The int8
operators and the fp32 glue that carries arithmetic (LayerNormalization,
Softmax, MatMul) come from the C++ oracle (oracle.cpp, each citing its
reference operator and restating its op order); element-wise Add / Sub /
Mul / Div are numpy float32 (one IEEE rounding per element, as ndarray's),
and Gather / Transpose / Reshape / Unsqueeze only move data.  The test suite
uses it as the checker of the GPU engine; the product never imports it.
"""

from __future__ import annotations

import numpy as np

from . import oracle

_ONNX2NP = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64, 9: np.bool_}


class CpuGraph:
    """Implements the same builder protocol as GpuGraphExecutor."""

    def __init__(self, threads: int = 8):
        self.inputs, self.inits, self.nodes = [], {}, []
        self.threads = threads

    def add_input(self, name, shape, dtype=np.float32):
        self.inputs.append(name)

    def add_initializer(self, name, array):
        self.inits[name] = np.ascontiguousarray(array)

    def add_node(self, name, op_type, inputs, outputs, attributes=None):
        self.nodes.append((name, op_type, list(inputs), list(outputs), dict(attributes or {})))

    def run(self, inputs: dict, outputs) -> dict:
        env = dict(self.inits)
        env.update({k: np.ascontiguousarray(v) for k, v in inputs.items()})
        pending = list(self.nodes)
        while pending:
            progressed = False
            for node in list(pending):
                name, op, ins, outs, attrs = node
                if all((i == "" or i in env) for i in ins):
                    vals = [env[i] if i else None for i in ins]
                    res = self._exec(op, vals, attrs)
                    for o, r in zip(outs, res):
                        env[o] = r
                    pending.remove(node)
                    progressed = True
            if not progressed:
                raise RuntimeError("graph has a cycle or missing input")
        return {o: env[o] for o in outputs}

    def _exec(self, op, v, a):
        f32 = np.float32
        if op == "DynamicQuantizeLinear":
            y, s, z = oracle.dynamic_quantize_linear(v[0])
            return [y, np.array(s, f32), np.array(z, np.uint8)]
        if op == "MatMulInteger":
            return [oracle.matmul_integer(v[0], v[1], v[2] if len(v) > 2 else None,
                                          v[3] if len(v) > 3 else None, threads=self.threads)]
        if op == "Cast":
            x = v[0]
            if x.dtype == np.int32 and a.get("to") == 1:
                return [oracle.cast_i32_f32(x)]
            return [x.astype(_ONNX2NP[a["to"]])]
        if op in ("Add", "Sub", "Mul", "Div"):
            x, y = v[0].astype(f32), v[1].astype(f32)
            fn = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.divide}[op]
            return [fn(x, y, dtype=f32)]
        if op == "Erf":
            return [oracle.erf(v[0])]
        if op == "DequantizeLinear":
            return [oracle.dequantize_linear(v[0], v[1], v[2] if len(v) > 2 else None, a.get("axis", 1))]
        if op == "Identity":
            return [v[0]]
        if op == "Gather":
            return [np.take(v[0], v[1], axis=0)]
        if op == "LayerNormalization":
            if a.get("axis", -1) not in (-1, v[0].ndim - 1):
                raise NotImplementedError("LayerNormalization over a non-last axis")
            bias = v[2] if len(v) > 2 else None
            return [oracle.layer_normalization(v[0], v[1], bias, a.get("epsilon", 1e-5))]
        if op == "Softmax":
            if a.get("axis", -1) not in (-1, v[0].ndim - 1):
                raise NotImplementedError("Softmax over a non-last axis")
            return [oracle.softmax(v[0])]
        if op == "MatMul":
            return [oracle.matmul(v[0], v[1])]
        if op == "Transpose":
            perm = a.get("perm")
            return [np.ascontiguousarray(np.transpose(v[0], perm))]
        if op == "Reshape":
            shape = [int(d) for d in v[1]]
            shape = [v[0].shape[i] if d == 0 else d for i, d in enumerate(shape)]
            return [v[0].reshape(shape)]
        if op == "Unsqueeze":
            x = v[0]
            for ax in sorted(a["axes"]):
                x = np.expand_dims(x, ax)
            return [x]
        raise NotImplementedError(op)
