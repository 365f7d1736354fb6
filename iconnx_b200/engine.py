"""GpuGraphExecutor: host-side mirror of the reference's public executor API
(src/cuda/inference/mod.rs:222-659) over the C++ engine in
libiconnx_b200.so (include/iconnx_b200.h, icx_engine_*).

    ex = GpuGraphExecutor.new()            # or GpuGraphExecutor.from_model(model)
    ex.add_input("x", [32, 128, 768])
    ex.add_initializer("W", np_int8_array)
    ex.add_node("n0", "DynamicQuantizeLinear", ["x"], ["q", "s", "z"])
    ...
    outs = ex.run({"x": x}, ["y"])         # host arrays in, host arrays out

As in the reference, lowering happens lazily on the first run; a run whose
input shape conflicts with a declared static dimension raises
``IcxError`` with status ICX_ERR_SHAPE_MISMATCH (the reference's
CudaError::InputShapeMismatch).  One executor per thread: the reference's is
``!Sync`` and so is this one.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import IcxError, check

_NP2ICX = {np.dtype(np.uint8): _lib.ICX_U8, np.dtype(np.int8): _lib.ICX_S8,
           np.dtype(np.int32): _lib.ICX_S32, np.dtype(np.float32): _lib.ICX_F32,
           np.dtype(np.int64): _lib.ICX_S64, np.dtype(np.bool_): _lib.ICX_BOOL}
_ICX2NP = {v: k for k, v in _NP2ICX.items()}
_DT_NAMES = {"float32": np.float32, "uint8": np.uint8, "int8": np.int8, "int32": np.int32,
             "int64": np.int64, "bool": np.bool_}


class _Attr(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("i", ctypes.c_int64),
                ("f", ctypes.c_float), ("ints", ctypes.POINTER(ctypes.c_int64)),
                ("floats", ctypes.POINTER(ctypes.c_float)), ("n", ctypes.c_int),
                ("s", ctypes.c_char_p)]


def _strs(items):
    arr = (ctypes.c_char_p * max(len(items), 1))()
    for i, s in enumerate(items):
        arr[i] = s.encode() if s else b""
    return arr


class GpuGraphExecutor:
    """One GPU graph executor (one CUDA stream on ``device``)."""

    def __init__(self, device: int = 0):
        L = _lib.load()
        self._L = L
        self._h = L.icx_engine_create(device)
        if not self._h:
            raise IcxError(-2, "icx_engine_create failed: " + L.icx_last_error().decode())
        self.device = device
        self._keep = []

    @classmethod
    def new(cls, device: int = 0) -> "GpuGraphExecutor":
        return cls(device)

    @classmethod
    def from_model(cls, model, device: int = 0) -> "GpuGraphExecutor":
        """Builds an executor from an OnnxModel (iconnx_b200.onnx.OnnxParser),
        like GpuGraphExecutor::from_model (src/cuda/inference/mod.rs:246-267)."""
        ex = cls(device)
        for name, (dtype, shape) in model.input_shapes().items():
            ex.add_input(name, shape, dtype)
        for name, arr in model.extract_weights().items():
            ex.add_initializer(name, arr)
        for i, node in enumerate(model.nodes):
            ex.add_node(node.name or f"n{i}", node.op_type, node.inputs, node.outputs, node.attrs)
        return ex

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.icx_engine_destroy(h)
            self._h = None

    # ------------------------------------------------------------- builder
    def add_input(self, name: str, shape, dtype=np.float32) -> None:
        dims = (ctypes.c_int64 * max(len(shape), 1))(*[int(d) if d is not None else -1 for d in shape])
        check(self._L.icx_engine_add_input(self._h, name.encode(), _NP2ICX[np.dtype(dtype)],
                                           len(shape), dims))

    def add_initializer(self, name: str, array) -> None:
        a = np.ascontiguousarray(array)
        if a.dtype not in _NP2ICX:
            raise IcxError(-1, f"add_initializer {name}: dtype {a.dtype} unsupported")
        dims = (ctypes.c_int64 * max(a.ndim, 1))(*a.shape)
        check(self._L.icx_engine_add_initializer(self._h, name.encode(), _NP2ICX[a.dtype], a.ndim,
                                                 dims, a.ctypes.data_as(ctypes.c_void_p)))

    def add_node(self, name: str, op_type: str, inputs, outputs, attributes=None) -> None:
        attrs = attributes or {}
        arr = (_Attr * max(len(attrs), 1))()
        keep = []
        for k, (key, v) in enumerate(attrs.items()):
            a = arr[k]
            a.name = key.encode()
            if isinstance(v, bool) or isinstance(v, (int, np.integer)):
                a.kind, a.i = 1, int(v)
            elif isinstance(v, (float, np.floating)):
                a.kind, a.f = 2, float(v)
            elif isinstance(v, str):
                a.kind, a.s = 4, v.encode()
            else:
                vals = list(v)
                if vals and isinstance(vals[0], (float, np.floating)):
                    buf = (ctypes.c_float * len(vals))(*vals)
                    a.kind, a.floats = 5, buf
                else:
                    buf = (ctypes.c_int64 * max(len(vals), 1))(*[int(x) for x in vals])
                    a.kind, a.ints = 3, buf
                a.n = len(vals)
                keep.append(buf)
        check(self._L.icx_engine_add_node(self._h, (name or "").encode(), op_type.encode(),
                                          len(inputs), _strs(inputs), len(outputs), _strs(outputs),
                                          len(attrs), arr))

    # ----------------------------------------------------------------- run
    def run(self, inputs: dict, outputs) -> dict:
        """Host arrays in, host arrays out (src/cuda/inference/mod.rs:428-464)."""
        self.run_device(inputs, outputs)
        return {name: self.fetch(name) for name in outputs}

    def run_device(self, inputs: dict, outputs) -> None:
        """Runs the graph; the outputs stay on the GPU until :meth:`fetch`."""
        names = list(inputs)
        arrs = [np.ascontiguousarray(inputs[n]) for n in names]
        for n, a in zip(names, arrs):
            if a.dtype not in _NP2ICX:
                raise IcxError(-1, f"run: input '{n}' dtype {a.dtype} unsupported")
        k = len(names)
        dtypes = (ctypes.c_int * max(k, 1))(*[_NP2ICX[a.dtype] for a in arrs])
        ranks = (ctypes.c_int * max(k, 1))(*[a.ndim for a in arrs])
        flat = [d for a in arrs for d in a.shape]
        dims = (ctypes.c_int64 * max(len(flat), 1))(*flat)
        ptrs = (ctypes.c_void_p * max(k, 1))(*[a.ctypes.data for a in arrs])
        self._inputs_alive = arrs
        check(self._L.icx_engine_run(self._h, k, _strs(names), dtypes, ranks, dims, ptrs,
                                     len(outputs), _strs(list(outputs))))

    def submit(self, inputs: dict, outputs, host_outs) -> int:
        """Pipelined run for serving loops: queues the inputs' upload, the
        plan and the download of ``outputs`` into the preallocated arrays
        ``host_outs`` (pinned memory lets the download overlap the next
        submission's compute) and returns a ticket without waiting.  The
        input and output arrays must stay alive until :meth:`wait`.  Two
        submissions can be in flight."""
        names = list(inputs)
        arrs = [np.ascontiguousarray(inputs[n]) for n in names]
        for n, a in zip(names, arrs):
            if a.dtype not in _NP2ICX:
                raise IcxError(-1, f"submit: input '{n}' dtype {a.dtype} unsupported")
        outs = list(outputs)
        if len(host_outs) != len(outs) or any(not h.flags.c_contiguous for h in host_outs):
            raise IcxError(-1, "submit: one contiguous host array per output")
        k = len(names)
        dtypes = (ctypes.c_int * max(k, 1))(*[_NP2ICX[a.dtype] for a in arrs])
        ranks = (ctypes.c_int * max(k, 1))(*[a.ndim for a in arrs])
        flat = [d for a in arrs for d in a.shape]
        dims = (ctypes.c_int64 * max(len(flat), 1))(*flat)
        ptrs = (ctypes.c_void_p * max(k, 1))(*[a.ctypes.data for a in arrs])
        optrs = (ctypes.c_void_p * max(len(outs), 1))(*[h.ctypes.data for h in host_outs])
        obytes = (ctypes.c_size_t * max(len(outs), 1))(*[h.nbytes for h in host_outs])
        ticket = ctypes.c_int64()
        check(self._L.icx_engine_submit(self._h, k, _strs(names), dtypes, ranks, dims, ptrs,
                                        len(outs), _strs(outs), optrs, obytes, ctypes.byref(ticket)))
        self._in_flight = getattr(self, "_in_flight", {})
        self._in_flight[ticket.value] = (arrs, list(host_outs))
        return ticket.value

    def wait(self, ticket: int) -> None:
        """Blocks until submission ``ticket`` has its outputs in its host arrays."""
        check(self._L.icx_engine_wait(self._h, int(ticket)))
        getattr(self, "_in_flight", {}).pop(int(ticket), None)

    def set_global_dql(self, nccl_id: bytes | None, nranks: int, rank: int) -> None:
        """Global DynamicQuantizeLinear across batch-sharded executors: every
        DQL takes (min, max) over all ``nranks`` executors through an 8-byte
        NCCL all-reduce, so the shards quantise exactly as one executor over
        the whole batch.  All ranks call this concurrently with the id from
        :func:`nccl_unique_id`; ``nranks <= 1`` turns it off."""
        buf = ctypes.create_string_buffer(bytes(nccl_id or b""), 128) if nccl_id else None
        check(self._L.icx_engine_set_global_dql(self._h, buf, int(nranks), int(rank)))

    def abort_collectives(self) -> None:
        """Aborts the global-DQL communicator (ncclCommAbort): all-reduces
        waiting for a peer that will not join return.  Callable from another
        thread while this executor's thread is blocked in :meth:`run`; later
        runs fail until :meth:`set_global_dql` is called again."""
        check(self._L.icx_engine_abort_global_dql(self._h))

    def fetch(self, name: str, out: np.ndarray | None = None) -> np.ndarray:
        dt, rk = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 6)()
        check(self._L.icx_engine_output_info(self._h, name.encode(), ctypes.byref(dt),
                                             ctypes.byref(rk), dims))
        shape = tuple(dims[i] for i in range(rk.value))
        if out is None:
            out = np.empty(shape, dtype=_ICX2NP[dt.value])
        check(self._L.icx_engine_output_copy(self._h, name.encode(), out.ctypes.data_as(ctypes.c_void_p),
                                             out.nbytes))
        return out

    # -------------------------------------------------------- introspection
    def plan(self) -> list[str]:
        """The compiled launch plan, one 'op node -> output' line per step."""
        return [ln for ln in self._L.icx_engine_plan(self._h).decode().splitlines() if ln]

    def run_with_profiling(self, inputs: dict, outputs) -> tuple[dict, list]:
        """Runs, then times every step of the plan with CUDA events (like the
        reference's run_with_profiling).  Returns (outputs, [(ms, op, node, out)])."""
        res = self.run(inputs, outputs)
        txt = self._L.icx_engine_profile(self._h)
        if txt is None:
            raise IcxError(-2, self._L.icx_last_error().decode())
        prof = []
        for ln in txt.decode().splitlines():
            ms, op, node, out = ln.split("\t")
            prof.append((float(ms), op, node, out))
        return res, prof

    @staticmethod
    def profile_summary(prof) -> str:
        """Per-op-type totals, like ProfileData::print_summary."""
        agg = {}
        for ms, op, _, _ in prof:
            t, c = agg.get(op, (0.0, 0))
            agg[op] = (t + ms, c + 1)
        total = sum(t for t, _ in agg.values()) or 1.0
        lines = [f"{t * 1e3:10.1f} us {100 * t / total:5.1f}% {c:4d}  {op}"
                 for op, (t, c) in sorted(agg.items(), key=lambda kv: -kv[1][0])]
        return "\n".join(lines + [f"total {total * 1e3:.1f} us"])

    def replay(self) -> None:
        """Re-run the compiled plan on the device-resident inputs of the last
        run (asynchronous, on :meth:`stream`)."""
        check(self._L.icx_engine_replay(self._h))

    def stream(self) -> int:
        """The executor's cudaStream_t as an integer handle."""
        return int(self._L.icx_engine_stream(self._h) or 0)

    def kernel_launches(self) -> int:
        return int(self._L.icx_engine_kernel_launches(self._h))

    # ------------------------------------------------ per-step debug access
    def steps(self) -> list[tuple[str, str, str, dict]]:
        """The compiled plan's steps as (op, node, output, info) where info
        maps the names of the values the step reads and writes (see
        icx_engine_step_info).  Empty before the first run."""
        out = []
        for i in range(int(self._L.icx_engine_step_count(self._h))):
            raw = self._L.icx_engine_step_info(self._h, i)
            if raw is None:
                raise IcxError(-1, self._L.icx_last_error().decode())
            op, node, o, info = raw.decode().split("\t", 3)
            kv = dict(item.split("=", 1) for item in info.split(";") if "=" in item)
            out.append((op, node, o, kv))
        return out

    def run_step(self, i: int) -> None:
        """Runs plan step ``i`` alone and waits for it (call in plan order,
        after a run, to re-execute the plan stage by stage)."""
        check(self._L.icx_engine_run_step(self._h, int(i)))

    def value(self, name: str) -> np.ndarray:
        """Current contents of any value the compiled plan materialises."""
        dt, rk = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 6)()
        check(self._L.icx_engine_value_info(self._h, name.encode(), ctypes.byref(dt),
                                            ctypes.byref(rk), dims))
        out = np.empty(tuple(dims[i] for i in range(rk.value)), dtype=_ICX2NP[dt.value])
        check(self._L.icx_engine_value_copy(self._h, name.encode(),
                                            out.ctypes.data_as(ctypes.c_void_p), out.nbytes))
        return out

    def set_cuda_graphs(self, enabled: bool) -> None:
        check(self._L.icx_engine_set_cuda_graphs(self._h, int(enabled)))


def nccl_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for :meth:`GpuGraphExecutor.set_global_dql`."""
    from . import _lib as L
    buf = ctypes.create_string_buffer(128)
    check(L.load().icx_nccl_unique_id(buf, 128))
    return buf.raw
