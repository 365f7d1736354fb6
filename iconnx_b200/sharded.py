"""Batch-sharded multi-GPU inference: one executor per GPU.

The reference has no multi-GPU code and its GpuGraphExecutor is !Sync and
hard-wired to device 0 (src/cuda/context.rs:49-60).  Inference of the int8
encoder shards by batch with no cross-GPU exchange, so the B200 design is one
GpuGraphExecutor per device, each owned and driven by its own host thread, the
batch split along axis 0 and the outputs concatenated on the host.  No NCCL
collective is on the data path.

Per-shard dynamic quantisation takes its min/max over the shard, so a sharded
run equals, shard by shard, an independent executor on that sub-batch; it is
not bit-equal to a single executor over the whole batch.  With
``global_dql=True`` every DynamicQuantizeLinear takes (min, max) over all
shards through one 8-byte NCCL all-reduce (NVLink), and the sharded run is
bit-equal to one executor over the whole batch.

A failing shard raises in the caller; a shard that does not finish within
``timeout`` seconds raises TimeoutError without waiting for it.  Either way
the runner is then unusable (a stalled worker may still be driving its
executor, which is single-threaded), and with ``global_dql`` every
executor's communicator is aborted first, so that no all-reduce stays
waiting on a GPU for a shard that will not join.
"""

from __future__ import annotations

import threading
import time
from typing import Callable

import numpy as np


def shard_bounds(n: int, shards: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) rows per shard, sizes differing by at most 1."""
    base, extra = divmod(n, shards)
    out, s = [], 0
    for i in range(shards):
        e = s + base + (1 if i < extra else 0)
        out.append((s, e))
        s = e
    return out


class ShardedRunner:
    """Runs one graph on several devices, splitting every input along axis 0.

    ``build(builder, batch)`` adds the graph for `batch` rows to a builder and
    returns nothing; ``factory(device)`` returns an executor (default:
    GpuGraphExecutor on that CUDA device).  Each executor is created, built and
    run only on its own worker thread.
    """

    def __init__(self, build: Callable, devices: list, batch: int,
                 factory: Callable | None = None, global_dql: bool = False,
                 nccl_id: bytes | None = None):
        if factory is None:
            from .engine import GpuGraphExecutor
            factory = GpuGraphExecutor.new
        self.devices = list(devices)
        self.bounds = [b for b in shard_bounds(batch, len(self.devices))]
        self._build, self._factory = build, factory
        self._ex = [None] * len(self.devices)
        self._nccl_id = None
        self._broken = None
        if global_dql and len(self.devices) > 1:
            if any(e <= s for s, e in self.bounds):
                raise ValueError("global_dql needs at least one row per shard")
            if nccl_id is None:
                from .engine import nccl_unique_id
                nccl_id = nccl_unique_id()
            self._nccl_id = nccl_id

    def _ensure(self, i):
        if self._ex[i] is None:
            ex = self._factory(self.devices[i])
            s, e = self.bounds[i]
            self._build(ex, e - s)
            if self._nccl_id is not None:
                # collective set-up: every worker thread reaches this together
                ex.set_global_dql(self._nccl_id, len(self.devices), i)
            self._ex[i] = ex
        return self._ex[i]

    def _fail(self, why: str) -> None:
        """Marks the runner unusable and, with global_dql, aborts every
        executor's communicator so no all-reduce stays waiting for a peer."""
        self._broken = why
        if self._nccl_id is not None:
            for ex in self._ex:
                if ex is not None:
                    try:
                        ex.abort_collectives()
                    except Exception:  # already aborted / never joined
                        pass

    def run(self, inputs: dict, outputs, timeout: float | None = None) -> dict:
        if self._broken is not None:
            raise RuntimeError(f"ShardedRunner is unusable after a failed run ({self._broken}); "
                               "build a new one")
        n = len(self.devices)
        results: list = [None] * n
        errors: list = [None] * n

        def work(i):
            try:
                ex = self._ensure(i)
                s, e = self.bounds[i]
                results[i] = ex.run({k: v[s:e] for k, v in inputs.items()}, outputs)
            except BaseException as exc:  # propagated to the caller below
                errors[i] = exc

        threads = [threading.Thread(target=work, args=(i,), daemon=True) for i in range(n)
                   if self.bounds[i][1] > self.bounds[i][0]]
        for t in threads:
            t.start()
        deadline = None if timeout is None else time.monotonic() + timeout
        for t in threads:
            # one deadline for the whole run; a failed shard ends the wait
            # early, since with global_dql the others may wait on it forever
            while t.is_alive():
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    break
                t.join(0.05 if left is None else min(0.05, left))
                if any(e is not None for e in errors):
                    break
            if any(e is not None for e in errors):
                break
            if t.is_alive():
                self._fail("timeout")
                raise TimeoutError(f"a shard did not finish within {timeout} s")
        for i, err in enumerate(errors):
            if err is not None:
                self._fail(f"shard {i} failed")
                raise RuntimeError(f"shard {i} (device {self.devices[i]}) failed: {err}") from err
        return {o: np.concatenate([r[o] for r in results if r is not None], axis=0) for o in outputs}


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar over the default process group (timings are
    reported as the slowest rank); identity without torch.distributed."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
