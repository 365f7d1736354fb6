"""ShardedRunner (batch-sharded independent executors) and the multi-rank
host logic of the benchmark, tested on CPU: fake executors that compute,
fail or stall, and a world_size-2 gloo group for the max-over-ranks timing."""
import os
import threading
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from iconnx_b200.sharded import ShardedRunner, max_over_ranks, shard_bounds
from oracle.graph_executor import CpuGraph


def test_shard_bounds_cover_batch():
    for n, k in [(32, 8), (33, 8), (5, 8), (1, 2), (64, 3)]:
        b = shard_bounds(n, k)
        assert len(b) == k and b[0][0] == 0 and b[-1][1] == n
        assert all(b[i][1] == b[i + 1][0] for i in range(k - 1))
        sizes = [e - s for s, e in b]
        assert max(sizes) - min(sizes) <= 1


def _linear(builder, batch):
    from iconnx_b200 import graphs
    graphs.build_ffn(builder, batch=batch, seq=4, hidden=32, ffn=64)


def test_sharded_equals_independent_executors_per_shard():
    from iconnx_b200 import synth
    x = synth.normal((6 * 4, 32), 1.0, 3)
    runner = ShardedRunner(_linear, devices=[0, 1, 2], batch=6, factory=lambda d: CpuGraph(threads=1))
    # inputs are [batch*seq, hidden]: shard rows by sequence
    runner.bounds = [(s * 4, e * 4) for s, e in shard_bounds(6, 3)]
    out = runner.run({"x": x}, ["y"])["y"]
    ref = []
    for s, e in runner.bounds:
        g = CpuGraph(threads=1)
        _linear(g, (e - s) // 4)
        ref.append(g.run({"x": x[s:e]}, ["y"])["y"])
    np.testing.assert_array_equal(out, np.concatenate(ref))


class _Failing:
    def __init__(self, dev):
        self.dev = dev

    def add_input(self, *a, **k):
        pass

    add_initializer = add_node = add_input

    def run(self, inputs, outputs):
        if self.dev == 1:
            raise RuntimeError("injected shard failure")
        return {o: np.zeros((len(next(iter(inputs.values()))), 1)) for o in outputs}


class _Stalling(_Failing):
    def run(self, inputs, outputs):
        if self.dev == 1:
            time.sleep(30)
        return super().run(inputs, outputs)


def test_one_shard_failure_propagates():
    r = ShardedRunner(lambda b, n: None, [0, 1, 2], 6, factory=_Failing)
    with pytest.raises(RuntimeError, match="shard 1"):
        r.run({"x": np.zeros((6, 2))}, ["y"])


def test_stalled_shard_times_out_without_hanging():
    r = ShardedRunner(lambda b, n: None, [0, 1], 4, factory=_Stalling)
    t0 = time.time()
    with pytest.raises(TimeoutError):
        r.run({"x": np.zeros((4, 2))}, ["y"], timeout=1.0)
    assert time.time() - t0 < 10


class _Collective(_Failing):
    """A fake executor in global-DQL mode: set_global_dql and abort_collectives
    are recorded; shard 1 fails before its plan runs, shard 2 stalls as an
    all-reduce would wait for the missing peer (until it is aborted)."""
    log: list = []

    def set_global_dql(self, nccl_id, nranks, rank):
        _Collective.log.append(("join", self.dev))
        self.aborted = threading.Event()

    def abort_collectives(self):
        _Collective.log.append(("abort", self.dev))
        self.aborted.set()

    def run(self, inputs, outputs):
        if self.dev == 1:
            raise RuntimeError("injected failure before the plan runs")
        if self.dev == 2:
            if not self.aborted.wait(20):
                raise AssertionError("never aborted")
            raise RuntimeError("all-reduce aborted")
        return super().run(inputs, outputs)


def test_global_dql_failure_aborts_every_shards_collectives():
    _Collective.log = []
    r = ShardedRunner(lambda b, n: None, [0, 1, 2], 6, factory=_Collective, global_dql=True,
                      nccl_id=b"\0" * 128)
    t0 = time.time()
    with pytest.raises(RuntimeError, match="shard 1"):
        r.run({"x": np.zeros((6, 2))}, ["y"], timeout=60)
    assert time.time() - t0 < 15          # the failure ends the wait, not the timeout
    aborted = {d for what, d in _Collective.log if what == "abort"}
    assert {0, 2} <= aborted               # every built executor's communicator
    with pytest.raises(RuntimeError, match="unusable"):
        r.run({"x": np.zeros((6, 2))}, ["y"])


def test_timeout_marks_runner_unusable():
    r = ShardedRunner(lambda b, n: None, [0, 1], 4, factory=_Stalling)
    with pytest.raises(TimeoutError):
        r.run({"x": np.zeros((4, 2))}, ["y"], timeout=0.5)
    with pytest.raises(RuntimeError, match="unusable"):
        r.run({"x": np.zeros((4, 2))}, ["y"])


def _rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q.put((rank, max_over_ranks(10.0 + rank)))
    dist.destroy_process_group()


def test_max_over_ranks_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
    assert res == {0: 11.0, 1: 11.0}


@pytest.mark.gpu
def test_sharded_on_gpus_matches_per_shard_executors():
    import torch
    from iconnx_b200 import graphs
    from iconnx_b200.engine import GpuGraphExecutor
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    cfg = graphs.BertConfig(layers=1, vocab=1000)
    build = lambda b, batch: graphs.build_bert(b, cfg, batch, 16)  # noqa: E731
    runner = ShardedRunner(build, list(range(n)), batch=2 * n)
    inp = graphs.bert_inputs(2 * n, 16, vocab=1000)
    out = runner.run(inp, ["last_hidden_state"], timeout=300)["last_hidden_state"]
    for i, (s, e) in enumerate(runner.bounds):
        ex = GpuGraphExecutor.new(i)
        build(ex, e - s)
        ref = ex.run({k: v[s:e] for k, v in inp.items()}, ["last_hidden_state"])["last_hidden_state"]
        np.testing.assert_array_equal(out[s:e], ref)


@pytest.mark.gpu
def test_global_dql_sharded_equals_full_batch():
    """global_dql: each DynamicQuantizeLinear takes (min, max) over all shards
    through an NCCL all-reduce, so the sharded encoder is bit-equal to one
    executor over the whole batch (every other op is per row)."""
    import torch
    from iconnx_b200 import graphs
    from iconnx_b200.engine import GpuGraphExecutor
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    cfg = graphs.BertConfig(layers=2, vocab=1000)
    build = lambda b, batch: graphs.build_bert(b, cfg, batch, 32)  # noqa: E731
    runner = ShardedRunner(build, list(range(n)), batch=2 * n, global_dql=True)
    inp = graphs.bert_inputs(2 * n, 32, vocab=1000)
    outs = [runner.run(inp, ["last_hidden_state"], timeout=300)["last_hidden_state"] for _ in range(3)]
    ex = GpuGraphExecutor.new(0)
    build(ex, 2 * n)
    ref = ex.run(inp, ["last_hidden_state"])["last_hidden_state"]
    for out in outs:   # eager, capture and replayed graph runs
        np.testing.assert_array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_global_dql_needs_rows_on_every_shard():
    with pytest.raises(ValueError):
        ShardedRunner(lambda b, n: None, [0, 1, 2], batch=2, factory=lambda d: None,
                      global_dql=True)
