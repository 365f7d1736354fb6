"""The graph executor (GpuGraphExecutor over the C++ engine) against the CPU
graph interpreter restating the reference's CPU GraphExecutor
(src/graph_executor.rs:92-278), on the synthetic configuration graphs.

int8 chains: bit-exact (u8/s32 and the dequantised f32); after erf-GELU
1e-5; whole encoders (fp32 LayerNorm / softmax / attention GEMMs round
differently on the GPU, which can move a quantised value by one step):
5e-2 absolute on the LayerNorm-normalised hidden states.
"""
import numpy as np
import pytest

from iconnx_b200 import IcxError, graphs, synth
from oracle.graph_executor import CpuGraph

gpu = pytest.mark.gpu


def both(build, *args, **kw):
    from iconnx_b200.engine import GpuGraphExecutor
    ex, cpu = GpuGraphExecutor.new(), CpuGraph()
    out = build(ex, *args, **kw)
    build(cpu, *args, **kw)
    return ex, cpu, out


def test_cpu_interpreter_runs_config1_chain():
    cpu = CpuGraph()
    out = graphs.build_linear(cpu, M=8, K=32, N=16)
    x = synth.normal((1, 8, 32), 1.0, 0)
    y = cpu.run({"x": x}, [out])[out]
    assert y.shape == (1, 8, 16) and y.dtype == np.float32


def test_engine_create_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from iconnx_b200.engine import GpuGraphExecutor
    with pytest.raises(IcxError):
        GpuGraphExecutor.new()


@gpu
def test_config1_linear_bit_exact_and_fused():
    ex, cpu, out = both(graphs.build_linear)
    x = synth.normal((1, 128, 768), 1.0, 0)
    g = ex.run({"x": x}, [out])[out]
    r = cpu.run({"x": x}, [out])[out]
    np.testing.assert_array_equal(g.view(np.uint32), r.view(np.uint32))
    plan = ex.plan()
    assert any(s.startswith("QuantLinear ") for s in plan)
    assert not any(s.startswith(("MatMulInteger", "Cast", "Mul", "Add")) for s in plan)
    # second run replays the captured CUDA graph
    g2 = ex.run({"x": x}, [out])[out]
    np.testing.assert_array_equal(g2, g)


@gpu
def test_config2_ffn_block():
    ex, cpu, out = both(graphs.build_ffn, batch=2, seq=128)
    x = synth.normal((256, 768), 1.0, 0)
    g = ex.run({"x": x}, [out])[out]
    r = cpu.run({"x": x}, [out])[out]
    plan = ex.plan()
    assert any(s.startswith("QuantLinear+GELU") for s in plan)
    assert any(s.startswith("DynamicQuantizeLinear(quantise)") for s in plan)
    np.testing.assert_allclose(g, r, atol=2e-3, rtol=1e-4)


@gpu
def test_unfused_per_op_dispatch_bit_exact():
    """MatMulInteger / DequantizeLinear reached through the per-op dispatch
    (u8 weights with zero points, rank-3 activations), like layout.rs:978-1097."""
    def build(g):
        g.add_input("a", [2, 16, 64], np.uint8)
        g.add_initializer("b", np.random.default_rng(0).integers(0, 256, (64, 40), dtype=np.uint8))
        g.add_initializer("az", np.array(7, np.uint8))
        g.add_initializer("bz", np.array(130, np.uint8))
        g.add_initializer("sc", np.array(0.02, np.float32))
        g.add_node("mmi", "MatMulInteger", ["a", "b", "az", "bz"], ["acc"])
        g.add_node("deq", "DequantizeLinear", ["acc", "sc"], ["y"])
        return "y"
    ex, cpu, out = both(build)
    a = np.random.default_rng(1).integers(0, 256, (2, 16, 64), dtype=np.uint8)
    g = ex.run({"a": a}, [out, "acc"])
    r = cpu.run({"a": a}, [out, "acc"])
    np.testing.assert_array_equal(g["acc"], r["acc"])
    np.testing.assert_array_equal(g[out], r[out])


@gpu
def test_shape_guard_and_dtype_errors():
    from iconnx_b200.engine import GpuGraphExecutor
    ex = GpuGraphExecutor.new()
    out = graphs.build_linear(ex)
    with pytest.raises(IcxError, match="InputShapeMismatch"):
        ex.run({"x": np.zeros((1, 64, 768), np.float32)}, [out])
    with pytest.raises(IcxError, match="dtype"):
        ex.run({"x": np.zeros((1, 128, 768), np.int32)}, [out])


@gpu
@pytest.mark.parametrize("cfg,batch,seq", [
    (graphs.BertConfig(layers=2, w_scale=graphs.REALISTIC_W_SCALE), 2, 16),
    (graphs.BertConfig(layers=1, per_channel=True, token_type=True,
                       w_scale=graphs.REALISTIC_W_SCALE), 2, 32),
])
def test_encoder_matches_cpu_interpreter(cfg, batch, seq):
    ex, cpu, out = both(graphs.build_bert, cfg, batch, seq)
    inp = graphs.bert_inputs(batch, seq)
    g = ex.run(inp, [out])[out]
    r = cpu.run(inp, [out])[out]
    assert g.shape == (batch, seq, cfg.hidden)
    np.testing.assert_allclose(g, r, atol=5e-2)
    assert np.mean(np.abs(g - r) > 1e-3) < 0.05  # quantisation-boundary flips
    plan = ex.plan()
    fused = [s for s in plan if s.startswith("QuantLinear")]
    assert len(fused) == 4 * cfg.layers          # Q/K/V share one merged GEMM
    assert len([s for s in plan if s.startswith("QuantLinear(QKV)")]) == cfg.layers
    assert len([s for s in plan if s.startswith("Attention ")]) == cfg.layers
    assert not any(s.startswith(("Transpose", "Softmax", "MatMul ")) for s in plan)
    assert len([s for s in plan if s.startswith("QuantLinear+Residual")]) == 2 * cfg.layers


@gpu
@pytest.mark.parametrize("cfg", [graphs.BertConfig(layers=1),
                                 graphs.BertConfig(layers=1, per_channel=True, token_type=True)])
def test_encoder_at_config_weight_scale(cfg):
    """The configs' own weight scale (0.01, per-channel [0.005, 0.02]): scores
    of order 10^3 make softmax nearly one-hot, and where two keys nearly tie,
    any fp32 reordering of the score sums (this tensor-core attention, the
    reference's cuBLAS path, numpy) moves the context by ~1e-3, which can
    push a requantised value across a u8 boundary in that token's row.  So:
    every row matches to 5e-2 except at most 10% of the rows, and the median
    row agrees to 1e-4."""
    ex, cpu, out = both(graphs.build_bert, cfg, 2, 32)
    inp = graphs.bert_inputs(2, 32)
    g = ex.run(inp, [out])[out]
    r = cpu.run(inp, [out])[out]
    row_err = np.abs(g - r).max(axis=-1)
    assert np.mean(row_err > 5e-2) <= 0.1, row_err
    assert np.median(row_err) < 1e-4, np.median(row_err)


@gpu
def test_cuda_graph_replay_equals_eager():
    from iconnx_b200.engine import GpuGraphExecutor
    cfg = graphs.BertConfig(layers=1)
    inp = graphs.bert_inputs(2, 16)
    outs = []
    for graphs_on in (True, False):
        ex = GpuGraphExecutor.new()
        out = graphs.build_bert(ex, cfg, 2, 16)
        ex.set_cuda_graphs(graphs_on)
        for _ in range(3):
            outs.append(ex.run(inp, [out])[out])
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])


@gpu
def test_replay_rereads_last_inputs():
    """replay() re-executes the plan on the inputs of the last run: graph
    inputs must not share arena space with intermediates."""
    from iconnx_b200.engine import GpuGraphExecutor
    import torch
    cfg = graphs.BertConfig(layers=2)
    ex = GpuGraphExecutor.new()
    out = graphs.build_bert(ex, cfg, 4, 32)
    inp = graphs.bert_inputs(4, 32)
    ref = ex.run(inp, [out])[out]
    for _ in range(3):
        ex.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ex.fetch(out), ref)
    np.testing.assert_array_equal(ex.run(inp, [out])[out], ref)


def test_quantized_export_layout_on_cpu_interpreter():
    """The export layout runs through the CPU interpreter (u8 Gather,
    DequantizeLinear, Transpose of u8 weights, u8 weight zero points)."""
    cpu = CpuGraph()
    e, h, y = graphs.build_quantized_export(cpu, batch=1, seq=8, hidden=128, ffn=256)
    out = cpu.run({"input_ids": synth.token_ids((1, 8), 6, 1000)}, [e, h, y])
    assert out[e].dtype == np.float32 and out[y].shape == (1, 8, 128)


@gpu
def test_quantized_export_layout_fuses_and_matches():
    """u8 embedding Gather + DequantizeLinear (bit-exact), Transpose of the u8
    `_transposed_quantized` weights folded at compile, u8 weights with scalar
    and per-column u8 zero points converted exactly to s8 (w ^ 0x80, z ^ 0x80)
    and run as fused QuantLinears: FFN1+GELU within 1e-5 of the interpreter,
    FFN2 within the bound of test_config2_ffn_block."""
    ex, cpu, outs = both(graphs.build_quantized_export, batch=2, seq=64)
    e, h, y = outs
    inp = {"input_ids": synth.token_ids((2, 64), 6, 1000)}
    g = ex.run(inp, list(outs))
    r = cpu.run(inp, list(outs))
    np.testing.assert_array_equal(g[e].view(np.uint32), r[e].view(np.uint32))
    np.testing.assert_allclose(g[h], r[h], atol=1e-5, rtol=0)
    np.testing.assert_allclose(g[y], r[y], atol=2e-3, rtol=1e-4)
    plan = ex.plan()
    assert len([s for s in plan if s.startswith("QuantLinear")]) == 2, plan
    assert not any(s.startswith("Transpose") for s in plan), plan


@gpu
def test_quantized_export_through_onnx_file(tmp_path):
    """The same graph written as a .onnx file and loaded with
    OnnxParser.parse_file / GpuGraphExecutor.from_model."""
    from iconnx_b200.engine import GpuGraphExecutor
    from iconnx_b200.onnx import GraphRecorder, OnnxParser, save_model
    rec = GraphRecorder()
    outs = graphs.build_quantized_export(rec, batch=2, seq=16, hidden=128, ffn=256)
    path = tmp_path / "export.onnx"
    save_model(path, rec, list(outs))
    ex = GpuGraphExecutor.from_model(OnnxParser.parse_file(path))
    cpu = CpuGraph()
    graphs.build_quantized_export(cpu, batch=2, seq=16, hidden=128, ffn=256)
    inp = {"input_ids": synth.token_ids((2, 16), 7, 1000)}
    g = ex.run(inp, list(outs))
    r = cpu.run(inp, list(outs))
    np.testing.assert_array_equal(g[outs[0]].view(np.uint32), r[outs[0]].view(np.uint32))
    np.testing.assert_allclose(g[outs[1]], r[outs[1]], atol=1e-5, rtol=0)


@gpu
def test_submit_wait_pipeline_equals_run():
    """submit / wait (two submissions in flight, outputs downloaded into host
    arrays on a second stream) gives exactly what run() gives, per submission,
    including when a third submission reuses the first one's staging set."""
    from iconnx_b200.engine import GpuGraphExecutor
    cfg = graphs.BertConfig(layers=1, vocab=1000, w_scale=graphs.REALISTIC_W_SCALE)
    ex = GpuGraphExecutor.new()
    out = graphs.build_bert(ex, cfg, 2, 16)
    batches = [graphs.bert_inputs(2, 16, vocab=1000, seed=s) for s in (3, 4, 5, 6)]
    ref = [ex.run(b, [out])[out].copy() for b in batches]
    hosts = [np.empty_like(ref[0]) for _ in batches]
    tickets = []
    for b, h in zip(batches, hosts):
        tickets.append(ex.submit(b, [out], [h]))
        if len(tickets) == 2:
            ex.wait(tickets.pop(0))
    for t in tickets:
        ex.wait(t)
    for h, r in zip(hosts, ref):
        np.testing.assert_array_equal(h.view(np.uint32), r.view(np.uint32))


@gpu
@pytest.mark.parametrize("rows,D,eps", [(4096, 768, 1e-12), (37, 768, 1e-5), (256, 100, 0.1)])
def test_layernorm_matches_the_reference_operator(rows, D, eps):
    """LayerNormalization on the GPU against the restated reference operator
    (src/operators/layer_normalization.rs:25-80) over the whole tensor: the
    kernel sums with a warp tree and multiplies by rsqrt(var + eps), so the
    bound is fp32 rounding, 4e-6 absolute on outputs of order 1-5."""
    from iconnx_b200.engine import GpuGraphExecutor
    from oracle import oracle
    gamma = (1.0 + synth.normal((D,), 0.02, 61)).astype(np.float32)
    beta = synth.normal((D,), 0.02, 62)
    ex = GpuGraphExecutor.new()
    ex.add_input("x", [rows, D])
    ex.add_initializer("g", gamma)
    ex.add_initializer("b", beta)
    ex.add_node("ln", "LayerNormalization", ["x", "g", "b"], ["y"], {"axis": -1, "epsilon": eps})
    x = synth.normal((rows, D), 3.0, 63) + np.float32(0.5)
    x[0, :] = np.float32(1.25)          # a constant row: zero variance
    got = ex.run({"x": x}, ["y"])["y"]
    ref = oracle.layer_normalization(x, gamma, beta, eps)
    assert np.abs(got.astype(np.float64) - ref).max() <= 4e-6
