"""Fused self-attention (Reshape/Transpose -> MatMul -> Div -> Add(mask) ->
Softmax -> MatMul -> Transpose -> Reshape, one kernel on the GPU) against a
float64 evaluation of the same graph and against the CPU graph interpreter
that restates the reference's fp32 ops (src/graph_executor.rs:92-278).

The reference computes attention in fp32; the fused kernel runs on the
tensor cores with split-precision TF32 (three MMAs per product), so the
bound is fp32-level: 2e-5 absolute on outputs of magnitude ~1.
"""
import numpy as np
import pytest

from iconnx_b200 import graphs, synth
from oracle.graph_executor import CpuGraph

gpu = pytest.mark.gpu
TOL = 2e-5


def _inputs(batch, seq, hidden, mask, seed):
    inp = {t: synth.normal((batch, seq, hidden), 1.0, seed + i) for i, t in enumerate("qkv")}
    if mask != "none":
        rows = batch if mask == "batch" else 1
        keep = np.ones((rows, seq), np.float32)
        for r in range(rows):  # ragged: row r keeps its first seq - 3r keys
            keep[r, max(1, seq - 3 * r):] = 0.0
        inp["mask_bias"] = ((1.0 - keep) * np.float32(-10000.0)).reshape(rows, 1, 1, seq)
    return inp


def test_attention_reference_matches_cpu_interpreter():
    inp = _inputs(2, 8, 128, "batch", 40)
    cpu = CpuGraph()
    out = graphs.build_attention(cpu, 2, 8, 128, 2, "batch")
    r = cpu.run(inp, [out])[out]
    ref = graphs.attention_reference(inp["q"], inp["k"], inp["v"], 2, inp["mask_bias"])
    assert np.max(np.abs(r - ref)) < TOL


@gpu
@pytest.mark.parametrize("batch,seq,hidden,heads,mask", [
    (2, 128, 768, 12, "batch"),    # one query tile, two key tiles
    (3, 200, 256, 4, "shared"),    # ragged query and key tiles
    (2, 16, 128, 2, "none"),       # one partial tile
    (1, 1, 64, 1, "batch"),        # a single key
    (1, 384, 768, 12, "batch"),    # three query tiles, six key tiles (wide tiling)
    (2, 300, 256, 4, "shared"),    # ragged tiles on the wide tiling
    (2, 512, 768, 12, "batch"),    # the BERT-base sequence length
])
def test_fused_attention_matches_float64(batch, seq, hidden, heads, mask):
    from iconnx_b200.engine import GpuGraphExecutor
    ex = GpuGraphExecutor.new()
    out = graphs.build_attention(ex, batch, seq, hidden, heads, mask)
    inp = _inputs(batch, seq, hidden, mask, 50 + seq)
    g = ex.run(inp, [out])[out]
    assert [s for s in ex.plan() if s.startswith("Attention ")], ex.plan()
    ref = graphs.attention_reference(inp["q"], inp["k"], inp["v"], heads, inp.get("mask_bias"))
    err = np.max(np.abs(g.astype(np.float64) - ref))
    assert err < TOL, err
    if seq <= 128:
        cpu = CpuGraph()
        graphs.build_attention(cpu, batch, seq, hidden, heads, mask)
        r = cpu.run(inp, [out])[out]
        assert np.max(np.abs(g - r)) < TOL


@gpu
def test_fused_attention_large_scores_as_accurate_as_fp32():
    """Scores of order 10^2-10^3, where softmax turns any rounding of the
    scores into visible output changes: the kernel's error against float64
    stays within twice that of the fp32 CPU interpreter (numpy fp32 MatMul)."""
    from iconnx_b200.engine import GpuGraphExecutor
    batch, seq, hidden, heads = 2, 128, 256, 4
    inp = _inputs(batch, seq, hidden, "batch", 90)
    inp["q"] = inp["q"] * np.float32(12.0)
    inp["k"] = inp["k"] * np.float32(12.0)
    ref = graphs.attention_reference(inp["q"], inp["k"], inp["v"], heads, inp["mask_bias"])
    cpu = CpuGraph()
    out = graphs.build_attention(cpu, batch, seq, hidden, heads, "batch")
    e_cpu = np.max(np.abs(cpu.run(inp, [out])[out] - ref))
    ex = GpuGraphExecutor.new()
    graphs.build_attention(ex, batch, seq, hidden, heads, "batch")
    e_gpu = np.max(np.abs(ex.run(inp, [out])[out] - ref))
    assert e_gpu <= 2.0 * e_cpu + 1e-6, (e_gpu, e_cpu)


@gpu
@pytest.mark.parametrize("batch", [2, 26])
def test_attention_fused_minmax_feeds_dynamic_quantize(batch):
    """DynamicQuantizeLinear on the attention output takes (min, max) from the
    attention kernel's epilogue and runs only its quantise pass.  At batch 26
    x 12 heads x 4 query tiles the kernel writes 1248 partials, more than a
    DQL slot holds; they are folded into one pair first.  Either way the
    quantised tensor, scale and zero point are bit-exact against the oracle's
    DynamicQuantizeLinear of the same attention output."""
    from iconnx_b200.engine import GpuGraphExecutor
    from oracle import oracle
    seq, hidden, heads = 512, 768, 12
    ex = GpuGraphExecutor.new()
    out = graphs.build_attention(ex, batch, seq, hidden, heads, "batch")
    ex.add_node("dql", "DynamicQuantizeLinear", [out], ["y", "y_scale", "y_zp"])
    inp = _inputs(batch, seq, hidden, "batch", 7 + batch)
    res = ex.run(inp, [out, "y", "y_scale", "y_zp"])
    plan = ex.plan()
    assert any(s.startswith("DynamicQuantizeLinear(quantise)") for s in plan), plan
    y, scale, zp = oracle.dynamic_quantize_linear(res[out])
    np.testing.assert_array_equal(res["y"], y)
    assert np.float32(res["y_scale"]).tobytes() == np.float32(scale).tobytes()
    assert np.uint8(res["y_zp"]) == np.uint8(zp)
