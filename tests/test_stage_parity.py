"""Stage-by-stage bit-exact parity of the executor's own compiled plans at
the benchmark configurations (the plans bench.py times: QKV merged, residual
Adds fused, producer-fused (min, max) with quantise-only DynamicQuantizeLinear,
CUDA-graph replay), against the oracle restatement of the reference operators.

LayerNormalization steps are checked within 4e-6 (fp32 rounding order).

Reference paths: GraphExecutor::run (src/graph_executor.rs:92-278) and
GpuGraphExecutor::run (src/cuda/inference/mod.rs:428-464).  Each int8 stage
gets its own GPU inputs (tests/stage_parity.py), so an fp32 glue difference
upstream (attention, LayerNorm) cannot hide or fake an int8 mismatch.
"""
import numpy as np
import pytest

from iconnx_b200 import graphs, synth
from oracle.graph_executor import CpuGraph

from stage_parity import check_plan

gpu = pytest.mark.gpu


def _build(build, *args):
    from iconnx_b200.engine import GpuGraphExecutor
    ex, rec = GpuGraphExecutor.new(), CpuGraph()
    out = build(ex, *args)
    build(rec, *args)
    ex.node_attrs = {name: attrs for name, _, _, _, attrs in rec.nodes}
    return ex, rec.inits, out


def _run_and_check(ex, inits, inp, out):
    first = ex.run(inp, [out])[out]
    second = ex.run(inp, [out])[out]          # captured-graph replay
    np.testing.assert_array_equal(first.view(np.uint32), second.view(np.uint32))
    counts = check_plan(ex, inits, attrs=getattr(ex, "node_attrs", None))
    # the step-by-step re-execution reproduces the run bit for bit
    np.testing.assert_array_equal(ex.fetch(out).view(np.uint32), first.view(np.uint32))
    return counts


@gpu
def test_config2_ffn_plan_stage_by_stage():
    """Config 2 (batch 32 x seq 128): QuantLinear+GELU -> quantise-only DQL
    (min, max from the GELU epilogue) -> QuantLinear, each stage exact."""
    ex, inits, out = _build(graphs.build_ffn, 32, 128)
    counts = _run_and_check(ex, inits, {"x": synth.normal((4096, 768), 1.0, 0)}, out)
    assert counts == {"dql": 2, "QuantLinear+GELU": 1, "QuantLinear": 1}, counts
    assert any(s.startswith("DynamicQuantizeLinear(quantise)") for s in ex.plan())


@gpu
def test_config3_distilbert_plan_stage_by_stage():
    """Config 3: DistilBERT-base, batch 32 x seq 128, 6 layers, w_scale 0.01."""
    cfg = graphs.DISTILBERT
    ex, inits, out = _build(graphs.build_bert, cfg, 32, 128)
    counts = _run_and_check(ex, inits, graphs.bert_inputs(32, 128), out)
    L = cfg.layers
    assert counts["dql"] == 4 * L
    assert counts["QuantLinear(QKV)"] == L
    # O-proj and FFN2 with their residual Add; the LayerNorm after them in the
    # same kernel where the GPU runs the LayerNorm-fused GEMM
    assert counts.get("QuantLinear+Residual", 0) + counts.get("QuantLinear+Residual+LayerNorm", 0) == 2 * L
    assert counts["QuantLinear+GELU"] == L
    assert counts["layernorm"] == 2 * L + 1


@gpu
def test_config4_bert_base_plan_stage_by_stage():
    """Config 4: BERT-base, batch 64 x seq 512, 12 layers, per-column w_scale
    and int8 weight zero points (the column-sum correction)."""
    cfg = graphs.BERT_BASE
    ex, inits, out = _build(graphs.build_bert, cfg, 64, 512)
    counts = _run_and_check(ex, inits, graphs.bert_inputs(64, 512), out)
    L = cfg.layers
    assert counts["dql"] == 4 * L
    assert counts["QuantLinear(QKV)"] == L
    # O-proj and FFN2 with their residual Add; the LayerNorm after them in the
    # same kernel where the GPU runs the LayerNorm-fused GEMM
    assert counts.get("QuantLinear+Residual", 0) + counts.get("QuantLinear+Residual+LayerNorm", 0) == 2 * L
    assert counts["QuantLinear+GELU"] == L
    assert counts["layernorm"] == 2 * L + 1


@gpu
def test_step_interface_errors():
    from iconnx_b200 import IcxError
    from iconnx_b200.engine import GpuGraphExecutor
    ex = GpuGraphExecutor.new()
    out = graphs.build_linear(ex)
    assert ex.steps() == []
    ex.run({"x": synth.normal((1, 128, 768), 1.0, 0)}, [out])
    steps = ex.steps()
    assert [s[0] for s in steps][-1].startswith("QuantLinear")
    with pytest.raises(IcxError):
        ex.run_step(len(steps))
    with pytest.raises(IcxError, match="not materialised"):
        ex.value("acc_7")  # the s32 accumulator lives in tensor memory only
