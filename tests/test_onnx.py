"""OnnxParser.parse_file / GpuGraphExecutor.from_model round trip
(src/onnx_parser.rs:138, src/cuda/inference/mod.rs:246-267)."""
import os

import numpy as np
import pytest

from iconnx_b200 import graphs
from iconnx_b200.onnx import GraphRecorder, OnnxParser, save_model


def _saved(tmp_path, cfg=graphs.BertConfig(layers=1, vocab=1000), batch=2, seq=16):
    rec = GraphRecorder()
    out = graphs.build_bert(rec, cfg, batch, seq)
    path = os.path.join(tmp_path, "model.onnx")
    save_model(path, rec, [out])
    return rec, out, path


def test_parse_round_trip(tmp_path):
    rec, out, path = _saved(tmp_path)
    m = OnnxParser.parse_file(path)
    assert [n.op_type for n in m.nodes] == [n.op_type for n in rec.nodes]
    assert [n.inputs for n in m.nodes] == [n.inputs for n in rec.nodes]
    for a, b in zip(m.nodes, rec.nodes):
        assert a.attrs.keys() == b.attrs.keys()
        for k in a.attrs:
            np.testing.assert_allclose(np.asarray(a.attrs[k], dtype=np.float64),
                                       np.asarray(b.attrs[k], dtype=np.float64), rtol=1e-7)
    w = m.extract_weights()
    assert w.keys() == rec.inits.keys()
    for k, v in rec.inits.items():
        assert w[k].dtype == v.dtype and w[k].shape == v.shape
        np.testing.assert_array_equal(w[k], v)
    shapes = m.input_shapes()
    assert shapes["input_ids"][1] == [2, 16] and shapes["input_ids"][0] == np.int64
    assert m.output_names() == [out]


def test_int8_and_uint8_initializers_survive(tmp_path):
    rec = GraphRecorder()
    rec.add_input("x", [4], np.float32)
    rec.add_initializer("w8", np.array([-128, -1, 0, 127], np.int8))
    rec.add_initializer("u8", np.array([0, 1, 255], np.uint8))
    rec.add_node("n", "Identity", ["x"], ["y"])
    p = os.path.join(tmp_path, "m.onnx")
    save_model(p, rec, ["y"])
    w = OnnxParser.parse_file(p).extract_weights()
    assert w["w8"].tolist() == [-128, -1, 0, 127] and w["u8"].tolist() == [0, 1, 255]


@pytest.mark.gpu
def test_from_model_matches_builder(tmp_path):
    from iconnx_b200.engine import GpuGraphExecutor
    rec, out, path = _saved(tmp_path)
    ex1 = GpuGraphExecutor.from_model(OnnxParser.parse_file(path))
    ex2 = GpuGraphExecutor.new()
    graphs.build_bert(ex2, graphs.BertConfig(layers=1, vocab=1000), 2, 16)
    inp = graphs.bert_inputs(2, 16, vocab=1000)
    np.testing.assert_array_equal(ex1.run(inp, [out])[out], ex2.run(inp, [out])[out])
