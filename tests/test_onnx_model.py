"""ONNX model files (tenzor_b200/onnx_model.py): the protobuf reader on hand-built encoder-layer
fixtures (tests/onnx_writer.py; no `.onnx` file or `onnx` package exists in this environment), and the
whole graph executed on the CUDA op map against the NumPy restatement of the executor's ops
(oracle/onnx_ref.py)."""
import numpy as np
import pytest

import onnx_ref
import onnx_writer as W


@pytest.mark.parametrize("raw", [True, False])
@pytest.mark.parametrize("gelu", ["Gelu", "Erf"])
def test_reader_round_trip(raw, gelu):
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer(seed=1, gelu=gelu, raw=raw)
    m = M.parse_model(data)
    assert m.inputs == ["ids"] and m.outputs == ["y"] and m.opset == {"": 20} and m.ir_version == 9
    ops = [n.op_type for n in m.nodes]
    assert ops[:3] == ["Gather", "Add", "LayerNormalization"] and ops[-1] == "LayerNormalization"
    assert ("Erf" in ops) == (gelu == "Erf") and ("Gelu" in ops) == (gelu == "Gelu")
    ln = m.nodes[2]
    assert ln.attrs["axis"] == -1 and abs(ln.attrs["epsilon"] - 1e-12) < 1e-18
    gemm = [n for n in m.nodes if n.op_type == "Gemm"][0]
    assert gemm.attrs == {"transB": 1}
    assert m.initializers["word"].shape == (97, 64) and m.initializers["word"].dtype == np.float32
    # the restatement runs the parsed graph: the reader kept every tensor bit-for-bit
    y = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs)[0]
    assert y.shape == (24, 64) and np.isfinite(y).all()


def test_reader_rejects_truncated_files():
    from tenzor_b200 import onnx_model as M
    data, _ = W.bert_layer(seed=2)
    with pytest.raises(M.OnnxFormatError):
        M.parse_model(data[: len(data) // 2])


def test_reader_skips_unknown_fields():
    from tenzor_b200 import onnx_model as M
    data, _ = W.bert_layer(seed=3)
    extra = W._str(14, "unknown string field") + W._int(15, 123456789)  # fields the reader does not use
    m = M.parse_model(extra + data + W._key(16, 1) + b"\x00" * 8)
    assert len(m.nodes) == 22 and m.outputs == ["y"]


@pytest.mark.gpu
@pytest.mark.parametrize("gelu", ["Gelu", "Erf"])
def test_bert_layer_on_cuda_vs_restatement(ctx, gelu):
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer(seed=4, gelu=gelu)
    m = M.parse_model(data)
    y = M.run(ctx, m, feeds)[0].cpu().numpy()
    ref = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs)[0]
    # tf32 MatMul / Gemm operands: LayerNorm outputs of unit scale, tolerance as for the op tests
    assert np.abs(y - ref).max() < 2e-2
    cos = (y * ref).sum(1) / np.linalg.norm(y, axis=1) / np.linalg.norm(ref, axis=1)
    assert cos.min() > 0.9999
