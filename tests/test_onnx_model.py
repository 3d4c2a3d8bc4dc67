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


# Tolerance of the CUDA op map against the f64 restatement: f32 arithmetic throughout (split-tf32
# tensor-core GEMMs, f32 attention products), outputs are LayerNorm rows of magnitude up to ~5.
ONNX_MAX_ABS, ONNX_MIN_COS = 2e-4, 0.999999


def _close(y, ref, what):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    d = float(np.abs(y - ref).max())
    yy, rr = y.reshape(-1, y.shape[-1]), ref.reshape(-1, ref.shape[-1])
    cos = float(((yy * rr).sum(1) / np.linalg.norm(yy, axis=1) / np.linalg.norm(rr, axis=1)).min())
    print(f"{what}: max-abs {d:.3e}, min cos {cos:.8f}")
    assert d < ONNX_MAX_ABS and cos > ONNX_MIN_COS, (what, d, cos)


def test_restatement_follows_the_reference_executor():
    """onnx_ref's default semantics are the reference executor's: Gelu the tanh form
    (executor.zig:122), Erf the A&S polynomial (125-137, within its stated 1.5e-7), LayerNormalization
    at epsilon 1e-5 whatever the node says (3318); spec=True is the ONNX specification."""
    import math
    x = np.linspace(-6, 6, 2001)
    assert np.abs(onnx_ref.erf_as(x) - np.vectorize(math.erf)(x)).max() <= 1.5e-7
    assert abs(onnx_ref.erf_as(0.0)) <= 1.5e-7 and np.allclose(onnx_ref.erf_as(-x), -onnx_ref.erf_as(x))
    from tenzor_b200.onnx_ops import Node
    h = np.linspace(-4, 4, 64, dtype=np.float32)[None, :]
    g_ref = onnx_ref.run([Node("Gelu", ["h"], ["y"])], {}, {"h": h}, ["y"])[0]
    assert np.allclose(g_ref, h * 0.5 * (1 + np.tanh(0.7978845608 * (h + 0.044715 * h ** 3))), atol=1e-6)
    g_spec = onnx_ref.run([Node("Gelu", ["h"], ["y"])], {}, {"h": h}, ["y"], spec=True)[0]
    assert np.allclose(g_spec, 0.5 * h * (1 + np.vectorize(math.erf)(h / np.sqrt(2))), atol=1e-6)
    r = np.random.default_rng(0).normal(0, 1e-3, (4, 8)).astype(np.float32)  # variance near eps
    one, zero = np.ones(8, np.float32), np.zeros(8, np.float32)
    ln = [Node("LayerNormalization", ["x", "g", "b"], ["y"], {"epsilon": 1e-12})]
    y_ref = onnx_ref.run(ln, {"g": one, "b": zero}, {"x": r}, ["y"])[0]
    y_spec = onnx_ref.run(ln, {"g": one, "b": zero}, {"x": r}, ["y"], spec=True)[0]
    m = r.mean(1, keepdims=True)
    v = ((r - m) ** 2).mean(1, keepdims=True)
    assert np.allclose(y_ref, (r - m) / np.sqrt(v + 1e-5), atol=1e-5)
    assert np.allclose(y_spec, (r - m) / np.sqrt(v + 1e-12), atol=1e-4)


def test_reference_executor_kats():
    """The reference's own executor tests (executor.zig:6197-6244 Add, 6246-6293 MatMul)."""
    import kats
    from tenzor_b200.onnx_ops import Node
    for op, a, b, sa, sb, want in kats.ONNX_EXECUTOR:
        y = onnx_ref.run([Node(op, ["A", "B"], ["C"])], {}, {"A": np.array(a, np.float32).reshape(sa),
                                                            "B": np.array(b, np.float32).reshape(sb)}, ["C"])[0]
        assert np.array_equal(y.reshape(-1), np.array(want, np.float32))


@pytest.mark.parametrize("variant", [{}, {"decomposed_ln": True}, {"where_mask": True}])
def test_exported_layer_restatement_vs_torch(variant):
    """The exporter-style fixture is a BERT layer: its restatement (ONNX-spec semantics) agrees with the
    same layer written with torch.nn.functional on the CPU in f64."""
    import torch
    import torch.nn.functional as F
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer_exported(seed=5, **variant)
    m = M.parse_model(data)
    y, cls = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs, spec=True)
    P = {k: torch.from_numpy(np.asarray(v)).double() for k, v in m.initializers.items()}
    ids = torch.from_numpy(feeds["input_ids"])
    mask = torch.from_numpy(feeds["attention_mask"]).double()
    B, S = ids.shape
    x = P["word"][ids] + P["pos"][:S][None] + P["type"][0][None, None]
    x = F.layer_norm(x, (384,), P["ln_e_g"], P["ln_e_b"], 1e-12)
    heads = lambda t: t.reshape(B, S, 12, 32).transpose(1, 2)
    q, k, v = (heads(x @ P["w" + c] + P["b" + c]) for c in "qkv")
    add = (1.0 - mask)[:, None, None, :] * -3.4028234663852886e38
    a = torch.softmax(q @ k.transpose(-1, -2) / np.sqrt(32) + add, -1) @ v
    x1 = F.layer_norm(a.transpose(1, 2).reshape(B, S, 384) @ P["wo"] + P["bo"] + x, (384,), P["ln1_g"], P["ln1_b"], 1e-12)
    h = F.gelu(x1 @ P["w1"] + P["b1"])
    y2 = F.layer_norm(h @ P["w2"] + P["b2"] + x1, (384,), P["ln2_g"], P["ln2_b"], 1e-12)
    assert np.abs(y - y2.numpy()).max() < 1e-4
    assert np.abs(cls - y2[:, 0].numpy()).max() < 1e-4


def test_exported_layer_reader_round_trip():
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer_exported(seed=6)
    m = M.parse_model(data)
    assert m.inputs == ["input_ids", "attention_mask"] and m.outputs == ["y", "cls"] and m.opset == {"": 17}
    ops = {n.op_type for n in m.nodes}
    assert {"Shape", "Slice", "Unsqueeze", "Concat", "Reshape", "Transpose", "Cast", "Erf", "Softmax"} <= ops
    assert m.initializers["position_ids"].dtype == np.int64 and m.initializers["s1"].shape == ()
    mha, _ = W.mha_model(with_mask=True)
    node = M.parse_model(mha).nodes[-1]
    assert node.inputs == ["q", "k", "v", "", "kpm"] and node.attrs == {"num_heads": 12}


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [False, True])
@pytest.mark.parametrize("gelu", ["Gelu", "Erf"])
def test_bert_layer_on_cuda_vs_restatement(ctx, gelu, spec):
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer(seed=4, gelu=gelu)
    m = M.parse_model(data)
    y = M.run(ctx, m, feeds, spec=spec)[0].cpu().numpy()
    ref = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs, spec=spec)[0]
    _close(y, ref, f"one-head layer, {gelu}, spec={spec}")


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [False, True])
@pytest.mark.parametrize("variant", [{}, {"decomposed_ln": True}, {"where_mask": True}])
def test_exported_12_head_layer_on_cuda_vs_restatement(ctx, variant, spec):
    """The exporter-style Arctic-size layer (hidden 384, 12 heads) on the CUDA op map."""
    from tenzor_b200 import onnx_model as M
    data, feeds = W.bert_layer_exported(seed=7, **variant)
    m = M.parse_model(data)
    y, cls = (t.cpu().numpy() for t in M.run(ctx, m, feeds, spec=spec))
    y_ref, cls_ref = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs, spec=spec)
    _close(y, y_ref, f"12-head layer {variant}, spec={spec}")
    _close(cls, cls_ref, "CLS rows")


@pytest.mark.gpu
@pytest.mark.parametrize("spec,with_mask", [(False, False), (True, False), (True, True)])
def test_multi_head_attention_on_cuda_vs_restatement(ctx, spec, with_mask):
    """MultiHeadAttention: 8 heads and no mask as the reference executes it, or the node's num_heads
    (12) and key_padding_mask with spec=True."""
    from tenzor_b200 import onnx_model as M
    data, feeds = W.mha_model(seed=8, with_mask=with_mask)
    m = M.parse_model(data)
    o = M.run(ctx, m, feeds, spec=spec)[0].cpu().numpy()
    ref = onnx_ref.run(m.nodes, m.initializers, feeds, m.outputs, spec=spec)[0]
    _close(o, ref, f"MHA spec={spec} mask={with_mask}")


@pytest.mark.gpu
def test_reference_executor_kats_on_cuda(ctx):
    import kats
    import torch
    from tenzor_b200.onnx_ops import Node, run_graph
    for op, a, b, sa, sb, want in kats.ONNX_EXECUTOR:
        A = torch.tensor(a, dtype=torch.float32).reshape(sa).cuda()
        B = torch.tensor(b, dtype=torch.float32).reshape(sb).cuda()
        y = run_graph(ctx, [Node(op, ["A", "B"], ["C"])], {}, {"A": A, "B": B}, ["C"])[0]
        assert np.array_equal(y.cpu().numpy().reshape(-1), np.array(want, np.float32)), op
