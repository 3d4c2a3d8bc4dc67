"""The `.eval()` backend (tenzor_b200.expr) and the ONNX op map (tenzor_b200.onnx_ops) on the B200:
each fusion plan lowered to library launches, checked against the CPU oracle / an fp32 reference."""
import numpy as np
import pytest
import torch

import kats

pytestmark = pytest.mark.gpu


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_matmul_epilogue_plan(ctx, oracle):
    from tenzor_b200 import expr as E
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (300, 384)).astype(np.float32)
    b = rng.uniform(-1, 1, (384, 1536)).astype(np.float32)
    bias = rng.uniform(-1, 1, 1536).astype(np.float32)
    e = E.matmul(cu(a), cu(b)).add(cu(bias)).gelu()
    assert E.analyze(e) == "matmul_epilogue"
    y = e.eval(ctx).cpu().numpy()
    ref = oracle.matmul_epilogue(a, b, bias, [1, 3])
    assert np.abs(y - ref).max() <= 4e-3 * np.sqrt(384) * 0.6
    # the reference's KAT (codegen.zig:331-348), K padded to the 16-byte TMA row
    a0, b0, bias0, chain, want = kats.MATMUL_EPILOGUE
    a0 = np.pad(np.array(a0, np.float32), ((0, 0), (0, 2)))
    b0 = np.pad(np.array(b0, np.float32), ((0, 2), (0, 0)))
    y0 = E.matmul(cu(a0), cu(b0)).add(cu(np.array(bias0, np.float32))).relu().eval(ctx).cpu().numpy()
    assert (y0 == np.array(want, np.float32)).all()


def test_elementwise_plans(ctx, oracle):
    from tenzor_b200 import expr as E
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (256, 4096)).astype(np.float32)
    c = rng.uniform(-1, 1, (256, 4096)).astype(np.float32)
    b = rng.uniform(-1, 1, 4096).astype(np.float32)
    y = E.tensor(cu(a)).add(cu(b)).mul(cu(c)).exp().eval(ctx).cpu().numpy()  # configs[2](b)
    assert np.abs(y / oracle.ew_add_mul_exp(a, b, c) - 1).max() < 1e-6
    # a general graph: relu(a * 2 - c) / (1 + exp(b_row)) -> one program launch
    e = E.tensor(cu(a)).mul(2.0).sub(cu(c)).relu().div(E.tensor(cu(b)).exp().add(1.0))
    ref = np.maximum(a * 2 - c, 0) / (1 + np.exp(b))[None, :]
    assert np.abs(e.eval(ctx).cpu().numpy() - ref).max() < 1e-5
    x, chain, want, tol = kats.EW_CHAIN
    z = E.tensor(cu(np.array(x))).exp().relu().eval(ctx).cpu().numpy()
    assert np.abs(z - np.array(want)).max() <= tol


def test_reduce_and_single_plans(ctx, oracle):
    from tenzor_b200 import expr as E
    for op, pre, x, want, tol in kats.REDUCE:
        e = E.tensor(cu(np.array(x)))
        for p in pre:
            e = getattr(e, p)()
        assert abs(e.sum().eval(ctx).item() - want) <= tol
    rng = np.random.default_rng(2)
    x = rng.normal(0, 2, (1000, 384)).astype(np.float32)
    g = rng.normal(1, 0.1, 384).astype(np.float32)
    bb = rng.normal(0, 0.1, 384).astype(np.float32)
    y = E.tensor(cu(x)).layer_norm(cu(g), cu(bb)).eval(ctx).cpu().numpy()
    assert np.abs(y - oracle.layernorm(x, g, bb, 1e-5)).max() < 2e-5
    s = E.tensor(cu(x[:, :128])).softmax().eval(ctx).cpu().numpy()
    assert np.abs(s - oracle.softmax(x[:, :128])).max() < 1e-6
    t = rng.normal(0, 1, (50, 64)).astype(np.float32)
    ids = torch.tensor([3, 0, 49, 3], dtype=torch.int32).cuda()
    gth = E.gather(cu(t), ids).eval(ctx).cpu().numpy()
    assert (gth == t[[3, 0, 49, 3]]).all()


def test_onnx_encoder_block(ctx):
    """A hand-built ONNX graph of one post-LN encoder FFN block (the shape of an exported BERT layer:
    Gemm+bias, erf-Gelu, MatMul, Add, LayerNormalization, Softmax, Gather) on the CUDA op map."""
    from tenzor_b200.onnx_ops import Node, run_graph
    rng = np.random.default_rng(3)
    T, H, F = 200, 384, 1536
    emb = rng.normal(0, 1, (1000, H)).astype(np.float32)
    w1 = rng.normal(0, 0.05, (F, H)).astype(np.float32)
    b1 = rng.normal(0, 0.05, F).astype(np.float32)
    w2 = rng.normal(0, 0.05, (F, H)).astype(np.float32)
    g = rng.normal(1, 0.1, H).astype(np.float32)
    be = rng.normal(0, 0.1, H).astype(np.float32)
    ids = rng.integers(0, 1000, T).astype(np.int64)
    nodes = [
        Node("Gather", ["emb", "ids"], ["x"]),
        Node("Gemm", ["x", "w1", "b1"], ["h"], {"transB": 1}),
        Node("Gelu", ["h"], ["hg"]),
        Node("MatMul", ["hg", "w2"], ["f"]),
        Node("Add", ["f", "x"], ["r"]),
        Node("LayerNormalization", ["r", "g", "be"], ["y"], {"epsilon": 1e-12}),
        Node("Softmax", ["y"], ["p"], {"axis": -1}),
    ]
    init = {"emb": cu(emb), "w1": cu(w1), "b1": cu(b1), "w2": cu(w2), "g": cu(g), "be": cu(be)}
    # spec=True: the ONNX semantics this check restates (erf Gelu, the node's epsilon)
    y, p = run_graph(ctx, nodes, init, {"ids": torch.from_numpy(ids.astype(np.int32)).cuda()}, ["y", "p"], spec=True)
    x = emb[ids].astype(np.float64)
    h = x @ w1.T + b1
    from math import sqrt
    import scipy.special as sp
    hg = 0.5 * h * (1 + sp.erf(h / sqrt(2)))
    r = hg @ w2 + x
    mu = r.mean(1, keepdims=True)
    var = ((r - mu) ** 2).mean(1, keepdims=True)
    yr = (r - mu) / np.sqrt(var + 1e-12) * g + be
    pr = np.exp(yr - yr.max(1, keepdims=True))
    pr /= pr.sum(1, keepdims=True)
    # split-tf32 (f32-accurate) tensor-core GEMMs inside
    assert np.abs(y.cpu().numpy() - yr).max() < 2e-4
    assert np.abs(p.cpu().numpy() / pr - 1).max() < 1e-3
