"""The fusion planner restated in tenzor_b200.expr classifies graphs exactly as the reference's
analyzer.zig unit tests expect (analyzer.zig:303-382).  CPU only: no evaluation."""
import torch

from tenzor_b200 import expr as E


def leaf(*shape):
    return E.tensor(torch.zeros(*shape))


def test_single_tensor():
    assert E.analyze(leaf(4)) == "single"


def test_unary_is_single():
    assert E.analyze(leaf(4).relu()) == "single"


def test_elementwise_chain():
    e = leaf(4).exp().relu()
    assert E.analyze(e) == "elementwise_chain"
    chain, base = E.collect_unary_chain(e)
    assert chain == ["exp", "relu"] and base.kind == "tensor"


def test_matmul_epilogue():
    e = E.matmul(leaf(2, 3), leaf(3, 4)).add(leaf(4)).relu()
    p = E.plan(e)
    assert p.pattern == "matmul_epilogue"
    assert [op for op, _ in p.epilogue] == ["add", "relu"]
    assert E.find_matmul_base(e).kind == "matmul"


def test_binary_is_chain():
    assert E.analyze(leaf(4).add(leaf(4))) == "elementwise_chain"


def test_reduce_epilogue_and_broadcast_shapes():
    assert E.analyze(leaf(8).exp().sum()) == "reduce_epilogue"
    assert E.analyze(leaf(8).sum()) == "single"
    e = leaf(16, 4096).add(leaf(4096)).mul(leaf(16, 4096)).exp()
    assert E.analyze(e) == "elementwise_chain" and e.shape == (16, 4096)
    assert E._strides2d((4096,), (16, 4096)) == (0, 1)
    assert E._strides2d((16, 1), (16, 4096)) == (1, 0)
    assert E._strides2d((16, 4096), (16, 4096)) == (4096, 1)
