"""The general `.eval()` executor on the B200 (src/backend/cpu/executor.zig): N-D broadcasting
(152-197), evalMatmul's dot / vector / 2-D / batched cases (199-325), single-axis reductions
(327-361, reduce.zig:52-95), softmax on any axis (softmax.zig:157-220), transpose and reshape
(expr.zig TransposeExpr / ReshapeExpr), each checked against the reference's own executor tests
(executor.zig:742-1347) and against NumPy in f64 on seeded random shapes.  f32 kernels: relative
tolerance 1e-5 of the operand scale unless the test says otherwise."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def test_reference_batched_matmul_kats(ctx):
    from tenzor_b200 import expr as E
    # executor.zig:742-784: [2,2,3] @ [2,3,2]
    a = np.arange(1, 13, dtype=np.float32).reshape(2, 2, 3)
    b = np.array([1, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1, 1], np.float32).reshape(2, 3, 2)
    y = E.tensor(cu(a)).matmul(cu(b)).eval(ctx).cpu().numpy()
    assert y.shape == (2, 2, 2) and (y.reshape(-1) == [4, 5, 10, 11, 24, 24, 33, 33]).all()
    # executor.zig:786-819: [2,3,4] @ [4,5], first row ones
    a = np.zeros((2, 3, 4), np.float32)
    a[0, 0] = 1
    y = E.tensor(cu(a)).matmul(cu(np.ones((4, 5)))).eval(ctx).cpu().numpy()
    assert y.shape == (2, 3, 5) and (y[0, 0] == 4).all() and (y.reshape(-1)[5:] == 0).all()
    # executor.zig:821-852: the Arctic pattern [2,4,8] @ I8
    h = np.ones((2, 4, 8), np.float32)
    y = E.tensor(cu(h)).matmul(cu(np.eye(8))).eval(ctx).cpu().numpy()
    assert np.abs(y - h).max() <= 1e-5


def test_reference_softmax_transpose_reshape_kats(ctx):
    from tenzor_b200 import expr as E
    s = E.tensor(cu([1, 2, 3, 4])).softmax(-1).eval(ctx).cpu().numpy()  # executor.zig:854
    assert abs(s.sum() - 1) < 1e-5 and (np.diff(s) > 0).all()
    s = E.tensor(cu([[1, 2, 3], [0, 0, 0]])).softmax(-1).eval(ctx).cpu().numpy()  # 876
    assert np.abs(s.sum(1) - 1).max() < 1e-5 and np.abs(s[1] - 1 / 3).max() < 1e-5
    x = np.array([1, 2, 3, 4, 0, 0, 1, -1], np.float32).reshape(1, 2, 2, 2)  # 905: attention rows
    s = E.tensor(cu(x)).softmax(-1).eval(ctx).cpu().numpy().reshape(4, 2)
    assert np.abs(s.sum(1) - 1).max() < 1e-5 and np.abs(s[2] - 0.5).max() < 1e-5
    t = E.tensor(cu(np.arange(1, 7).reshape(2, 3))).transpose((1, 0)).eval(ctx).cpu().numpy()  # 1233
    assert t.shape == (3, 2) and (t.reshape(-1) == [1, 4, 2, 5, 3, 6]).all()
    x = np.arange(1, 13, dtype=np.float32).reshape(1, 2, 2, 3)  # 1261
    t = E.tensor(cu(x)).transpose((0, 2, 1, 3)).eval(ctx).cpu().numpy()
    assert t.shape == (1, 2, 2, 3) and (t.reshape(-1)[[0, 1, 2, 3, 4, 5, 6, 9]] == [1, 2, 3, 7, 8, 9, 4, 10]).all()
    h = np.arange(1, 13, dtype=np.float32).reshape(1, 2, 6)  # 1300: the attention reshape / transpose dance
    t = E.tensor(cu(h)).reshape((1, 2, 2, 3)).transpose((0, 2, 1, 3)).eval(ctx).cpu().numpy()
    assert (t.reshape(-1) == [1, 2, 3, 7, 8, 9, 4, 5, 6, 10, 11, 12]).all()
    r = E.tensor(cu(np.arange(1, 7))).reshape((2, 3)).eval(ctx).cpu().numpy()  # 1213
    assert r.shape == (2, 3) and (r.reshape(-1) == np.arange(1, 7)).all()


@pytest.mark.parametrize("sa,sb", [((3, 1, 5, 7), (4, 1, 7)), ((6,), (2, 3, 6)), ((2, 1, 4, 1), (1, 3, 1, 5)),
                                   ((5, 1, 1, 3, 2, 4), (1, 2, 1, 3, 1, 4)), ((), (3, 4))])
def test_nd_broadcast_programs(ctx, sa, sb):
    """N-D broadcasting (evalBinaryBroadcast) through one program launch, rank up to 6."""
    from tenzor_b200 import expr as E
    rng = np.random.default_rng(len(sa) * 7 + len(sb))
    a = rng.uniform(-2, 2, sa).astype(np.float32)
    b = rng.uniform(0.5, 2, sb).astype(np.float32)
    e = E.tensor(cu(a)).mul(cu(b)).sub(E.tensor(cu(b))).div(E.tensor(cu(b)).add(1.0))
    y = e.eval(ctx).cpu().numpy()
    ref = (a.astype(np.float64) * b - b) / (b + 1.0)
    assert y.shape == ref.shape and np.abs(y - ref).max() < 1e-5
    p = E.tensor(cu(np.abs(a) + 0.1)).pow(E.tensor(cu(b))).eval(ctx).cpu().numpy()
    assert np.abs(p / np.power(np.abs(a.astype(np.float64)) + 0.1, b) - 1).max() < 1e-5


@pytest.mark.parametrize("sa,sb", [((5,), (5,)), ((5,), (5, 3)), ((4, 5), (5,)), ((7, 33), (33, 9)),
                                   ((3, 7, 33), (3, 33, 9)), ((2, 1, 7, 33), (4, 33, 9)), ((3, 5, 64), (64, 48))])
def test_matmul_shapes_vs_numpy(ctx, sa, sb):
    from tenzor_b200 import expr as E
    rng = np.random.default_rng(sum(sa) + sum(sb))
    a = rng.uniform(-1, 1, sa).astype(np.float32)
    b = rng.uniform(-1, 1, sb).astype(np.float32)
    ref = np.matmul(a.astype(np.float64), b.astype(np.float64))
    y = E.tensor(cu(a)).matmul(cu(b)).eval(ctx).cpu().numpy()
    assert y.shape == ref.shape
    k = sa[-1]
    tf32 = len(sb) == 2 and len(sa) >= 2  # 2-D and [B, M, K] @ [K, N] products: one tf32 tensor-core pass
    tol = 4e-3 * np.sqrt(k) if tf32 else 1e-5 * k
    assert np.abs(y - ref).max() <= tol, float(np.abs(y - ref).max())
    if len(sa) == 2 and len(sb) == 2:  # the split-tf32 form of the 2-D product is f32-accurate
        y3 = E.matmul(cu(a), cu(b), precision="f32x3").eval(ctx).cpu().numpy()
        assert np.abs(y3 - ref).max() <= 1e-5 * k


@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "prod"])
@pytest.mark.parametrize("shape,axis", [((6, 7, 5), 0), ((6, 7, 5), 1), ((6, 7, 5), 2), ((1000, 384), -1),
                                        ((3, 4096, 2), 1)])
def test_reduce_axis_vs_numpy(ctx, op, shape, axis):
    from tenzor_b200 import expr as E
    rng = np.random.default_rng(3)
    x = rng.uniform(0.9, 1.1, shape).astype(np.float32) if op == "prod" else rng.normal(0, 1, shape).astype(np.float32)
    for keep in (False, True):
        y = getattr(E.tensor(cu(x)), op)(axis, keep).eval(ctx).cpu().numpy()
        fn = {"sum": np.sum, "mean": np.mean, "max": np.max, "min": np.min, "prod": np.prod}[op]
        ref = fn(x.astype(np.float64), axis=axis, keepdims=keep)
        assert y.shape == ref.shape
        assert np.abs(y - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))
    # a reduce over an elementwise chain (the reduce_epilogue plan) keeps the axis form
    y = E.tensor(cu(x)).abs().sqrt().sum(axis).eval(ctx).cpu().numpy()
    assert np.abs(y - np.sqrt(np.abs(x.astype(np.float64))).sum(axis)).max() < 1e-3


@pytest.mark.parametrize("shape,axis", [((4, 9, 6), 0), ((4, 9, 6), 1), ((2, 12, 16, 16), 1), ((96, 128, 128), -1)])
def test_softmax_any_axis_vs_numpy(ctx, shape, axis):
    from tenzor_b200 import expr as E
    x = np.random.default_rng(4).normal(0, 3, shape).astype(np.float32)
    y = E.tensor(cu(x)).softmax(axis).eval(ctx).cpu().numpy()
    e = np.exp(x.astype(np.float64) - x.max(axis, keepdims=True))
    ref = e / e.sum(axis, keepdims=True)
    assert np.abs(y - ref).max() < 1e-6


def test_permute_cast_concat(ctx):
    from tenzor_b200 import ops
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (2, 3, 4, 5, 6)).astype(np.float32)
    for perm in [(4, 3, 2, 1, 0), (0, 2, 1, 3, 4), (1, 0, 4, 2, 3)]:
        assert np.array_equal(ops.permute(ctx, cu(x), list(perm)).cpu().numpy(), x.transpose(perm))
    h = torch.from_numpy(x.astype(np.float16)).cuda()
    assert np.array_equal(ops.permute(ctx, h, [2, 0, 1, 4, 3]).cpu().numpy(), x.astype(np.float16).transpose(2, 0, 1, 4, 3))
    i = torch.arange(-5, 5, dtype=torch.int64).cuda()
    assert (ops.cast(ctx, i, torch.float32).cpu().numpy() == np.arange(-5, 5)).all()
    f = cu([-2.7, -0.5, 0.0, 0.5, 2.7, 1e6])
    assert (ops.cast(ctx, f, torch.int32).cpu().numpy() == [-2, 0, 0, 0, 2, 1000000]).all()
    assert (ops.cast(ctx, f, torch.uint8).cpu().numpy() == [1, 1, 0, 1, 1, 1]).all()
    parts = [rng.normal(0, 1, (3, n, 4)).astype(np.float32) for n in (1, 5, 2)]
    y = ops.concat(ctx, [cu(p) for p in parts], 1).cpu().numpy()
    assert np.array_equal(y, np.concatenate(parts, 1))
