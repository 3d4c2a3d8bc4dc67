"""NumPy restatement of the reference ONNX executor's op semantics for the ops of an exported
encoder graph, used as the checker of tenzor_b200.onnx_model / onnx_ops.  TEST INFRASTRUCTURE ONLY.

Follows src/onnx/executor.zig (reference default):
  execUnaryOp 1034 with the unary table 104-140: Gelu = x 0.5 (1 + tanh(0.7978845608 (x + 0.044715
    x^3))) (122), Erf = the Abramowitz-Stegun 7.1.26 polynomial in the order of 125-137, Relu, Tanh,
    Sigmoid, Exp, Log, Sqrt, Neg, Abs, Sin, Cos, Silu;
  execBinaryOp 1102 (numpy broadcasting), execPow 3558, execEqual 2656, execCompare, execWhere 2733;
  execMatMul 1490 (batched, numpy broadcasting of leading dims), execGemm 4561-4637 (transA, transB,
    alpha, beta, C broadcast);
  execLayerNorm 3306-3397: last axis, mean then mean of squared deviations, epsilon 1e-5 always;
  execSoftmax 2392-2462: the `axis` attribute, max-subtracted exp divided by the sum;
  execGather 1984, execConcat 2112, execReshape 2227 (0 copies the input extent), execTranspose 2296
    (default perm reverses), execSlice 2465, execConstant 2809, execShape 2828, execCast 2852,
    execUnsqueeze 3615 / execSqueeze 3709 (axes attribute or input), execExpand 3777,
    execReduceMean 4071 (axes attribute or input, keepdims default 1);
  execMultiHeadAttention 5763-5848: 8 heads always, scale 1/sqrt(head_dim), no mask.
`spec=True` restates the ONNX specification instead where the reference departs from it (Gelu's
`approximate` with exact erf, LayerNormalization's `epsilon`, MultiHeadAttention's `num_heads` and
key_padding_mask) -- the same switch as tenzor_b200.onnx_ops.run_graph.
Float arithmetic is f64 (the checker is at least as accurate as the f32 reference).
"""
from __future__ import annotations

import math

import numpy as np

_erf_exact = np.vectorize(math.erf, otypes=[np.float64])

_NP = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64, 9: np.bool_, 10: np.float16, 11: np.float64}


def erf_as(x):
    """executor.zig:125-137 (Abramowitz-Stegun 7.1.26)."""
    x = np.asarray(x, np.float64)
    ax = np.abs(x)
    t = 1.0 / (1.0 + 0.3275911 * ax)
    y = 1.0 - (((((1.061405429 * t + -1.453152027) * t) + 1.421413741) * t + -0.284496736) * t + 0.254829592) * t * np.exp(-ax * ax)
    return np.where(x < 0, -y, y)


def gelu_tanh(x):
    x = np.asarray(x, np.float64)
    return x * 0.5 * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * x * x * x)))


def gelu_erf(x):
    x = np.asarray(x, np.float64)
    return 0.5 * x * (1.0 + _erf_exact(x / math.sqrt(2.0)))


def _ln(x, g, b, eps):
    x = np.asarray(x, np.float64)
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * g + (0.0 if b is None else b)


def _softmax(x, axis):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis, keepdims=True))
    return e / e.sum(axis, keepdims=True)


def _ints(v):
    return [int(t) for t in np.asarray(v).reshape(-1)]


def _mha(q, k, v, nh, mask=None):
    q, k, v = (np.asarray(t, np.float64) for t in (q, k, v))
    B, Sq, H = q.shape
    Sk = k.shape[1]
    hd = H // nh
    qh = q.reshape(B, Sq, nh, hd).transpose(0, 2, 1, 3)
    kh = k.reshape(B, Sk, nh, hd).transpose(0, 2, 1, 3)
    vh = v.reshape(B, Sk, nh, hd).transpose(0, 2, 1, 3)
    s = qh @ kh.transpose(0, 1, 3, 2) / math.sqrt(hd)
    if mask is not None:
        s = s + (np.asarray(mask, np.float64).reshape(B, 1, 1, Sk) - 1.0) * 1e9
    p = _softmax(s, -1)
    return (p @ vh).transpose(0, 2, 1, 3).reshape(B, Sq, H)


def _f(v):
    return np.asarray(v, np.float64) if np.asarray(v).dtype.kind == "f" else np.asarray(v)


def run(nodes, initializers: dict, feeds: dict, outputs, spec: bool = False):
    env = {k: np.asarray(v) for k, v in initializers.items()}
    env.update({k: np.asarray(v) for k, v in feeds.items()})
    env[""] = None
    pending = list(nodes)
    while pending:
        progressed = False
        for n in list(pending):
            if not all(i in env for i in n.inputs):
                continue
            x = [env[i] for i in n.inputs]
            a = n.attrs
            op = n.op_type
            if op == "Gather":
                y = np.take(x[0], np.asarray(x[1]).astype(np.int64), axis=int(a.get("axis", 0)))
            elif op in ("Add", "Sub", "Mul", "Div", "Max", "Min", "Pow"):
                l, r = _f(x[0]), _f(x[1])
                if op == "Div" and l.dtype.kind in "iu" and r.dtype.kind in "iu":
                    y = l // r
                else:
                    y = {"Add": np.add, "Sub": np.subtract, "Mul": np.multiply, "Div": np.divide,
                         "Max": np.maximum, "Min": np.minimum, "Pow": np.power}[op](l, r)
            elif op in ("Equal", "Less", "Greater"):
                y = {"Equal": np.equal, "Less": np.less, "Greater": np.greater}[op](x[0], x[1])
            elif op == "Where":
                y = np.where(np.asarray(x[0]).astype(bool), _f(x[1]), _f(x[2]))
            elif op == "MatMul":
                y = np.matmul(_f(x[0]), _f(x[1]))
            elif op == "Gemm":
                A = x[0].T if a.get("transA", 0) else x[0]
                B = x[1].T if a.get("transB", 0) else x[1]
                y = float(a.get("alpha", 1.0)) * (_f(A) @ _f(B))
                if len(x) > 2 and x[2] is not None:
                    y = y + float(a.get("beta", 1.0)) * _f(x[2])
            elif op == "LayerNormalization":
                eps = float(a.get("epsilon", 1e-5)) if spec else 1e-5
                y = _ln(x[0], _f(x[1]), _f(x[2]) if len(x) > 2 and x[2] is not None else None, eps)
            elif op == "Softmax":
                y = _softmax(x[0], int(a.get("axis", -1)))
            elif op == "Gelu":
                y = gelu_erf(x[0]) if spec and a.get("approximate", "none") != "tanh" else gelu_tanh(x[0])
            elif op == "Erf":
                y = _erf_exact(_f(x[0])) if spec else erf_as(x[0])
            elif op in ("Relu", "Tanh", "Sigmoid", "Exp", "Log", "Sqrt", "Neg", "Abs", "Sin", "Cos", "Silu"):
                v = _f(x[0])
                y = {"Relu": lambda t: np.maximum(t, 0), "Tanh": np.tanh, "Sigmoid": lambda t: 1 / (1 + np.exp(-t)),
                     "Exp": np.exp, "Log": np.log, "Sqrt": np.sqrt, "Neg": np.negative, "Abs": np.abs,
                     "Sin": np.sin, "Cos": np.cos, "Silu": lambda t: t / (1 + np.exp(-t))}[op](v)
            elif op == "Reshape":
                tgt = _ints(x[1]) if len(x) > 1 else [int(t) for t in a["shape"]]
                tgt = [x[0].shape[i] if d == 0 else d for i, d in enumerate(tgt)]
                y = np.asarray(x[0]).reshape(tgt)
            elif op == "Transpose":
                y = np.transpose(x[0], a.get("perm"))
            elif op == "Concat":
                y = np.concatenate([np.atleast_1d(t) for t in x], axis=int(a["axis"]))
            elif op == "Shape":
                y = np.asarray(np.shape(x[0]), np.int64)
            elif op == "Constant":
                y = np.asarray(a.get("value", a.get("value_float", a.get("value_int", a.get("value_ints")))))
            elif op == "Cast":
                y = np.asarray(x[0]).astype(_NP[int(a["to"])])
            elif op in ("Unsqueeze", "Squeeze"):
                axes = _ints(x[1]) if len(x) > 1 and x[1] is not None else a.get("axes")
                t = np.asarray(x[0])
                if op == "Unsqueeze":
                    nd = t.ndim + len(axes)
                    y = np.expand_dims(t, tuple(sorted(ax % nd for ax in axes)))
                else:
                    y = np.squeeze(t, axis=None if axes is None else tuple(ax % t.ndim for ax in axes))
            elif op == "Slice":
                starts, ends = _ints(x[1]), _ints(x[2])
                axes = _ints(x[3]) if len(x) > 3 and x[3] is not None else list(range(len(starts)))
                steps = _ints(x[4]) if len(x) > 4 and x[4] is not None else [1] * len(starts)
                sl = [slice(None)] * np.ndim(x[0])
                for st, en, ax, sp in zip(starts, ends, axes, steps):
                    sl[ax % np.ndim(x[0])] = slice(st, en, sp)
                y = np.asarray(x[0])[tuple(sl)]
            elif op == "Expand":
                y = np.broadcast_to(x[0], np.broadcast_shapes(np.shape(x[0]), tuple(_ints(x[1])))).copy()
            elif op in ("ReduceMean", "ReduceSum", "ReduceMax", "ReduceProd"):
                axes = _ints(x[1]) if len(x) > 1 and x[1] is not None else a.get("axes")
                keep = bool(a.get("keepdims", 1))
                fn = {"ReduceMean": np.mean, "ReduceSum": np.sum, "ReduceMax": np.max, "ReduceProd": np.prod}[op]
                y = fn(_f(x[0]), axis=None if not axes else tuple(axes), keepdims=keep)
            elif op == "MultiHeadAttention":
                nh = int(a.get("num_heads", 8)) if spec else 8
                y = _mha(x[0], x[1], x[2], nh, x[4] if spec and len(x) > 4 else None)
            else:
                raise NotImplementedError(op)
            y = np.asarray(y)
            env[n.outputs[0]] = y.astype(np.float32) if y.dtype.kind == "f" else y
            pending.remove(n)
            progressed = True
        if not progressed:
            raise ValueError(f"unsatisfiable nodes: {[p.op_type for p in pending]}")
    return [env[o] for o in outputs]
