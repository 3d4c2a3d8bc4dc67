"""NumPy restatement of the reference ONNX executor's op semantics for the ops of an encoder graph,
used as the checker of tenzor_b200.onnx_model / onnx_ops.  TEST INFRASTRUCTURE ONLY.

Follows src/onnx/executor.zig: execMatMul 1490 (f32 matmul, numpy broadcasting of leading dims),
execGemm 4561-4637 (optional transA/transB, C broadcast as a bias), execLayerNorm 3306-3397 (mean,
then mean of squared deviations, over the last axis), execSoftmax 2392-2462 (max-subtracted exp over
the last axis), execGather 1984 (axis 0), execUnaryOp 1034 / execBinaryOp 1102 (elementwise with
broadcasting).  LayerNormalization takes the node's epsilon, as the CUDA op map does by default.
"""
from __future__ import annotations

import math

import numpy as np

_erf = np.vectorize(math.erf, otypes=[np.float64])


def _ln(x, g, b, eps):
    x = x.astype(np.float64)
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return ((x - m) / np.sqrt(v + eps) * g + b).astype(np.float32)


def _softmax(x):
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def _gelu(x, approximate="none"):
    x = x.astype(np.float64)
    if approximate == "tanh":
        return (0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))).astype(np.float32)
    return (0.5 * x * (1 + _erf(x / math.sqrt(2.0)))).astype(np.float32)


def run(nodes, initializers: dict, feeds: dict, outputs):
    env = {k: np.asarray(v) for k, v in initializers.items()}
    env.update({k: np.asarray(v) for k, v in feeds.items()})
    for n in nodes:  # fixtures are written in topological order
        x = [env[i] for i in n.inputs]
        a = n.attrs
        op = n.op_type
        if op == "Gather":
            y = np.take(x[0], x[1].astype(np.int64), axis=int(a.get("axis", 0)))
        elif op == "Add":
            y = x[0] + x[1]
        elif op == "Sub":
            y = x[0] - x[1]
        elif op == "Mul":
            y = x[0] * x[1]
        elif op == "Div":
            y = x[0] / x[1]
        elif op == "MatMul":
            y = np.matmul(x[0].astype(np.float64), x[1].astype(np.float64))
        elif op == "Gemm":
            A = x[0].T if a.get("transA", 0) else x[0]
            B = x[1].T if a.get("transB", 0) else x[1]
            y = float(a.get("alpha", 1.0)) * (A.astype(np.float64) @ B.astype(np.float64))
            if len(x) > 2:
                y = y + float(a.get("beta", 1.0)) * x[2]
        elif op == "LayerNormalization":
            y = _ln(x[0], x[1], x[2], float(a.get("epsilon", 1e-5)))
        elif op == "Softmax":
            y = _softmax(x[0].astype(np.float64))
        elif op == "Gelu":
            y = _gelu(x[0], a.get("approximate", "none"))
        elif op == "Erf":
            y = _erf(x[0].astype(np.float64))
        elif op == "Relu":
            y = np.maximum(x[0], 0)
        elif op == "Tanh":
            y = np.tanh(x[0])
        elif op == "Reshape":
            y = x[0].reshape([int(v) for v in x[1]])
        else:
            raise NotImplementedError(op)
        env[n.outputs[0]] = np.asarray(y).astype(np.float32) if np.asarray(y).dtype.kind == "f" else np.asarray(y)
    return [env[o] for o in outputs]
