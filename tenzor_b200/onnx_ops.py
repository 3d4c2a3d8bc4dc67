"""ONNX op map onto libtenzor_cuda.so: the CUDA side of the reference's runtime-shaped ONNX executor
(src/onnx/executor.zig: executeNode 953-1031 dispatching to execMatMul 1490, execGemm 4561-4637,
execLayerNorm 3306-3397, execSoftmax 2392-2462, execGather 1984, execUnaryOp/execBinaryOp 1034/1102).

`OP_MAP[op_type](ctx, inputs, attrs) -> outputs` for the ops an exported BERT/Arctic encoder graph
uses, and `run_graph` executing a topologically ordered node list like Executor.run (712-816) does
with its ready scan.  Values are f32 CUDA tensors; every op runs in the library (no CPU fallback).
Deviation from the reference, on purpose: LayerNormalization honours the node's `epsilon`
attribute (the reference ignores it and uses 1e-5, executor.zig:3318); `ref_ln_eps=True` restores
the reference behaviour.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import expr as E
from . import ops
from .runtime import Context


def _2d(t):
    return t.reshape(-1, t.shape[-1])


def _matmul(ctx, ins, attrs):
    a, b = ins
    out = ops.matmul_epilogue(ctx, _2d(a).contiguous(), b.contiguous(), None, [])
    return [out.reshape(*a.shape[:-1], b.shape[-1])]


def _gemm(ctx, ins, attrs):
    a, b = ins[0], ins[1]
    c = ins[2] if len(ins) > 2 else None
    if attrs.get("transA", 0) or attrs.get("alpha", 1.0) != 1.0 or attrs.get("beta", 1.0) != 1.0:
        raise NotImplementedError("Gemm with transA/alpha/beta != defaults")
    trans_b = bool(attrs.get("transB", 0))
    n = b.shape[0] if trans_b else b.shape[1]
    bias = None
    chain = []
    if c is not None:
        if c.numel() != n:
            raise NotImplementedError("Gemm C must be a [N] bias")
        bias, chain = c.reshape(-1).contiguous(), ["add"]
    return [ops.matmul_epilogue(ctx, a.contiguous(), b.contiguous(), bias, chain, trans_b=trans_b)]


def _layernorm(ctx, ins, attrs, ref_eps=False):
    x, g, b = ins
    if attrs.get("axis", -1) not in (-1, x.dim() - 1):
        raise NotImplementedError("LayerNormalization over a non-last axis")
    eps = 1e-5 if ref_eps else float(attrs.get("epsilon", 1e-5))
    y = ops.layer_norm_last_dim(ctx, _2d(x).contiguous(), g.contiguous(), b.contiguous(), eps)
    return [y.reshape(x.shape)]


def _softmax(ctx, ins, attrs):
    (x,) = ins
    if attrs.get("axis", -1) not in (-1, x.dim() - 1):
        raise NotImplementedError("Softmax over a non-last axis")
    return [ops.softmax_last_axis(ctx, _2d(x).contiguous()).reshape(x.shape)]


def _gather(ctx, ins, attrs):
    table, idx = ins
    if attrs.get("axis", 0) != 0:
        raise NotImplementedError("Gather on axis != 0")
    ids = idx.reshape(-1).to(torch.int32) if idx.dtype != torch.int32 else idx.reshape(-1)
    out = ops.gather_rows(ctx, table.contiguous(), ids.contiguous())
    return [out.reshape(*idx.shape, table.shape[1])]


def _unary(op):
    def f(ctx, ins, attrs):
        (x,) = ins
        if op == "gelu_erf" and attrs.get("approximate", "none") == "tanh":
            return [ops.ew_unary_chain(ctx, x.contiguous(), ["gelu"])]
        return [ops.ew_unary_chain(ctx, x.contiguous(), [op])]
    return f


def _binary(op):
    def f(ctx, ins, attrs):
        a, b = ins
        return [E.evaluate(ctx, E.Binary(op, E.Tensor(a.contiguous()), E.Tensor(b.contiguous())))]
    return f


def _reshape(ctx, ins, attrs):
    x, shape = ins[0], [int(v) for v in ins[1].tolist()] if len(ins) > 1 else attrs["shape"]
    return [x.reshape(shape)]


OP_MAP = {
    "MatMul": _matmul,
    "Gemm": _gemm,
    "LayerNormalization": _layernorm,
    "Softmax": _softmax,
    "Gather": _gather,
    "Add": _binary("add"), "Sub": _binary("sub"), "Mul": _binary("mul"), "Div": _binary("div"),
    "Max": _binary("max"), "Min": _binary("min"),
    "Relu": _unary("relu"), "Tanh": _unary("tanh"), "Sigmoid": _unary("sigmoid"), "Exp": _unary("exp"),
    "Log": _unary("log"), "Sqrt": _unary("sqrt"), "Neg": _unary("neg"), "Abs": _unary("abs"),
    "Erf": _unary("erf"), "Gelu": _unary("gelu_erf"),
    "Reshape": _reshape,
}


@dataclass
class Node:
    op_type: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


def run_graph(ctx: Context, nodes, initializers: dict, feeds: dict, outputs, ref_ln_eps=False):
    """Executes nodes whose inputs are ready until all outputs exist (Executor.run's ready scan)."""
    env = dict(initializers)
    env.update(feeds)
    pending = list(nodes)
    while pending:
        progressed = False
        for n in list(pending):
            if all(i in env for i in n.inputs):
                fn = OP_MAP.get(n.op_type)
                if fn is None:
                    raise NotImplementedError(f"ONNX op {n.op_type} is not mapped to the CUDA backend")
                ins = [env[i] for i in n.inputs]
                outs = _layernorm(ctx, ins, n.attrs, ref_ln_eps) if n.op_type == "LayerNormalization" else fn(ctx, ins, n.attrs)
                for name, v in zip(n.outputs, outs):
                    env[name] = v
                pending.remove(n)
                progressed = True
        if not progressed:
            raise ValueError(f"graph has unsatisfiable nodes: {[n.op_type for n in pending]}")
    return [env[o] for o in outputs]
