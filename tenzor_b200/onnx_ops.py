"""ONNX op map onto libtenzor_cuda.so: the CUDA side of the reference's runtime-shaped ONNX executor
(src/onnx/executor.zig: executeNode 953-1031 dispatching to execMatMul 1490, execGemm 4561-4637,
execLayerNorm 3306-3397, execSoftmax 2392-2462, execGather 1984, execConcat 2112, execReshape 2227,
execTranspose 2296, execSlice 2465, execEqual 2656, execWhere 2733, execConstant 2809, execShape
2828, execCast 2852, execPow 3558, execUnsqueeze 3615, execSqueeze 3709, execExpand 3777,
execReduceMean 4071, execMultiHeadAttention 5763-5848, execUnaryOp / execBinaryOp 1034 / 1102).

`OP_MAP[op_type](rt, inputs, attrs) -> outputs` and `run_graph`, which executes nodes as their
inputs become ready, like Executor.run (712-816).

Values.  Float data are f32 CUDA tensors and every op on them runs in the library.  Integer tensors
that describe shapes (the output of Shape and what is computed from it, integer Constants and
initializers such as axes or reshape targets) are small host arrays, as the reference keeps them in
its RuntimeTensor; ops whose inputs are all such arrays (Gather / Concat / Unsqueeze / Equal / Where
on shapes) are shape arithmetic on the host.  Integer graph inputs (input ids, attention masks) are
device tensors: gathers read them on the device and float ops convert them there (tz_cast).

Semantics.  By default each op does what the reference executor does:
  * Gelu is the tanh form 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) (executor.zig:122);
  * Erf is the Abramowitz-Stegun 7.1.26 polynomial (executor.zig:125-137, |error| <= 1.5e-7);
  * LayerNormalization uses epsilon 1e-5 whatever the node says (executor.zig:3318) and normalises
    the last axis;
  * MultiHeadAttention splits the hidden size into 8 heads whatever the node says and ignores the
    optional bias / mask inputs (executor.zig:5783-5785).
`spec=True` follows the ONNX specification instead (Gelu's `approximate` attribute with exact erf,
the device erff, LayerNormalization's `epsilon`, MultiHeadAttention's `num_heads` and its
key_padding_mask).  MatMul and Gemm run on the tcgen05 tensor cores with split-tf32 operands
(f32-accurate products, as the reference's f32 GEMMs); `precision="tf32"` selects one tf32 pass.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L
from . import expr as E
from . import ops
from .runtime import Context

# TensorProto.DataType -> torch / numpy (onnx.proto3)
_ONNX_TORCH = {1: torch.float32, 2: torch.uint8, 3: torch.int8, 6: torch.int32, 7: torch.int64, 9: torch.bool,
               10: torch.float16}
_ONNX_NP = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64, 9: np.bool_, 10: np.float16,
            11: np.float64}


@dataclass
class Runtime:
    ctx: Context
    spec: bool = False
    precision: str = "f32x3"


@dataclass
class Node:
    op_type: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


# ---- value helpers -----------------------------------------------------------------------------
def _c(a, dtype=None) -> np.ndarray:
    """A C-contiguous copy of the same rank (np.ascontiguousarray would turn a 0-d array into 1-d)."""
    return np.array(a, dtype=dtype, order="C", copy=True)


def _host(v) -> bool:
    return isinstance(v, np.ndarray) or np.isscalar(v)


def _f32(rt: Runtime, v) -> torch.Tensor:
    """A value as a contiguous f32 CUDA tensor (host arrays are copied up, integer device tensors
    converted by tz_cast)."""
    if _host(v):
        a = np.asarray(v)
        if a.dtype == np.float32:
            return torch.from_numpy(_c(a)).cuda()
        t = torch.from_numpy(_c(a.astype(np.int64) if a.dtype.kind in "biu" else a)).cuda()
        if t.dtype == torch.float32:
            return t
        if t.dtype == torch.float64:
            return torch.from_numpy(_c(a, np.float32)).cuda()
        return ops.cast(rt.ctx, t, torch.float32)
    v = v.contiguous()
    return v if v.dtype == torch.float32 else ops.cast(rt.ctx, v, torch.float32)


def _ints(v) -> list:
    """An integer tensor (shape, axes, indices) as a Python list (a host copy of a device value)."""
    if _host(v):
        return [int(x) for x in np.asarray(v).reshape(-1)]
    return [int(x) for x in v.reshape(-1).cpu().tolist()]


def _shape(v) -> list:
    return list(np.shape(v)) if _host(v) else list(v.shape)


def _attr_or_input(attrs, name, ins, idx):
    if len(ins) > idx and ins[idx] is not None:
        return _ints(ins[idx])
    if name in attrs:
        return [int(x) for x in attrs[name]]
    return None


# ---- elementwise on the device (one program launch) --------------------------------------------
def _program(rt: Runtime, values, instr, out_shape):
    """Runs an elementwise program over device values (broadcast to out_shape)."""
    prog = L.EwProgram()
    leaves = [(_f32(rt, v), tuple(_shape(v))) for v in values]
    res = instr[-1][1]
    return E._launch_program(rt.ctx, prog, leaves, instr, [], res, tuple(out_shape))


def _binary(op):
    np_op = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": None, "max": np.maximum,
             "min": np.minimum, "pow": np.power, "eq": np.equal, "lt": np.less, "gt": np.greater}[op]

    def f(rt, ins, attrs):
        a, b = ins
        if _host(a) and _host(b) and np.asarray(a).dtype.kind in "biu" and np.asarray(b).dtype.kind in "biu":
            a_, b_ = np.asarray(a), np.asarray(b)
            if op == "div":
                return [(a_ // b_).astype(np.result_type(a_, b_))]
            return [np_op(a_, b_)]
        shape = E._bshape(_shape(a), _shape(b))
        return [_program(rt, [a, b], [(L.EW_BINARY[op], 4, 0, 1)], shape)]
    return f


def _unary(op, spec_op=None):
    def f(rt, ins, attrs):
        (x,) = ins
        code = op
        if rt.spec and spec_op is not None:
            code = spec_op(attrs)
        return [ops.ew_unary_chain(rt.ctx, _f32(rt, x), [code])]
    return f


def _where(rt, ins, attrs):
    c, x, y = ins
    if all(_host(v) for v in ins):
        return [np.where(np.asarray(c).astype(bool), np.asarray(x), np.asarray(y))]
    shape = E._bshape(E._bshape(_shape(c), _shape(x)), _shape(y))
    return [_program(rt, [c, x, y], [(L.EW_WHERE, 4, 0, 1, 2)], shape)]


# ---- linear algebra ----------------------------------------------------------------------------
def _mm2d(rt, a, b, bias=None, chain=(), trans_b=False):
    f = E._mm2d_fn(rt.precision, a.shape[-1])
    return f(rt.ctx, a.contiguous(), b.contiguous(), bias, list(chain), trans_b=trans_b)


def _matmul(rt, ins, attrs):
    a, b = _f32(rt, ins[0]), _f32(rt, ins[1])
    if a.dim() >= 2 and b.dim() == 2:  # [.., M, K] @ [K, N]: one 2-D GEMM over the flattened rows
        out = _mm2d(rt, a.reshape(-1, a.shape[-1]), b)
        return [out.reshape(*a.shape[:-1], b.shape[-1])]
    return [E._matmul(rt.ctx, E.Matmul(E.Tensor(a), E.Tensor(b)))]


def _gemm(rt, ins, attrs):
    """execGemm (4561-4637): Y = alpha op(A) op(B) + beta C, C broadcast."""
    a, b = _f32(rt, ins[0]), _f32(rt, ins[1])
    alpha, beta = float(attrs.get("alpha", 1.0)), float(attrs.get("beta", 1.0))
    if attrs.get("transA", 0):
        a = ops.permute(rt.ctx, a, [1, 0])
    trans_b = bool(attrs.get("transB", 0))
    n = b.shape[0] if trans_b else b.shape[1]
    c = ins[2] if len(ins) > 2 else None
    if c is not None and alpha == 1.0 and beta == 1.0 and int(np.prod(_shape(c))) == n:
        return [_mm2d(rt, a, b, _f32(rt, c).reshape(-1), ["add"], trans_b)]
    y = _mm2d(rt, a, b, None, [], trans_b)
    instr, vals = [], [y]
    if alpha != 1.0:
        vals.append(np.full((), alpha, np.float32))
        instr.append((L.EW_BINARY["mul"], 4, 0, 1))
    if c is not None:
        vals.append(c)
        r = 4 if instr else 0
        if beta != 1.0:
            vals.append(np.full((), beta, np.float32))
            instr.append((L.EW_BINARY["mul"], 5, len(vals) - 2, len(vals) - 1))
            instr.append((L.EW_BINARY["add"], 6, r, 5))
        else:
            instr.append((L.EW_BINARY["add"], 5 if instr else 4, r, len(vals) - 1))
    if not instr:
        return [y]
    return [_program(rt, vals, instr, tuple(y.shape))]


# ---- normalisation / softmax ------------------------------------------------------------------
def _layernorm(rt, ins, attrs):
    x = _f32(rt, ins[0])
    g = _f32(rt, ins[1]).reshape(-1)
    b = _f32(rt, ins[2]).reshape(-1) if len(ins) > 2 and ins[2] is not None else torch.zeros_like(g)
    axis = int(attrs.get("axis", -1)) if rt.spec else -1
    eps = float(attrs.get("epsilon", 1e-5)) if rt.spec else 1e-5
    axis %= x.dim()
    cols = int(np.prod(x.shape[axis:]))
    y = ops.layer_norm_last_dim(rt.ctx, x.reshape(-1, cols), g, b, eps)
    return [y.reshape(x.shape)]


def _softmax(rt, ins, attrs):
    x = _f32(rt, ins[0])
    axis = int(attrs.get("axis", -1)) % x.dim()
    if axis == x.dim() - 1:
        return [ops.softmax_last_axis(rt.ctx, x.reshape(-1, x.shape[-1])).reshape(x.shape)]
    return [ops.softmax_axis(rt.ctx, x, axis)]


def _reduce(op):
    def f(rt, ins, attrs):
        """execReduceMean (4071) and its kin: axes from the attribute or (opset 13+) the second
        input; none = every axis (or a copy with noop_with_empty_axes); keepdims default 1."""
        x = ins[0]
        axes = _attr_or_input(attrs, "axes", ins, 1)
        keep = bool(attrs.get("keepdims", 1))
        if not axes:
            if attrs.get("noop_with_empty_axes", 0):
                return [x]
            axes = list(range(len(_shape(x))))
        if _host(x):
            a = np.asarray(x)
            fn = {"sum": np.sum, "mean": np.mean, "max": np.max, "min": np.min, "prod": np.prod}[op]
            return [fn(a, axis=tuple(axes), keepdims=keep)]
        y = _f32(rt, x)
        nd = y.dim()
        for ax in sorted((a_ % nd for a_ in axes), reverse=True):
            y = ops.reduce_axis(rt.ctx, op, y.contiguous(), ax, keepdims=True)
        if not keep:
            y = y.reshape([d for i, d in enumerate(y.shape) if i not in {a_ % nd for a_ in axes}])
        return [y]
    return f


# ---- gathers, shapes and data movement --------------------------------------------------------
def _gather(rt, ins, attrs):
    """execGather (1984): out = take(data, indices, axis), negative indices wrap."""
    data, idx = ins
    axis = int(attrs.get("axis", 0))
    if _host(data):
        a = np.asarray(data)
        return [np.take(a, np.asarray(idx).astype(np.int64), axis=axis % max(a.ndim, 1))]
    t = _f32(rt, data)
    axis %= t.dim()
    ishape = _shape(idx)
    inner = int(np.prod(t.shape[axis + 1:])) if axis + 1 < t.dim() else 1
    if axis == 0 and not _host(idx):  # device indices (an input_ids feed): converted on the device
        dev_ids = idx.contiguous() if idx.dtype == torch.int32 else ops.cast(rt.ctx, idx.contiguous(), torch.int32)
        out = ops.gather_rows(rt.ctx, t.reshape(-1, inner), dev_ids.reshape(-1))
        return [out.reshape(list(ishape) + list(t.shape[1:]))]
    ids = np.asarray(_ints(idx), np.int64)
    ln = t.shape[axis]
    ids = np.where(ids < 0, ids + ln, ids)
    outer = int(np.prod(t.shape[:axis])) if axis else 1
    if outer == 1:
        rows = ids
    else:  # rows of the [outer * len, inner] view
        rows = (np.arange(outer, dtype=np.int64)[:, None] * ln + ids[None, :]).reshape(-1)
    dev_ids = torch.from_numpy(rows.astype(np.uint32).view(np.int32)).cuda()
    out = ops.gather_rows(rt.ctx, t.reshape(-1, inner), dev_ids)
    return [out.reshape(list(t.shape[:axis]) + list(ishape) + list(t.shape[axis + 1:]))]


def _shape_op(rt, ins, attrs):
    s = _shape(ins[0])
    start, end = int(attrs.get("start", 0)), attrs.get("end")
    return [np.asarray(s[start:end] if end is not None else s[start:], np.int64)]


def _constant(rt, ins, attrs):
    if "value" in attrs:
        v = np.asarray(attrs["value"])
    elif "value_float" in attrs:
        v = np.asarray(attrs["value_float"], np.float32)
    elif "value_int" in attrs:
        v = np.asarray(attrs["value_int"], np.int64)
    elif "value_ints" in attrs:
        v = np.asarray(attrs["value_ints"], np.int64)
    else:
        raise NotImplementedError("Constant without value / value_float / value_int(s)")
    return [torch.from_numpy(_c(v, np.float32)).cuda() if v.dtype.kind == "f" and v.ndim else v]


def _reshape(rt, ins, attrs):
    x = ins[0]
    tgt = _ints(ins[1]) if len(ins) > 1 else [int(v) for v in attrs["shape"]]
    cur = _shape(x)
    tgt = [cur[i] if d == 0 and not attrs.get("allowzero", 0) else d for i, d in enumerate(tgt)]
    if _host(x):
        return [np.asarray(x).reshape(tgt)]
    return [x.contiguous().reshape(tgt)]


def _unsqueeze(rt, ins, attrs):
    x = ins[0]
    axes = _attr_or_input(attrs, "axes", ins, 1)
    nd = len(_shape(x)) + len(axes)
    shape = list(_shape(x))
    for a in sorted(a_ % nd for a_ in axes):
        shape.insert(a, 1)
    return [np.asarray(x).reshape(shape) if _host(x) else x.contiguous().reshape(shape)]


def _squeeze(rt, ins, attrs):
    x = ins[0]
    axes = _attr_or_input(attrs, "axes", ins, 1)
    s = _shape(x)
    keep = [d for i, d in enumerate(s) if (axes is not None and i not in {a % len(s) for a in axes})
            or (axes is None and d != 1)]
    return [np.asarray(x).reshape(keep) if _host(x) else x.contiguous().reshape(keep)]


def _flatten(rt, ins, attrs):
    x = ins[0]
    s = _shape(x)
    ax = int(attrs.get("axis", 1)) % (len(s) + 1)
    shape = [int(np.prod(s[:ax])), int(np.prod(s[ax:]))]
    return [np.asarray(x).reshape(shape) if _host(x) else x.contiguous().reshape(shape)]


def _transpose(rt, ins, attrs):
    x = ins[0]
    nd = len(_shape(x))
    perm = [int(p) for p in attrs.get("perm", list(range(nd))[::-1])]
    if _host(x):
        return [np.transpose(np.asarray(x), perm)]
    return [ops.permute(rt.ctx, x.contiguous(), perm)]


def _concat(rt, ins, attrs):
    axis = int(attrs["axis"])
    if all(_host(v) for v in ins):
        return [np.concatenate([np.atleast_1d(np.asarray(v)) for v in ins], axis=axis)]
    vals = [_f32(rt, v) for v in ins]
    return [ops.concat(rt.ctx, vals, axis % vals[0].dim())]


def _cast(rt, ins, attrs):
    x, to = ins[0], int(attrs["to"])
    if _host(x) and to not in (1, 10):  # integer / bool results of shape arithmetic stay on the host
        return [np.asarray(x).astype(_ONNX_NP[to])]
    if _host(x):  # an integer tensor entering float computation (e.g. an attention mask)
        a = np.asarray(x)
        x = torch.from_numpy(_c(a.astype(np.int64) if a.dtype.kind in "biu" else a)).cuda()
    want = _ONNX_TORCH[to]
    if want == torch.bool:
        want = torch.uint8
    return [x if x.dtype == want else ops.cast(rt.ctx, x.contiguous(), want)]


def _slice(rt, ins, attrs):
    """execSlice (2465): starts / ends / axes / steps inputs (opset 10+), clamped like numpy."""
    x = ins[0]
    starts, ends = _ints(ins[1]), _ints(ins[2])
    s = _shape(x)
    axes = _ints(ins[3]) if len(ins) > 3 and ins[3] is not None else list(range(len(starts)))
    steps = _ints(ins[4]) if len(ins) > 4 and ins[4] is not None else [1] * len(starts)
    if _host(x):
        sl = [slice(None)] * len(s)
        for st, en, ax, sp in zip(starts, ends, axes, steps):
            sl[ax % len(s)] = slice(st, en, sp)
        return [np.asarray(x)[tuple(sl)]]
    y = _f32(rt, x)
    for st, en, ax, sp in zip(starts, ends, axes, steps):
        ax %= y.dim()
        idx = np.arange(y.shape[ax])[slice(st, en, sp)]
        y = _gather(rt, [y, idx.astype(np.int64)], {"axis": ax})[0]
    return [y]


def _expand(rt, ins, attrs):
    x, shape = ins[0], _ints(ins[1])
    out = E._bshape(_shape(x), shape)
    if _host(x):
        return [np.broadcast_to(np.asarray(x), out).copy()]
    one = np.full((), 1.0, np.float32)
    return [_program(rt, [x, one], [(L.EW_BINARY["mul"], 4, 0, 1)], out)]


def _mha(rt, ins, attrs):
    """execMultiHeadAttention (5763-5848): query / key / value [B, S, H] -> [B, Sq, H]; head h uses
    columns h * hd .. (h + 1) * hd; softmax(Q K^T / sqrt(hd)) V per (batch, head).  The products read
    the interleaved head layout through strides (no transposes), on tz_batched_matmul."""
    q, k, v = (_f32(rt, t) for t in ins[:3])
    B, Sq, H = q.shape
    Sk = k.shape[1]
    nh = int(attrs.get("num_heads", 8)) if rt.spec else 8
    hd = H // nh
    if hd * nh != H:
        raise ValueError(f"hidden size {H} is not a multiple of {nh} heads")
    # scores [B, nh, Sq, Sk]: element (b, h, i, j) = sum_d q[b, i, h hd + d] k[b, j, h hd + d]
    s = ops.batched_matmul(rt.ctx, q, k, (B, nh, Sq, Sk), (B, nh), (Sq * H, hd), (Sk * H, hd), Sq, hd, Sk,
                           H, 1, 1, H)
    scale = np.full((), 1.0 / np.sqrt(np.float32(hd)), np.float32)
    vals, instr = [s, scale], [(L.EW_BINARY["mul"], 4, 0, 1)]
    if rt.spec and len(ins) > 4 and ins[4] is not None:  # key_padding_mask [B, Sk]: 0 = masked
        m = np.asarray(_ints(ins[4]), np.float32).reshape(B, 1, 1, Sk)
        vals.append((m - 1.0) * np.float32(1e9))
        instr.append((L.EW_BINARY["add"], 5, 4, 2))
    s = _program(rt, vals, instr, (B, nh, Sq, Sk))
    p = ops.softmax_last_axis(rt.ctx, s.reshape(-1, Sk))
    out = torch.empty((B, Sq, H), device=q.device, dtype=torch.float32)
    # out[b, i, h hd + d] = sum_j p[b, h, i, j] v[b, j, h hd + d]
    ops.batched_matmul(rt.ctx, p, v, None, (B, nh), (nh * Sq * Sk, Sq * Sk), (Sk * H, hd), Sq, Sk, hd,
                       Sk, 1, H, 1, out=out, c_view=((Sq * H, hd), H, 1))
    return [out]


def _gelu_spec(attrs):
    return "gelu_tanh" if attrs.get("approximate", "none") == "tanh" else "gelu_erf"


OP_MAP = {
    "MatMul": _matmul, "Gemm": _gemm,
    "LayerNormalization": _layernorm, "Softmax": _softmax,
    "Gather": _gather, "Shape": _shape_op, "Constant": _constant, "Reshape": _reshape,
    "Unsqueeze": _unsqueeze, "Squeeze": _squeeze, "Flatten": _flatten, "Transpose": _transpose,
    "Concat": _concat, "Cast": _cast, "Slice": _slice, "Expand": _expand, "Where": _where,
    "MultiHeadAttention": _mha,
    "ReduceMean": _reduce("mean"), "ReduceSum": _reduce("sum"), "ReduceMax": _reduce("max"),
    "ReduceProd": _reduce("prod"),
    "Add": _binary("add"), "Sub": _binary("sub"), "Mul": _binary("mul"), "Div": _binary("div"),
    "Max": _binary("max"), "Min": _binary("min"), "Pow": _binary("pow"), "Equal": _binary("eq"),
    "Less": _binary("lt"), "Greater": _binary("gt"),
    "Relu": _unary("relu"), "Tanh": _unary("tanh"), "Sigmoid": _unary("sigmoid"), "Exp": _unary("exp"),
    "Log": _unary("log"), "Sqrt": _unary("sqrt"), "Neg": _unary("neg"), "Abs": _unary("abs"),
    "Sin": _unary("sin"), "Cos": _unary("cos"), "Silu": _unary("silu"),
    "Erf": _unary("erf_as", lambda a: "erf"), "Gelu": _unary("gelu_tanh", _gelu_spec),
}


def run_graph(ctx: Context, nodes, initializers: dict, feeds: dict, outputs, spec: bool = False,
              precision: str = "f32x3"):
    """Executes nodes whose inputs are ready until all outputs exist (Executor.run's ready scan).
    Values: f32 CUDA tensors, or host integer arrays (shapes, indices, masks); see the module doc."""
    rt = Runtime(ctx, spec, precision)
    env = dict(initializers)
    env.update(feeds)
    env[""] = None  # an omitted optional input
    pending = list(nodes)
    while pending:
        progressed = False
        for n in list(pending):
            if all(i in env for i in n.inputs):
                fn = OP_MAP.get(n.op_type)
                if fn is None:
                    raise NotImplementedError(f"ONNX op {n.op_type} is not mapped to the CUDA backend")
                outs = fn(rt, [env[i] for i in n.inputs], n.attrs)
                for name, v in zip(n.outputs, outs):
                    env[name] = v
                pending.remove(n)
                progressed = True
        if not progressed:
            raise ValueError(f"graph has unsatisfiable nodes: {[n.op_type for n in pending]}")
    return [env[o] for o in outputs]
