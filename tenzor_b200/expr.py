"""Expression graphs and their CUDA evaluation: the host-side mirror of the reference's `.eval()` path
(src/ops/expr.zig node types, src/backend/cpu/executor.zig evalInto) with the fusion planner of
src/fusion/analyzer.zig deciding how each graph becomes launches of libtenzor_cuda.so.

Nodes: Tensor (leaf, a device tensor), Constant, Unary, Binary (2-D numpy-style broadcasting, as
executor.zig:152-197), Matmul (A @ B), Reduce (full reduction), Softmax (last axis), LayerNorm
(last axis, eps 1e-5 as executor.zig:420 hard-codes), Gather (rows of a table).

`analyze(expr)` restates analyzePattern (analyzer.zig:106-153): single / elementwise_chain /
matmul_epilogue / reduce_epilogue (the reference's fused_reduce pattern is never produced by
analyzePattern either).  `evaluate(ctx, expr)` lowers the plan:

  matmul_epilogue   -> tz_matmul_epilogue with the collected epilogue ops (collectEpilogueOps,
                       analyzer.zig:268-301); a [n] / [1, n] operand of an `add` is the bias
  elementwise_chain -> tz_ew_add_mul_exp for exp((a + b_row) * c), tz_ew_unary_chain for a unary
                       chain over one tensor, else one tz_ew_program_run over the whole graph
  reduce_epilogue   -> tz_reduce with the unary pre-ops
  single            -> the node's own kernel (layernorm, softmax, gather, matmul, reduce, ...)

There is no CPU fallback: every value is computed on the device by the library.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib as L
from . import ops
from .runtime import Context

UNARY = ("relu", "gelu", "sigmoid", "tanh", "exp", "neg", "abs", "silu", "log", "sqrt", "rsqrt", "sin", "cos",
         "erf", "gelu_erf")
BINARY = ("add", "sub", "mul", "div", "max", "min")
REDUCE = ("sum", "mean", "prod", "max", "min")


def _bshape(a, b):
    """numpy broadcast of two shapes (executor.zig's broadcast rule)."""
    n = max(len(a), len(b))
    a = (1,) * (n - len(a)) + tuple(a)
    b = (1,) * (n - len(b)) + tuple(b)
    out = []
    for x, y in zip(a, b):
        if x != y and 1 not in (x, y):
            raise ValueError(f"shapes {a} and {b} do not broadcast")
        out.append(max(x, y))
    return tuple(out)


class Expr:
    kind = "expr"
    shape: tuple = ()

    # builder methods mirroring the reference's fluent API (README: a.add(b).eval(...))
    def add(self, o): return Binary("add", self, _wrap(o))
    def sub(self, o): return Binary("sub", self, _wrap(o))
    def mul(self, o): return Binary("mul", self, _wrap(o))
    def div(self, o): return Binary("div", self, _wrap(o))
    def maximum(self, o): return Binary("max", self, _wrap(o))
    def minimum(self, o): return Binary("min", self, _wrap(o))
    def matmul(self, o): return Matmul(self, _wrap(o))
    def sum(self): return Reduce("sum", self)
    def mean(self): return Reduce("mean", self)
    def max(self): return Reduce("max", self)
    def min(self): return Reduce("min", self)
    def prod(self): return Reduce("prod", self)
    def softmax(self): return Softmax(self)
    def layer_norm(self, gamma, beta): return LayerNorm(self, _wrap(gamma), _wrap(beta))

    def eval(self, ctx: Context):
        return evaluate(ctx, self)


def _unary_method(op):
    def f(self):
        return Unary(op, self)
    return f


for _op in UNARY:
    setattr(Expr, _op, _unary_method(_op))


@dataclass(eq=False)
class Tensor(Expr):
    data: torch.Tensor
    kind = "tensor"

    def __post_init__(self):
        self.shape = tuple(self.data.shape)


@dataclass(eq=False)
class Constant(Expr):
    value: float
    kind = "constant"
    shape: tuple = ()


@dataclass(eq=False)
class Unary(Expr):
    op: str
    input: Expr
    kind = "unary"

    def __post_init__(self):
        assert self.op in UNARY, self.op
        self.shape = self.input.shape


@dataclass(eq=False)
class Binary(Expr):
    op: str
    lhs: Expr
    rhs: Expr
    kind = "binary"

    def __post_init__(self):
        assert self.op in BINARY, self.op
        self.shape = _bshape(self.lhs.shape, self.rhs.shape)


@dataclass(eq=False)
class Matmul(Expr):
    a: Expr
    b: Expr
    trans_b: bool = False
    kind = "matmul"

    def __post_init__(self):
        m, k = self.a.shape
        n = self.b.shape[0] if self.trans_b else self.b.shape[1]
        kb = self.b.shape[1] if self.trans_b else self.b.shape[0]
        if k != kb:
            raise ValueError(f"matmul inner dims {k} != {kb}")
        self.shape = (m, n)


@dataclass(eq=False)
class Reduce(Expr):
    op: str
    input: Expr
    kind = "reduce"

    def __post_init__(self):
        assert self.op in REDUCE
        self.shape = ()


@dataclass(eq=False)
class Softmax(Expr):
    input: Expr
    kind = "softmax"

    def __post_init__(self):
        self.shape = self.input.shape


@dataclass(eq=False)
class LayerNorm(Expr):
    input: Expr
    gamma: Expr
    beta: Expr
    eps: float = 1e-5  # executor.zig:420
    kind = "layernorm"

    def __post_init__(self):
        self.shape = self.input.shape


@dataclass(eq=False)
class Gather(Expr):
    table: Expr
    ids: torch.Tensor
    kind = "gather"

    def __post_init__(self):
        self.shape = (int(self.ids.numel()), self.table.shape[1])


def _wrap(x):
    if isinstance(x, Expr):
        return x
    if isinstance(x, torch.Tensor):
        return Tensor(x)
    return Constant(float(x))


def tensor(t: torch.Tensor) -> Tensor:
    return Tensor(t)


def matmul(a, b, trans_b=False) -> Matmul:
    return Matmul(_wrap(a), _wrap(b), trans_b)


def gather(table, ids) -> Gather:
    return Gather(_wrap(table), ids)


# ---- analyzer.zig restated ------------------------------------------------------------------------
def has_matmul_in_chain(e: Expr) -> bool:
    if e.kind == "matmul":
        return True
    if e.kind == "unary":
        return has_matmul_in_chain(e.input)
    if e.kind == "binary":
        return has_matmul_in_chain(e.lhs) or has_matmul_in_chain(e.rhs)
    return False


def is_elementwise_or_leaf(e: Expr) -> bool:
    return e.kind in ("tensor", "constant", "unary", "binary")


def is_elementwise_chain(e: Expr) -> bool:
    if e.kind in ("tensor", "constant"):
        return True
    if e.kind == "unary":
        return is_elementwise_chain(e.input)
    if e.kind == "binary":
        return is_elementwise_or_leaf(e.lhs) and is_elementwise_or_leaf(e.rhs)
    return False


def analyze(e: Expr) -> str:
    """analyzePattern, analyzer.zig:106-153."""
    if e.kind in ("tensor", "constant"):
        return "single"
    if e.kind == "unary":
        if has_matmul_in_chain(e.input):
            return "matmul_epilogue"
        if e.input.kind in ("unary", "binary") and is_elementwise_chain(e):
            return "elementwise_chain"
        return "single"
    if e.kind == "binary":
        if has_matmul_in_chain(e.lhs) or has_matmul_in_chain(e.rhs):
            return "matmul_epilogue"
        if is_elementwise_chain(e):
            return "elementwise_chain"
        return "single"
    if e.kind == "reduce":
        if e.input.kind in ("unary", "binary") and is_elementwise_chain(e.input):
            return "reduce_epilogue"
        return "single"
    return "single"


def find_matmul_base(e: Expr):
    """findMatmulBase, analyzer.zig:240-257."""
    if e.kind == "matmul":
        return e
    if e.kind == "unary":
        return find_matmul_base(e.input)
    if e.kind == "binary":
        if e.lhs.kind == "matmul":
            return e.lhs
        if e.rhs.kind == "matmul":
            return e.rhs
        return find_matmul_base(e.lhs) or find_matmul_base(e.rhs)
    return None


def collect_epilogue(e: Expr, out: list):
    """collectEpilogueOps, analyzer.zig:268-301: (op, other-operand) in chain order."""
    if e.kind == "matmul":
        return
    if e.kind == "unary":
        collect_epilogue(e.input, out)
        out.append((e.op, None))
    elif e.kind == "binary":
        if has_matmul_in_chain(e.lhs):
            collect_epilogue(e.lhs, out)
            out.append((e.op, e.rhs))
        else:
            collect_epilogue(e.rhs, out)
            out.append((e.op, e.lhs))


def collect_unary_chain(e: Expr):
    """Unary ops of a chain over one leaf, innermost first (collectElementwiseOps for unary chains)."""
    ops_ = []
    while e.kind == "unary":
        ops_.append(e.op)
        e = e.input
    return (list(reversed(ops_)), e) if e.kind == "tensor" else (None, None)


@dataclass
class Plan:
    pattern: str
    epilogue: list = field(default_factory=list)


def plan(e: Expr) -> Plan:
    p = Plan(analyze(e))
    if p.pattern == "matmul_epilogue":
        collect_epilogue(e, p.epilogue)
    return p


# ---- evaluation ---------------------------------------------------------------------------------
def _dev(shape):
    return torch.empty(shape, device="cuda", dtype=torch.float32)


def _as2d(shape):
    if len(shape) == 0:
        return 1, 1
    if len(shape) == 1:
        return 1, shape[0]
    rows = 1
    for s in shape[:-1]:
        rows *= s
    return rows, shape[-1]


def _strides2d(src_shape, out_shape):
    """(row_stride, col_stride) that read a broadcast source as the 2-D view of out_shape."""
    orow, ocol = _as2d(out_shape)
    if len(src_shape) == 0:
        return 0, 0
    s = (1,) * (len(out_shape) - len(src_shape)) + tuple(src_shape)
    if s == tuple(out_shape):
        return ocol, 1
    lead = s[:-1]
    if all(d == 1 for d in lead) and s[-1] == out_shape[-1]:
        return 0, 1  # row vector broadcast along rows
    if s[-1] == 1 and tuple(lead) == tuple(out_shape[:-1]):
        return 1, 0  # column vector broadcast along columns
    raise NotImplementedError(f"broadcast of {src_shape} to {out_shape} is not a 2-D row/column broadcast")


def _eval_leaf(ctx, e: Expr) -> torch.Tensor:
    if e.kind == "tensor":
        if not (e.data.is_cuda and e.data.dtype == torch.float32):
            raise TypeError("expression leaves must be f32 CUDA tensors to be evaluated")
        return e.data.contiguous()
    if e.kind == "constant":
        # a one-element device buffer (host -> device copy) read with stride 0
        return torch.tensor([e.value], dtype=torch.float32).to("cuda")
    return evaluate(ctx, e)


def _program(ctx, e: Expr) -> torch.Tensor:
    """Compile an elementwise graph into one tz_ew_program_run launch (inputs become leaves)."""
    prog = L.EwProgram()
    leaves, keep = [], []
    instr = []
    nxt = [4]

    consts = []

    def operand(x):
        if x.kind in ("unary", "binary"):
            return emit(x)
        if x.kind == "constant":  # immediates live in registers 12..15
            if x.value not in consts:
                if len(consts) == 4:
                    raise NotImplementedError("more than 4 distinct constants in one elementwise program")
                consts.append(x.value)
            return 12 + consts.index(x.value)
        t = _eval_leaf(ctx, x)
        keep.append(t)
        shape = () if x.kind == "constant" else tuple(t.shape)
        for i, (lt, _) in enumerate(leaves):
            if lt is t:
                return i
        if len(leaves) == 4:
            raise NotImplementedError("more than 4 distinct inputs in one elementwise program")
        leaves.append((t, shape))
        return len(leaves) - 1

    def emit(x):
        if x.kind == "unary":
            a = operand(x.input)
            op, b = L.OP[x.op], 0
        else:
            a = operand(x.lhs)
            b = operand(x.rhs)
            op = L.EW_BINARY[x.op]
        if nxt[0] >= 12 or len(instr) >= 16:
            raise NotImplementedError("elementwise program longer than 16 instructions")
        d = nxt[0]
        nxt[0] += 1
        instr.append((op, d, a, b))
        return d

    res = emit(e)
    out = _dev(e.shape)
    prog.n_inputs = len(leaves)
    for i, (t, shape) in enumerate(leaves):
        prog.in_[i] = t.data_ptr()
        rs, cs = _strides2d(shape, e.shape)
        prog.row_stride[i] = rs
        prog.col_stride[i] = cs
    prog.n_instr = len(instr)
    for i, (op, d, a, b) in enumerate(instr):
        prog.instr[i].op, prog.instr[i].dst, prog.instr[i].a, prog.instr[i].b = op, d, a, b
    prog.result = res
    for i, v in enumerate(consts):
        prog.consts[i] = v
    rows, cols = _as2d(e.shape)
    L.check(L.lib().tz_ew_program_run(ctx.handle, C.byref(prog), out.data_ptr(), rows, cols, ops._stream()))
    return out


def _match_add_mul_exp(e: Expr):
    """exp(mul(add(a, b_row), c)) with b a row vector: the configs[2](b) chain."""
    if e.kind == "unary" and e.op == "exp" and e.input.kind == "binary" and e.input.op == "mul":
        m = e.input
        if m.lhs.kind == "binary" and m.lhs.op == "add" and m.rhs.kind == "tensor":
            a, b, c = m.lhs.lhs, m.lhs.rhs, m.rhs
            if a.kind == "tensor" and b.kind == "tensor" and len(b.shape) == 1 and a.shape == c.shape \
                    and a.shape[-1] == b.shape[0]:
                return a.data, b.data, c.data
    return None


def evaluate(ctx: Context, e: Expr) -> torch.Tensor:
    """executor.evalInto (executor.zig:49-93) with FusionPlan-driven CUDA launches."""
    p = plan(e)
    if p.pattern == "matmul_epilogue":
        base = find_matmul_base(e)
        chain = []
        ok = True
        n = base.shape[1]
        bias = None
        for op, other in p.epilogue:
            if op in UNARY:
                chain.append(op)
            elif op == "add" and other is not None and bias is None and other.kind == "tensor" \
                    and other.shape in ((n,), (1, n)):
                chain.append("add")
                bias = other.data.reshape(-1)
            else:
                ok = False
                break
        if ok and len(chain) <= 8:
            a = _eval_leaf(ctx, base.a)
            b = _eval_leaf(ctx, base.b)
            return ops.matmul_epilogue(ctx, a, b, bias, chain, trans_b=base.trans_b)
        # epilogue not expressible as bias + activations: matmul, then the rest as a program
        mm = evaluate(ctx, base)
        return _program(ctx, _replace(e, base, Tensor(mm)))
    if p.pattern == "elementwise_chain":
        m = _match_add_mul_exp(e)
        if m is not None and not all(t.is_cuda and t.dtype == torch.float32 for t in m):
            raise TypeError("expression leaves must be f32 CUDA tensors to be evaluated")
        if m is not None:
            return ops.ew_add_mul_exp(ctx, *m)
        chain, leaf = collect_unary_chain(e)
        if chain is not None and len(chain) <= 8:
            return ops.ew_unary_chain(ctx, _eval_leaf(ctx, leaf), chain)
        return _program(ctx, e)
    if p.pattern == "reduce_epilogue":
        chain, leaf = collect_unary_chain(e.input)
        if chain is not None and len(chain) <= 8:
            return ops.reduce(ctx, e.op, chain, _eval_leaf(ctx, leaf))
        return ops.reduce(ctx, e.op, [], _program(ctx, e.input))
    # single
    k = e.kind
    if k in ("tensor", "constant"):
        return _eval_leaf(ctx, e)
    if k == "unary":
        x = _eval_leaf(ctx, e.input)
        return ops.ew_unary_chain(ctx, x.contiguous(), [e.op])
    if k == "binary":
        return _program(ctx, Binary(e.op, Tensor(_eval_leaf(ctx, e.lhs)) if e.lhs.kind not in ("tensor", "constant") else e.lhs,
                                    Tensor(_eval_leaf(ctx, e.rhs)) if e.rhs.kind not in ("tensor", "constant") else e.rhs))
    if k == "matmul":
        return ops.matmul_epilogue(ctx, _eval_leaf(ctx, e.a), _eval_leaf(ctx, e.b), None, [], trans_b=e.trans_b)
    if k == "reduce":
        return ops.reduce(ctx, e.op, [], _eval_leaf(ctx, e.input).contiguous())
    if k == "softmax":
        return ops.softmax_last_axis(ctx, _eval_leaf(ctx, e.input).contiguous())
    if k == "layernorm":
        return ops.layer_norm_last_dim(ctx, _eval_leaf(ctx, e.input).contiguous(), _eval_leaf(ctx, e.gamma),
                                       _eval_leaf(ctx, e.beta), e.eps)
    if k == "gather":
        return ops.gather_rows(ctx, _eval_leaf(ctx, e.table), e.ids)
    raise NotImplementedError(k)


def _replace(e: Expr, old: Expr, new: Expr) -> Expr:
    if e is old:
        return new
    if e.kind == "unary":
        return Unary(e.op, _replace(e.input, old, new))
    if e.kind == "binary":
        return Binary(e.op, _replace(e.lhs, old, new), _replace(e.rhs, old, new))
    return e
