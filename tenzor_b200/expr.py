"""Expression graphs and their CUDA evaluation: the host-side mirror of the reference's `.eval()` path
(src/ops/expr.zig node types, src/backend/cpu/executor.zig evalInto) with the fusion planner of
src/fusion/analyzer.zig deciding how each graph becomes launches of libtenzor_cuda.so.

Nodes: Tensor (leaf, a device tensor), Constant, Unary, Binary (numpy-style broadcasting of any rank
up to 6, as executor.zig:152-197), Matmul (evalMatmul, executor.zig:199-325: dot, vector-matrix,
matrix-vector, 2-D and batched with broadcast batch dimensions), Reduce (full, or over one axis with
keep_dims: executor.zig:327-361), Softmax (any axis: softmax.zig:157-220), LayerNorm (last axis, eps
1e-5 as executor.zig:420 hard-codes), Gather (rows of a table), Transpose and Reshape (expr.zig
TransposeExpr / ReshapeExpr).

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
         "erf", "gelu_erf", "erf_as", "gelu_tanh")
BINARY = ("add", "sub", "mul", "div", "max", "min", "pow", "eq", "lt", "gt")
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
    def pow(self, o): return Binary("pow", self, _wrap(o))
    def matmul(self, o): return Matmul(self, _wrap(o))
    def sum(self, axis=None, keep_dims=False): return Reduce("sum", self, axis, keep_dims)
    def mean(self, axis=None, keep_dims=False): return Reduce("mean", self, axis, keep_dims)
    def max(self, axis=None, keep_dims=False): return Reduce("max", self, axis, keep_dims)
    def min(self, axis=None, keep_dims=False): return Reduce("min", self, axis, keep_dims)
    def prod(self, axis=None, keep_dims=False): return Reduce("prod", self, axis, keep_dims)
    def softmax(self, axis=-1): return Softmax(self, axis)
    def layer_norm(self, gamma, beta): return LayerNorm(self, _wrap(gamma), _wrap(beta))
    def transpose(self, perm): return Transpose(self, tuple(perm))
    def reshape(self, shape): return Reshape(self, tuple(shape))

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
    """evalMatmul (executor.zig:199-325) shapes: [K]@[K] -> (), [K]@[K,N] -> [N], [M,K]@[K] -> [M],
    [M,K]@[K,N] -> [M,N], and batched [..., M, K] @ [..., K, N] with numpy-broadcast batch dims.
    `trans_b` (2-D only) reads b as [N, K]; `precision` is the 2-D tensor-core form: "tf32" or
    "f32x3" (split tf32, f32-accurate products)."""
    a: Expr
    b: Expr
    trans_b: bool = False
    precision: str = "tf32"
    kind = "matmul"

    def __post_init__(self):
        sa, sb = tuple(self.a.shape), tuple(self.b.shape)
        if self.trans_b:
            if len(sa) != 2 or len(sb) != 2:
                raise ValueError("trans_b needs 2-D operands")
            sb = (sb[1], sb[0])
        if not sa or not sb:
            raise ValueError("matmul of a scalar")
        ka = sa[-1]
        kb = sb[0] if len(sb) == 1 else sb[-2]
        if ka != kb:
            raise ValueError(f"matmul inner dims {ka} != {kb}")
        if len(sa) == 1 and len(sb) == 1:
            self.shape = ()
        elif len(sa) == 1:
            self.shape = sb[:-2] + (sb[-1],)
        elif len(sb) == 1:
            self.shape = sa[:-1]
        else:
            self.shape = _bshape(sa[:-2], sb[:-2]) + (sa[-2], sb[-1])


@dataclass(eq=False)
class Reduce(Expr):
    """ReduceExpr: over every element (axis None) or one axis (reduceAxis), keep_dims as given."""
    op: str
    input: Expr
    axis: object = None
    keep_dims: bool = False
    kind = "reduce"

    def __post_init__(self):
        assert self.op in REDUCE
        ish = tuple(self.input.shape)
        if self.axis is None:
            self.shape = (1,) * len(ish) if self.keep_dims else ()
        else:
            ax = self.axis % len(ish)
            self.axis = ax
            self.shape = ish[:ax] + ((1,) if self.keep_dims else ()) + ish[ax + 1:]


@dataclass(eq=False)
class Softmax(Expr):
    input: Expr
    axis: int = -1
    kind = "softmax"

    def __post_init__(self):
        self.shape = self.input.shape


@dataclass(eq=False)
class Transpose(Expr):
    """TransposeExpr (expr.zig:927): output dimension d is input dimension perm[d]."""
    input: Expr
    perm: tuple
    kind = "transpose"

    def __post_init__(self):
        if sorted(self.perm) != list(range(len(self.input.shape))):
            raise ValueError(f"bad permutation {self.perm} for rank {len(self.input.shape)}")
        self.shape = tuple(self.input.shape[p] for p in self.perm)


@dataclass(eq=False)
class Reshape(Expr):
    """ReshapeExpr (expr.zig:856): the same elements in row-major order, a new shape (one -1 allowed)."""
    input: Expr
    target: tuple
    kind = "reshape"

    def __post_init__(self):
        n = 1
        for d in self.input.shape:
            n *= d
        t = list(self.target)
        if t.count(-1) > 1:
            raise ValueError("at most one -1 in a reshape")
        if -1 in t:
            known = 1
            for d in t:
                if d != -1:
                    known *= d
            t[t.index(-1)] = n // known if known else 0
        m = 1
        for d in t:
            m *= d
        if m != n:
            raise ValueError(f"cannot reshape {self.input.shape} to {self.target}")
        self.shape = tuple(t)


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


def matmul(a, b, trans_b=False, precision="tf32") -> Matmul:
    return Matmul(_wrap(a), _wrap(b), trans_b, precision)


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


def _is_2d_matmul(m: "Matmul") -> bool:
    return len(m.a.shape) == 2 and len(m.b.shape) == 2


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
    """(row_stride, col_stride) that read a broadcast source as the 2-D view of out_shape, or None
    when the broadcast is not a row / column broadcast of that view (then the N-D form is used)."""
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
    return None


def _bstrides(src_shape, out_shape):
    """broadcastStrides (core/strides.zig): element strides of a contiguous source read at every
    index of out_shape (0 along broadcast dimensions)."""
    s = (1,) * (len(out_shape) - len(src_shape)) + tuple(src_shape)
    st, acc = [0] * len(s), 1
    for d in range(len(s) - 1, -1, -1):
        st[d] = 0 if s[d] == 1 and out_shape[d] != 1 else acc
        acc *= s[d]
    return st


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
    return _launch_program(ctx, prog, leaves, instr, consts, res, e.shape)


def _launch_program(ctx, prog, leaves, instr, consts, res, out_shape):
    """One tz_ew_program_run launch (2-D row / column broadcasts) or tz_ew_program_run_nd (any
    other broadcast, rank <= 6).  instr: (op, dst, a, b[, c]) tuples."""
    out = _dev(out_shape)
    prog.n_inputs = len(leaves)
    s2d = [_strides2d(shape, out_shape) for _, shape in leaves]
    for i, (t, shape) in enumerate(leaves):
        prog.in_[i] = t.data_ptr()
        rs, cs = s2d[i] if s2d[i] is not None else (0, 0)
        prog.row_stride[i] = rs
        prog.col_stride[i] = cs
    prog.n_instr = len(instr)
    for i, ins in enumerate(instr):
        op, d, a, b = ins[:4]
        prog.instr[i].op, prog.instr[i].dst, prog.instr[i].a, prog.instr[i].b = op, d, a, b
        prog.instr[i].c = ins[4] if len(ins) > 4 else 0
    prog.result = res
    for i, v in enumerate(consts):
        prog.consts[i] = v
    if out.numel() == 0:
        return out
    if all(x is not None for x in s2d) and len(out_shape) >= 1:
        rows, cols = _as2d(out_shape)
        L.check(L.lib().tz_ew_program_run(ctx.handle, C.byref(prog), out.data_ptr(), rows, cols, ops._stream()))
        return out
    if len(out_shape) > L.MAX_DIMS:
        raise ValueError(f"rank {len(out_shape)} is above {L.MAX_DIMS}")
    lay = L.NdLayout()
    lay.ndim = len(out_shape)
    for d, n in enumerate(out_shape):
        lay.shape[d] = n
    for i, (t, shape) in enumerate(leaves):
        for d, st in enumerate(_bstrides(shape, out_shape)):
            lay.stride[i][d] = st
    L.check(L.lib().tz_ew_program_run_nd(ctx.handle, C.byref(prog), C.byref(lay), out.data_ptr(), ops._stream()))
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
    if p.pattern == "matmul_epilogue" and not _is_2d_matmul(find_matmul_base(e)):
        base = find_matmul_base(e)  # batched / vector products: the product, then the rest as a program
        mm = evaluate(ctx, base)
        return _program(ctx, _replace(e, base, Tensor(mm)))
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
            mm = _mm2d_fn(base.precision, a.shape[1])
            return mm(ctx, a, b, bias, chain, trans_b=base.trans_b)
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
    if p.pattern == "reduce_epilogue" and e.axis is not None:
        return _reduce_axis(ctx, e, _program(ctx, e.input))
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
        return _matmul(ctx, e)
    if k == "reduce":
        x = _eval_leaf(ctx, e.input).contiguous()
        if e.axis is not None:
            return _reduce_axis(ctx, e, x)
        r = ops.reduce(ctx, e.op, [], x)
        return r.reshape(e.shape)
    if k == "softmax":
        x = _eval_leaf(ctx, e.input).contiguous()
        if len(e.shape) <= 1 or e.axis % len(e.shape) == len(e.shape) - 1:
            return ops.softmax_last_axis(ctx, x.reshape(-1, x.shape[-1] if x.dim() else 1)).reshape(e.shape)
        return ops.softmax_axis(ctx, x, e.axis)
    if k == "transpose":
        return ops.permute(ctx, _eval_leaf(ctx, e.input).contiguous(), list(e.perm))
    if k == "reshape":
        return _eval_leaf(ctx, e.input).contiguous().reshape(e.shape)  # a view: no data moves
    if k == "layernorm":
        return ops.layer_norm_last_dim(ctx, _eval_leaf(ctx, e.input).contiguous(), _eval_leaf(ctx, e.gamma),
                                       _eval_leaf(ctx, e.beta), e.eps)
    if k == "gather":
        return ops.gather_rows(ctx, _eval_leaf(ctx, e.table), e.ids)
    raise NotImplementedError(k)


def _mm2d_fn(precision, k):
    """The 2-D tensor-core product: one tf32 pass, or split tf32 when asked for or when K is not a
    whole number of 16-byte TMA units (the split operands are padded to 32 columns)."""
    return ops.matmul_f32x3 if precision == "f32x3" or k % 4 else ops.matmul_epilogue


def _reduce_axis(ctx, e: Reduce, x):
    return ops.reduce_axis(ctx, e.op, x.contiguous(), e.axis, e.keep_dims)


def _matmul(ctx, e: Matmul):
    """evalMatmul (executor.zig:199-325): 2-D products and [B, M, K] @ [K, N] (flattened to one
    2-D GEMM, the batchedMatmulBroadcastB case) on the tcgen05 GEMM; vector and batched products
    with distinct or broadcast batch matrices on tz_batched_matmul."""
    a = _eval_leaf(ctx, e.a).contiguous()
    b = _eval_leaf(ctx, e.b).contiguous()
    mm = _mm2d_fn(e.precision, a.shape[-1])
    if a.dim() == 2 and b.dim() == 2:
        return mm(ctx, a, b, None, [], trans_b=e.trans_b)
    if a.dim() >= 3 and b.dim() == 2 and a.shape[-1] % 4 == 0 and b.shape[1] % 4 == 0:
        return mm(ctx, a.reshape(-1, a.shape[-1]), b, None, []).reshape(e.shape)
    sa = tuple(a.shape) if a.dim() >= 2 else (1,) + tuple(a.shape)   # [K] -> [1, K]
    sb = tuple(b.shape) if b.dim() >= 2 else tuple(b.shape) + (1,)   # [K] -> [K, 1]
    m, k, n = sa[-2], sa[-1], sb[-1]
    batch = _bshape(sa[:-2], sb[:-2])
    if len(batch) > 4:
        raise ValueError("more than 4 batch dimensions")

    def bstr(shape):
        full = (1,) * (len(batch) - len(shape[:-2])) + tuple(shape[:-2])
        mat, st, acc = shape[-2] * shape[-1], [0] * len(batch), shape[-2] * shape[-1]
        for d in range(len(batch) - 1, -1, -1):
            st[d] = 0 if full[d] == 1 else acc
            acc *= full[d]
        return st
    out = ops.batched_matmul(ctx, a, b, tuple(batch) + (m, n), batch, bstr(sa), bstr(sb), m, k, n, k, 1, n, 1)
    return out.reshape(e.shape)


def _replace(e: Expr, old: Expr, new: Expr) -> Expr:
    if e is old:
        return new
    if e.kind == "unary":
        return Unary(e.op, _replace(e.input, old, new))
    if e.kind == "binary":
        return Binary(e.op, _replace(e.lhs, old, new), _replace(e.rhs, old, new))
    return e
