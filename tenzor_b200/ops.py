"""Op-level entry points on device tensors (torch CUDA tensors are used only as device memory;
every computation runs in libtenzor_cuda.so).  Names follow the reference kernels they replace:

  layer_norm_last_dim   layernorm.zig:26-116          softmax_last_axis   softmax.zig:20-155
  linear (f32)          arctic.zig:599-620 / matmul.zig:54-77 (tcgen05 kind::tf32)
  linear_w8a32          matmul_w8a32.zig:14-58        linear_w8a8         (W8A8, no counterpart)
  gemm_i8_i32           exact int32 accumulators      quantize_weight_rows  quantize_arctic_xs.zig:94-115
  matmul_epilogue       codegen.zig:78-147            ew_add_mul_exp      executor.zig:114-197
  ew_unary_chain        codegen.zig:15-74             reduce              codegen.zig:151-205
  gather_rows           gather.zig:15-57
N-D forms (executor.zig / onnx/executor.zig): batched_matmul, matmul_f32x3, reduce_axis, softmax_axis,
permute, cast, concat.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .runtime import Context


def _p(t):
    return None if t is None else t.data_ptr()


CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the handle torch's default stream (0) stands for


def _stream(s=None):
    """The stream to launch on: torch's current stream.  Its default stream has handle 0, which the C
    ABI reads as 'the context's own stream', so it is passed as cudaStreamLegacy instead."""
    h = torch.cuda.current_stream().cuda_stream if s is None else s
    return C.c_void_p(h if h else CUDA_STREAM_LEGACY)


def _dev(t, dtype):
    assert t.is_cuda and t.is_contiguous() and t.dtype == dtype, (t.device, t.dtype, t.is_contiguous())
    return t


def layer_norm_last_dim(ctx: Context, x, gamma, beta, eps: float, out=None):
    _dev(x, torch.float32)
    out = torch.empty_like(x) if out is None else out
    cols = x.shape[-1]
    L.check(L.lib().tz_layernorm_last_dim(ctx.handle, _p(x), _p(gamma), _p(beta), _p(out), x.numel() // cols,
                                          cols, eps, _stream()))
    return out


def softmax_last_axis(ctx: Context, x, mask=None, out=None):
    _dev(x, torch.float32)
    out = torch.empty_like(x) if out is None else out
    cols = x.shape[-1]
    L.check(L.lib().tz_softmax_last_axis(ctx.handle, _p(x), _p(mask), _p(out), x.numel() // cols, cols, _stream()))
    return out


def softmax_keylen(ctx: Context, x, key_len, out=None):
    """x [G, R, C]; group g keeps its first key_len[g] columns."""
    _dev(x, torch.float32)
    out = torch.empty_like(x) if out is None else out
    G, R, Cc = x.shape
    L.check(L.lib().tz_softmax_keylen(ctx.handle, _p(x), _p(key_len), _p(out), G, R, Cc, _stream()))
    return out


def attention(ctx: Context, qkv, cu_seqlens, max_len: int, out=None):
    """selfAttention (arctic.zig:639-747) over packed sequences: qkv [T, 1152] float16 or bfloat16
    (Q | K | V, 12 heads of 32), cu_seqlens int32 [B + 1] on the device; returns [T, 384] of qkv's type."""
    if qkv.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("attention: qkv must be float16 or bfloat16")
    _dev(qkv, qkv.dtype)
    _dev(cu_seqlens, torch.int32)
    T = qkv.shape[0]
    if qkv.shape != (T, 1152):
        raise ValueError(f"attention: qkv must be [T, 1152], got {tuple(qkv.shape)}")
    out = torch.empty((T, 384), device=qkv.device, dtype=qkv.dtype) if out is None else out
    L.check(L.lib().tz_attention(ctx.handle, _p(qkv), T, _p(cu_seqlens), cu_seqlens.numel() - 1, int(max_len), _p(out),
                                 int(qkv.dtype == torch.bfloat16), _stream()))
    return out


def linear(ctx: Context, x, w, bias=None, residual=None, out=None):
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty((m, n), device=x.device, dtype=torch.float32) if out is None else out
    L.check(L.lib().tz_linear_f32(ctx.handle, _p(x), _p(w), _p(bias), _p(residual), _p(out), m, k, n, _stream()))
    return out


def linear_w8a32(ctx: Context, x, wq, scale_f16, bias, out=None):
    m, k = x.shape
    n = wq.shape[0]
    out = torch.empty((m, n), device=x.device, dtype=torch.float32) if out is None else out
    L.check(L.lib().tz_linear_w8a32(ctx.handle, _p(x), _p(wq), _p(scale_f16), _p(bias), _p(out), m, k, n, _stream()))
    return out


def linear_w8a8(ctx: Context, x, wq, scale_f16, bias, out=None):
    m, k = x.shape
    n = wq.shape[0]
    out = torch.empty((m, n), device=x.device, dtype=torch.float32) if out is None else out
    L.check(L.lib().tz_linear_w8a8(ctx.handle, _p(x), _p(wq), _p(scale_f16), _p(bias), _p(out), m, k, n, _stream()))
    return out


def gemm_i8_i32(ctx: Context, a, w, out=None):
    m, k = a.shape
    n = w.shape[0]
    out = torch.empty((m, n), device=a.device, dtype=torch.int32) if out is None else out
    L.check(L.lib().tz_gemm_i8_i32(ctx.handle, _p(a), _p(w), _p(out), m, k, n, _stream()))
    return out


def quantize_weight_rows(ctx: Context, w):
    rows, cols = w.shape
    q = torch.empty((rows, cols), device=w.device, dtype=torch.int8)
    s = torch.empty(rows, device=w.device, dtype=torch.int16)  # IEEE half bits
    L.check(L.lib().tz_quantize_weight_rows(ctx.handle, _p(w), _p(q), _p(s), rows, cols, _stream()))
    return q, s


def quantize_act_rows(ctx: Context, x):
    rows, cols = x.shape
    q = torch.empty((rows, cols), device=x.device, dtype=torch.int8)
    s = torch.empty(rows, device=x.device, dtype=torch.float32)
    L.check(L.lib().tz_quantize_act_rows(ctx.handle, _p(x), _p(q), _p(s), rows, cols, _stream()))
    return q, s


def matmul_epilogue(ctx: Context, a, b, bias, ops, trans_b=False, out=None):
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    out = torch.empty((m, n), device=a.device, dtype=torch.float32) if out is None else out
    codes = (C.c_int * max(1, len(ops)))(*[L.OP[o] if isinstance(o, str) else int(o) for o in ops])
    L.check(L.lib().tz_matmul_epilogue(ctx.handle, _p(a), _p(b), int(trans_b), _p(bias), C.addressof(codes),
                                       len(ops), _p(out), m, k, n, _stream()))
    return out


def ew_add_mul_exp(ctx: Context, a, b_row, c, out=None):
    out = torch.empty_like(a) if out is None else out
    cols = b_row.numel()
    L.check(L.lib().tz_ew_add_mul_exp(ctx.handle, _p(a), _p(b_row), _p(c), _p(out), a.numel() // cols, cols,
                                      _stream()))
    return out


def ew_unary_chain(ctx: Context, x, ops, out=None):
    out = torch.empty_like(x) if out is None else out
    codes = (C.c_int * max(1, len(ops)))(*[L.OP[o] for o in ops])
    L.check(L.lib().tz_ew_unary_chain(ctx.handle, _p(x), _p(out), x.numel(), C.addressof(codes), len(ops),
                                      _stream()))
    return out


def reduce(ctx: Context, op: str, pre_ops, x):
    out = torch.empty(1, device=x.device, dtype=torch.float32)
    codes = (C.c_int * max(1, len(pre_ops)))(*[L.OP[o] for o in pre_ops])
    L.check(L.lib().tz_reduce(ctx.handle, L.RED[op], C.addressof(codes), len(pre_ops), _p(x), x.numel(), _p(out),
                              _stream()))
    return out


def gather_rows(ctx: Context, table, ids, out=None):
    rows, cols = table.shape
    out = torch.empty((ids.numel(), cols), device=table.device, dtype=torch.float32) if out is None else out
    L.check(L.lib().tz_gather_rows(ctx.handle, _p(table), rows, _p(ids), ids.numel(), cols, _p(out), _stream()))
    return out


# ---- N-D ops -------------------------------------------------------------------------------------
_TORCH_DT = {torch.float32: "f32", torch.float16: "f16", torch.int8: "i8", torch.int32: "i32",
             torch.int64: "i64", torch.uint8: "u8", torch.bool: "u8"}


def matmul_f32x3(ctx: Context, a, b, bias, ops, trans_b=False, out=None):
    """matmul_epilogue with f32-accurate products (split tf32 on the tensor cores)."""
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    out = torch.empty((m, n), device=a.device, dtype=torch.float32) if out is None else out
    codes = (C.c_int * max(1, len(ops)))(*[L.OP[o] if isinstance(o, str) else int(o) for o in ops])
    L.check(L.lib().tz_matmul_f32x3(ctx.handle, _p(a), _p(b), int(trans_b), _p(bias), C.addressof(codes),
                                    len(ops), _p(out), m, k, n, _stream()))
    return out


def batched_matmul(ctx: Context, a, b, out_shape, batch_shape, a_bstride, b_bstride, m, k, n,
                   a_rs, a_cs, b_rs, b_cs, out=None, c_view=None):
    """Batched matmul on element strides (tz_batched_matmul).  The output is a new contiguous
    tensor of out_shape unless `out` is given with `c_view` = (c_bstride, c_rs, c_cs)."""
    if out is None:
        out = torch.empty(out_shape, device=a.device, dtype=torch.float32)
    lay = L.BmmLayout()
    lay.batch_ndim = len(batch_shape)
    if c_view is None:
        cb, acc = [], m * n
        for d in reversed(batch_shape):
            cb.append(acc)
            acc *= d
        c_view = (list(reversed(cb)), n, 1)
    for d, e in enumerate(batch_shape):
        lay.batch_shape[d] = e
        lay.a_bstride[d] = a_bstride[d]
        lay.b_bstride[d] = b_bstride[d]
        lay.c_bstride[d] = c_view[0][d]
    lay.a_rs, lay.a_cs, lay.b_rs, lay.b_cs = a_rs, a_cs, b_rs, b_cs
    lay.c_rs, lay.c_cs = c_view[1], c_view[2]
    lay.m, lay.k, lay.n = m, k, n
    L.check(L.lib().tz_batched_matmul(ctx.handle, _p(a), _p(b), _p(out), C.byref(lay), _stream()))
    return out


def _split_axis(shape, axis):
    axis = axis % len(shape) if shape else 0
    outer = 1
    for d in shape[:axis]:
        outer *= d
    inner = 1
    for d in shape[axis + 1:]:
        inner *= d
    return axis, outer, shape[axis], inner


def reduce_axis(ctx: Context, op: str, x, axis: int, keepdims=False):
    """reduceAxis (reduce.zig:52-95): one axis of a contiguous f32 tensor."""
    shape = list(x.shape)
    axis, outer, ln, inner = _split_axis(shape, axis)
    oshape = shape[:axis] + ([1] if keepdims else []) + shape[axis + 1:]
    out = torch.empty(oshape, device=x.device, dtype=torch.float32)
    L.check(L.lib().tz_reduce_axis(ctx.handle, L.RED[op], _p(x), outer, ln, inner, _p(out), _stream()))
    return out


def softmax_axis(ctx: Context, x, axis: int = -1, out=None):
    """softmaxAxis (softmax.zig:157-220)."""
    shape = list(x.shape)
    axis, outer, ln, inner = _split_axis(shape, axis)
    out = torch.empty_like(x) if out is None else out
    L.check(L.lib().tz_softmax_axis(ctx.handle, _p(x), _p(out), outer, ln, inner, _stream()))
    return out


def permute(ctx: Context, x, perm):
    """Transpose (onnx/executor.zig:2296): a contiguous copy of x.permute(perm)."""
    shape = list(x.shape)
    out = torch.empty([shape[p] for p in perm], device=x.device, dtype=x.dtype)
    sh = (C.c_int64 * max(1, len(shape)))(*shape)
    pm = (C.c_int * max(1, len(perm)))(*perm)
    L.check(L.lib().tz_permute(ctx.handle, _p(x), _p(out), x.element_size(), len(shape), C.addressof(sh),
                               C.addressof(pm), _stream()))
    return out


def cast(ctx: Context, x, dtype):
    """Cast (onnx/executor.zig:2852) on the device."""
    out = torch.empty(x.shape, device=x.device, dtype=dtype)
    L.check(L.lib().tz_cast(ctx.handle, _p(x), L.DT[_TORCH_DT[x.dtype]], _p(out), L.DT[_TORCH_DT[dtype]], x.numel(),
                            _stream()))
    return out


def concat(ctx: Context, xs, axis: int):
    """Concat (onnx/executor.zig:2112) of contiguous tensors of one dtype along `axis`."""
    shape = list(xs[0].shape)
    axis = axis % len(shape)
    outer = 1
    for d in shape[:axis]:
        outer *= d
    inner = 1
    for d in shape[axis + 1:]:
        inner *= d
    lens = [int(t.shape[axis]) for t in xs]
    oshape = shape[:axis] + [sum(lens)] + shape[axis + 1:]
    out = torch.empty(oshape, device=xs[0].device, dtype=xs[0].dtype)
    ptrs = (C.c_void_p * len(xs))(*[t.data_ptr() for t in xs])
    ln = (C.c_int64 * len(xs))(*lens)
    L.check(L.lib().tz_concat(ctx.handle, C.addressof(ptrs), C.addressof(ln), len(xs), outer, inner,
                              xs[0].element_size(), _p(out), _stream()))
    return out
