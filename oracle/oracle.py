"""ctypes front end of the CPU oracle (libtz_oracle.so, built from tz_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg as the checker.  The product (tenzor_b200/) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtz_oracle.so")

MODE_F32, MODE_W8A32, MODE_W8A8 = 0, 1, 2
H, LAYERS, FFN = 384, 6, 1536

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p


def _declare(L):
    L.tzo_f32_to_f16.restype = C.c_uint16
    L.tzo_f32_to_f16.argtypes = [C.c_float]
    L.tzo_f16_to_f32.restype = C.c_float
    L.tzo_f16_to_f32.argtypes = [C.c_uint16]
    for name in ("tzo_gelu_model", "tzo_gelu_simd"):
        getattr(L, name).restype = C.c_float
        getattr(L, name).argtypes = [C.c_float]
    L.tzo_unary.restype = C.c_float
    L.tzo_unary.argtypes = [C.c_int, C.c_float]
    L.tzo_layernorm_rows.argtypes = [P, P, P, P, C.c_int64, C.c_int, C.c_float]
    L.tzo_softmax_rows.argtypes = [P, P, P, C.c_int64, C.c_int]
    L.tzo_l2_normalize.argtypes = [P, C.c_int]
    L.tzo_sgemm_nt.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_sgemm_nn.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_attention_packed.argtypes = [P, P, C.c_int, P]
    L.tzo_linear_f32.argtypes = [P, P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_linear_w8a32.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_linear_w8a8.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_gemm_i8_i32.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int]
    L.tzo_quantize_act_rows.argtypes = [P, P, P, C.c_int64, C.c_int]
    L.tzo_dequant_epilogue.argtypes = [P, P, P, P, P, C.c_int, C.c_int]
    L.tzo_quantize_weight_rows.argtypes = [P, P, P, C.c_int64, C.c_int]
    L.tzo_matmul_epilogue.argtypes = [P, P, C.c_int, P, P, C.c_int, P, C.c_int, C.c_int, C.c_int]
    L.tzo_ew_add_mul_exp.argtypes = [P, P, P, P, C.c_int64, C.c_int]
    L.tzo_reduce.restype = C.c_float
    L.tzo_reduce.argtypes = [C.c_int, P, C.c_int, P, C.c_int64]
    L.tzo_arctic_forward.restype = C.c_int
    L.tzo_arctic_forward.argtypes = [P, C.c_int, P, P, C.c_int, P, C.c_int]
    L.tzo_arctic_forward_dump.restype = C.c_int
    L.tzo_arctic_forward_dump.argtypes = [P, C.c_int, P, P, C.c_int, P, C.c_int, P]
    L.tzo_blas_status.restype = C.c_char_p
    L.tzo_lenet_forward.argtypes = [P, C.c_int, P, C.c_int64, P, C.c_int]


def ptr(a):
    return None if a is None else a.ctypes.data


def c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- element / row helpers -------------------------------------------------------------------
def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    L = lib()
    return np.array([L.tzo_f32_to_f16(float(v)) for v in np.ravel(x)], np.uint16).reshape(
        np.shape(x))


def gelu_model(x: float) -> float:
    return lib().tzo_gelu_model(float(x))


def gelu_simd(x: float) -> float:
    return lib().tzo_gelu_simd(float(x))


def unary(op: int, x: float) -> float:
    return lib().tzo_unary(op, float(x))


def layernorm(x, g, b, eps):
    x = c32(x)
    y = np.empty_like(x)
    cols = x.shape[-1]
    lib().tzo_layernorm_rows(ptr(x), ptr(c32(g)), ptr(c32(b)), ptr(y), x.size // cols, cols, eps)
    return y


def softmax(x, mask=None):
    x = c32(x)
    y = np.empty_like(x)
    cols = x.shape[-1]
    m = None if mask is None else c32(np.broadcast_to(mask, x.shape))
    lib().tzo_softmax_rows(ptr(x), ptr(m), ptr(y), x.size // cols, cols)
    return y


def l2_normalize(v):
    v = c32(v).copy()
    lib().tzo_l2_normalize(ptr(v), v.size)
    return v


def sgemm_nt(a, b):
    a, b = c32(a), c32(b)
    m, k = a.shape
    n = b.shape[0]
    c = np.empty((m, n), np.float32)
    lib().tzo_sgemm_nt(ptr(a), ptr(b), ptr(c), m, k, n)
    return c


def sgemm_nn(a, b):
    a, b = c32(a), c32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().tzo_sgemm_nn(ptr(a), ptr(b), ptr(c), m, k, n)
    return c


def attention_packed(qkv, cu_seqlens):
    """tzo_attention_packed: qkv [T, 1152] f32, cu_seqlens [B + 1] -> [T, 384] f32."""
    qkv = c32(qkv)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    out = np.zeros((qkv.shape[0], 384), np.float32)
    lib().tzo_attention_packed(ptr(qkv), ptr(cu), len(cu) - 1, ptr(out))
    return out


def linear_w8a32(x, wq, s16, bias):
    x = c32(x)
    wq = np.ascontiguousarray(wq, np.int8)
    m, k = x.shape
    n = wq.shape[0]
    y = np.empty((m, n), np.float32)
    lib().tzo_linear_w8a32(ptr(x), ptr(wq), ptr(np.ascontiguousarray(s16, np.uint16)),
                           ptr(c32(bias)), ptr(y), m, k, n)
    return y


def linear_w8a8(x, wq, s16, bias):
    x = c32(x)
    wq = np.ascontiguousarray(wq, np.int8)
    m, k = x.shape
    n = wq.shape[0]
    y = np.empty((m, n), np.float32)
    lib().tzo_linear_w8a8(ptr(x), ptr(wq), ptr(np.ascontiguousarray(s16, np.uint16)),
                          ptr(c32(bias)), ptr(y), m, k, n)
    return y


def gemm_i8_i32(a, w):
    a = np.ascontiguousarray(a, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), np.int32)
    lib().tzo_gemm_i8_i32(ptr(a), ptr(w), ptr(c), m, k, n)
    return c


def quantize_act_rows(x):
    x = c32(x)
    rows, cols = x.size // x.shape[-1], x.shape[-1]
    q = np.empty(x.shape, np.int8)
    s = np.empty(rows, np.float32)
    lib().tzo_quantize_act_rows(ptr(x), ptr(q), ptr(s), rows, cols)
    return q, s


def dequant_epilogue(acc, a_s, w_s16, bias):
    acc = np.ascontiguousarray(acc, np.int32)
    m, n = acc.shape
    y = np.empty((m, n), np.float32)
    lib().tzo_dequant_epilogue(ptr(acc), ptr(c32(a_s)), ptr(np.ascontiguousarray(w_s16, np.uint16)),
                               ptr(c32(bias)), ptr(y), m, n)
    return y


def quantize_weight_rows(w):
    w = c32(w)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.uint16)
    lib().tzo_quantize_weight_rows(ptr(w), ptr(q), ptr(s), rows, cols)
    return q, s


def matmul_epilogue(a, b, bias, ops, trans_b=False):
    a, b = c32(a), c32(b)
    m, k = a.shape
    n = b.shape[0] if trans_b else b.shape[1]
    c = np.empty((m, n), np.float32)
    o = np.ascontiguousarray(ops, np.int32)
    lib().tzo_matmul_epilogue(ptr(a), ptr(b), int(trans_b), ptr(None if bias is None else c32(bias)),
                              ptr(o), len(ops), ptr(c), m, k, n)
    return c


def ew_add_mul_exp(a, b_row, c):
    a, b_row, c = c32(a), c32(b_row), c32(c)
    out = np.empty_like(a)
    cols = b_row.size
    lib().tzo_ew_add_mul_exp(ptr(a), ptr(b_row), ptr(c), ptr(out), a.size // cols, cols)
    return out


def reduce(op, pre_ops, x):
    x = c32(x).ravel()
    o = np.ascontiguousarray(pre_ops, np.int32)
    return lib().tzo_reduce(op, ptr(o), len(pre_ops), ptr(x), x.size)


# ---- the model -------------------------------------------------------------------------------
class _Layer(C.Structure):
    _fields_ = [(n, P) for n in (
        "q_w k_w v_w o_w ffn1_w ffn2_w q_q k_q v_q o_q ffn1_q ffn2_q "
        "q_s k_s v_s o_s ffn1_s ffn2_s q_b k_b v_b o_b ffn1_b ffn2_b "
        "ln1_g ln1_b ln2_g ln2_b").split()]


class _Weights(C.Structure):
    _fields_ = [(n, P) for n in "word_w pos_w type_w word_q pos_q word_s pos_s emb_ln_g emb_ln_b".split()]
    _fields_ += [("layers", _Layer * LAYERS)]


def quantize_checkpoint(w: dict) -> dict:
    """quantize_arctic_xs.zig:22-34 + 94-115 over a name->array checkpoint: every 2-D f32
    '.weight' (not LayerNorm) with >= 4096 elements becomes I8 + '<name>.scale' F16 bits."""
    out = {}
    for name, t in w.items():
        if (t.dtype == np.float32 and t.ndim == 2 and name.endswith(".weight")
                and "LayerNorm" not in name and t.size >= 4096):
            q, s = quantize_weight_rows(t)
            out[name] = q
            out[name + ".scale"] = s
        else:
            out[name] = t
    return out


class OracleModel:
    """Holds the arrays alive and the ctypes struct that points at them."""

    def __init__(self, ckpt: dict):
        self.keep = {k: np.ascontiguousarray(v) for k, v in ckpt.items()}
        k = self.keep
        s = _Weights()
        e = "embeddings."

        def f(name):
            a = k.get(name)
            return ptr(a) if a is not None and a.dtype == np.float32 else None

        def q(name):
            a = k.get(name)
            return ptr(a) if a is not None and a.dtype == np.int8 else None

        def sc(name):
            a = k.get(name + ".scale")
            return ptr(a) if a is not None else None

        s.word_w, s.pos_w = f(e + "word_embeddings.weight"), f(e + "position_embeddings.weight")
        s.type_w = f(e + "token_type_embeddings.weight")
        s.word_q, s.pos_q = q(e + "word_embeddings.weight"), q(e + "position_embeddings.weight")
        s.word_s, s.pos_s = sc(e + "word_embeddings.weight"), sc(e + "position_embeddings.weight")
        s.emb_ln_g, s.emb_ln_b = f(e + "LayerNorm.weight"), f(e + "LayerNorm.bias")
        for i in range(LAYERS):
            p = f"encoder.layer.{i}."
            names = {"q": "attention.self.query", "k": "attention.self.key",
                     "v": "attention.self.value", "o": "attention.output.dense",
                     "ffn1": "intermediate.dense", "ffn2": "output.dense"}
            lw = s.layers[i]
            for key, nm in names.items():
                setattr(lw, key + "_w", f(p + nm + ".weight"))
                setattr(lw, key + "_q", q(p + nm + ".weight"))
                setattr(lw, key + "_s", sc(p + nm + ".weight"))
                setattr(lw, key + "_b", f(p + nm + ".bias"))
            lw.ln1_g, lw.ln1_b = f(p + "attention.output.LayerNorm.weight"), f(p + "attention.output.LayerNorm.bias")
            lw.ln2_g, lw.ln2_b = f(p + "output.LayerNorm.weight"), f(p + "output.LayerNorm.bias")
        self.struct = s

    def forward(self, packed_ids, cu_seqlens, mode, nthreads=0, dump=False):
        ids = np.ascontiguousarray(packed_ids, np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        B = len(cu) - 1
        out = np.zeros((B, H), np.float32)
        T = int(cu[-1])
        d = np.zeros((LAYERS + 1, T, H), np.float32) if dump else None
        rc = lib().tzo_arctic_forward_dump(C.addressof(self.struct), mode, ptr(ids), ptr(cu), B,
                                           ptr(out), nthreads, ptr(d))
        if rc != 0:
            raise ValueError(f"oracle forward rejected the input (rc={rc})")
        return (out, d) if dump else out


def blas_status() -> str:
    return lib().tzo_blas_status().decode()


# ---- LeNet-5 (tz_oracle_lenet.c) ----
LENET_REF, LENET_PAD2 = 0, 1
LENET_KEYS = ("conv1_w", "conv1_b", "conv2_w", "conv2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "fc3_w", "fc3_b")


class _LenetWeights(C.Structure):
    _fields_ = [(k, P) for k in LENET_KEYS]


def lenet_forward(w: dict, variant: int, images: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """images [n, 28, 28, 1] (or [n, 784]) f32 -> [n, 10] (logits for LENET_REF, softmax for
    LENET_PAD2); weights as in tz_oracle.h (NHWC conv weights [out, kh, kw, in])."""
    keep = {k: c32(w[k]) for k in LENET_KEYS}
    ws = _LenetWeights(*[ptr(keep[k]) for k in LENET_KEYS])
    x = c32(images).reshape(-1, 784)
    out = np.empty((x.shape[0], 10), np.float32)
    lib().tzo_lenet_forward(C.byref(ws), variant, ptr(x), x.shape[0], ptr(out), nthreads)
    return out
