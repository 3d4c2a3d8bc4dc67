"""ctypes bindings of include/tenzor_cuda.h (libtenzor_cuda.so, built in-tree).

There is no fallback: if the library is missing or cannot load, importing a compute entry point
raises.  Build it with ``python -m tenzor_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libtenzor_cuda.so")

TZ_OK, TZ_EINVAL, TZ_ENOMEM, TZ_ECUDA, TZ_ETIMEOUT, TZ_EUNSUPPORTED, TZ_EMISSING = range(7)
QUANT_F32, QUANT_W8A32, QUANT_W8A8 = 0, 1, 2
OP = {"add": 1, "relu": 2, "gelu": 3, "sigmoid": 4, "tanh": 5, "exp": 6, "neg": 7, "abs": 8,
      "silu": 9, "log": 10, "sqrt": 11, "rsqrt": 12, "sin": 13, "cos": 14, "erf": 15, "gelu_erf": 16,
      "erf_as": 17, "gelu_tanh": 18}
EW_BINARY = {"add": 20, "sub": 21, "mul": 22, "div": 23, "max": 24, "min": 25, "pow": 26, "eq": 27, "lt": 28, "gt": 29}
EW_WHERE = 30
RED = {"sum": 0, "mean": 1, "prod": 2, "max": 3, "min": 4}

# Every symbol include/tenzor_cuda.h declares (checked by tests/test_abi.py).
EXPORTS = [
    "tz_get_last_error", "tz_version", "tz_cuda_create", "tz_cuda_destroy", "tz_cuda_synchronize",
    "tz_cuda_check_status", "tz_cuda_sm_count", "tz_cuda_set_sm_reserve", "tz_cuda_selftest_wait", "tz_alloc", "tz_free", "tz_upload", "tz_download",
    "tz_arctic_load", "tz_arctic_load_ex", "tz_arctic_load_safetensors", "tz_arctic_free", "tz_arctic_reserve",
    "tz_arctic_forward", "tz_arctic_forward_padded", "tz_arctic_forward_device",
    "tz_arctic_debug_hidden", "tz_arctic_debug_operand", "tz_arctic_debug_accum", "tz_arctic_debug_gemm_input",
    "tz_arctic_debug_capture", "tz_arctic_set_ffn_fusion",
    "tz_arctic_profile", "tz_arctic_profile_read", "tz_layernorm_last_dim",
    "tz_softmax_last_axis", "tz_softmax_keylen", "tz_attention", "tz_linear_f32", "tz_linear_w8a32",
    "tz_linear_w8a8", "tz_linear_w8a8_noalloc", "tz_gemm_i8_i32", "tz_quantize_weight_rows", "tz_quantize_act_rows",
    "tz_matmul_epilogue", "tz_ew_add_mul_exp", "tz_ew_program_run", "tz_ew_unary_chain", "tz_reduce",
    "tz_gather_rows", "tz_lenet_load", "tz_lenet_free", "tz_lenet_reserve", "tz_lenet_forward",
    "tz_lenet_forward_device", "tz_tokenizer_create", "tz_tokenizer_free", "tz_tokenizer_set_special",
    "tz_tokenizer_load_vocab", "tz_tokenizer_load_vocab_bytes", "tz_tokenizer_put", "tz_tokenizer_vocab_size",
    "tz_tokenizer_encode", "tz_tokenizer_encode_raw", "tz_tokenizer_encode_batch", "tz_arctic_embed_texts",
    "tz_doc_chunk_count", "tz_arctic_embed_documents", "tz_tenzor_hash_name", "tz_tenzor_open",
    "tz_tenzor_close", "tz_tenzor_count", "tz_tenzor_entry_at", "tz_tenzor_find", "tz_tenzor_metadata",
    "tz_lenet_load_tenzor", "tz_arctic_load_tenzor", "tz_ew_program_run_nd", "tz_batched_matmul",
    "tz_matmul_f32x3", "tz_reduce_axis", "tz_softmax_axis", "tz_permute", "tz_cast", "tz_concat",
]


class TenzorError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[tz status {code}] {msg}")
        self.code = code


P = C.c_void_p


class MatWeight(C.Structure):
    _fields_ = [("f32", P), ("q8", P), ("scale_f16", P)]


class ArcticLayer(C.Structure):
    _fields_ = [(n, MatWeight) for n in ("query", "key", "value", "attn_output", "intermediate", "output")]
    _fields_ += [(n, P) for n in ("query_bias", "key_bias", "value_bias", "attn_output_bias",
                                  "intermediate_bias", "output_bias", "attn_ln_gamma", "attn_ln_beta",
                                  "output_ln_gamma", "output_ln_beta")]


class TenzorEntry(C.Structure):
    _fields_ = [("name_hash", C.c_uint64), ("dtype", C.c_int), ("ndim", C.c_int), ("shape", C.c_uint32 * 5),
                ("data", P), ("bytes", C.c_uint64)]


class EwInstr(C.Structure):
    _fields_ = [("op", C.c_int), ("dst", C.c_int), ("a", C.c_int), ("b", C.c_int), ("c", C.c_int)]


class EwProgram(C.Structure):
    _fields_ = [("n_inputs", C.c_int), ("in_", P * 4), ("row_stride", C.c_int64 * 4), ("col_stride", C.c_int64 * 4),
                ("n_instr", C.c_int), ("instr", EwInstr * 16), ("result", C.c_int), ("consts", C.c_float * 4)]


MAX_DIMS = 6
DT = {"f32": 0, "f16": 1, "bf16": 2, "f64": 3, "i8": 4, "i16": 5, "i32": 6, "i64": 7, "u8": 8}


class NdLayout(C.Structure):
    _fields_ = [("ndim", C.c_int), ("shape", C.c_int64 * MAX_DIMS), ("stride", (C.c_int64 * MAX_DIMS) * 4)]


class BmmLayout(C.Structure):
    _fields_ = [("batch_ndim", C.c_int), ("batch_shape", C.c_int64 * 4), ("a_bstride", C.c_int64 * 4),
                ("b_bstride", C.c_int64 * 4), ("c_bstride", C.c_int64 * 4)]
    _fields_ += [(n, C.c_int64) for n in ("a_rs", "a_cs", "b_rs", "b_cs", "c_rs", "c_cs")]
    _fields_ += [("m", C.c_int), ("k", C.c_int), ("n", C.c_int)]


class ArcticWeights(C.Structure):
    _fields_ = [("word_embeddings", MatWeight), ("position_embeddings", MatWeight),
                ("token_type_embeddings", MatWeight), ("ln_gamma", P), ("ln_beta", P),
                ("layers", ArcticLayer * 6)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m tenzor_b200.build` "
                              "(there is no CPU fallback)")
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L):
    i, i64, u = C.c_int, C.c_int64, C.c_size_t
    L.tz_get_last_error.restype = C.c_char_p
    L.tz_version.restype = C.c_char_p
    sig = {
        "tz_cuda_create": [i, C.POINTER(P)],
        "tz_cuda_destroy": [P], "tz_cuda_synchronize": [P], "tz_cuda_check_status": [P],
        "tz_cuda_sm_count": [P], "tz_cuda_set_sm_reserve": [P, i], "tz_cuda_selftest_wait": [P],
        "tz_alloc": [P, u, C.POINTER(P)], "tz_free": [P, P],
        "tz_upload": [P, P, P, u], "tz_download": [P, P, P, u],
        "tz_arctic_load": [P, C.POINTER(ArcticWeights), i, C.POINTER(P)],
        "tz_arctic_load_ex": [P, C.POINTER(ArcticWeights), i, i, C.POINTER(P)],
        "tz_arctic_load_safetensors": [P, C.c_char_p, i, C.POINTER(P)],
        "tz_arctic_free": [P], "tz_arctic_reserve": [P, i, i64],
        "tz_arctic_forward": [P, P, P, i, P],
        "tz_arctic_forward_padded": [P, P, P, i, i, P],
        "tz_arctic_forward_device": [P, P, P, i, i64, i, P, P],
        "tz_arctic_debug_hidden": [P, i, P, i64],
        "tz_arctic_debug_operand": [P, i, P, P, i64],
        "tz_arctic_debug_accum": [P, i, P, i64], "tz_arctic_debug_capture": [P, i], "tz_arctic_debug_gemm_input": [P, i, P, i64],
        "tz_arctic_set_ffn_fusion": [P, i],
        "tz_arctic_profile": [P, i], "tz_arctic_profile_read": [P, P, P],
        "tz_layernorm_last_dim": [P, P, P, P, P, i64, i, C.c_float, P],
        "tz_softmax_last_axis": [P, P, P, P, i64, i, P],
        "tz_softmax_keylen": [P, P, P, P, i64, i, i, P],
        "tz_attention": [P, P, i64, P, i, i, P, i, P],
        "tz_linear_f32": [P, P, P, P, P, P, i, i, i, P],
        "tz_linear_w8a32": [P, P, P, P, P, P, i, i, i, P],
        "tz_linear_w8a8": [P, P, P, P, P, P, i, i, i, P],
        "tz_linear_w8a8_noalloc": [P, P, P, P, P, P, i, i, i, P],
        "tz_gemm_i8_i32": [P, P, P, P, i, i, i, P],
        "tz_quantize_weight_rows": [P, P, P, P, i64, i, P],
        "tz_quantize_act_rows": [P, P, P, P, i64, i, P],
        "tz_matmul_epilogue": [P, P, P, i, P, P, i, P, i, i, i, P],
        "tz_ew_add_mul_exp": [P, P, P, P, P, i64, i, P],
        "tz_ew_unary_chain": [P, P, P, i64, P, i, P],
        "tz_ew_program_run": [P, C.POINTER(EwProgram), P, i64, i, P],
        "tz_reduce": [P, i, P, i, P, i64, P, P],
        "tz_gather_rows": [P, P, i64, P, i64, i, P, P],
        "tz_lenet_load": [P, P, i, C.POINTER(P)], "tz_lenet_free": [P], "tz_lenet_reserve": [P, i64],
        "tz_lenet_forward": [P, P, i64, P], "tz_lenet_forward_device": [P, P, i64, P, P],
        "tz_tokenizer_create": [C.POINTER(P)], "tz_tokenizer_free": [P],
        "tz_tokenizer_set_special": [P, C.c_uint32, C.c_uint32, C.c_uint32],
        "tz_tokenizer_load_vocab": [P, C.c_char_p], "tz_tokenizer_load_vocab_bytes": [P, C.c_char_p, i64],
        "tz_tokenizer_put": [P, C.c_char_p, i64, C.c_uint32], "tz_tokenizer_vocab_size": [P, C.POINTER(i64)],
        "tz_tokenizer_encode": [P, C.c_char_p, i64, P, i64, C.POINTER(i64)],
        "tz_tokenizer_encode_raw": [P, C.c_char_p, i64, P, i64, C.POINTER(i64)],
        "tz_tokenizer_encode_batch": [P, P, P, i, i, P, P, i64],
        "tz_arctic_embed_texts": [P, P, P, P, i, P],
        "tz_arctic_embed_documents": [P, P, P, P, i, P],
        "tz_tenzor_open": [C.c_char_p, C.POINTER(P)], "tz_tenzor_close": [P],
        "tz_tenzor_entry_at": [P, i64, C.POINTER(TenzorEntry)],
        "tz_tenzor_find": [P, C.c_char_p, C.POINTER(TenzorEntry)],
        "tz_tenzor_metadata": [P, C.POINTER(C.c_char_p), C.POINTER(C.c_uint64)],
        "tz_lenet_load_tenzor": [P, C.c_char_p, i, C.POINTER(P)],
        "tz_arctic_load_tenzor": [P, C.c_char_p, i, C.POINTER(P)],
        "tz_ew_program_run_nd": [P, C.POINTER(EwProgram), C.POINTER(NdLayout), P, P],
        "tz_batched_matmul": [P, P, P, P, C.POINTER(BmmLayout), P],
        "tz_matmul_f32x3": [P, P, P, i, P, P, i, P, i, i, i, P],
        "tz_reduce_axis": [P, i, P, i64, i64, i64, P, P],
        "tz_softmax_axis": [P, P, P, i64, i64, i64, P],
        "tz_permute": [P, P, P, i, i, P, P, P],
        "tz_cast": [P, P, i, P, i, i64, P],
        "tz_concat": [P, P, P, i, i64, i64, i, P, P],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = C.c_int
    L.tz_doc_chunk_count.argtypes = [i64]
    L.tz_doc_chunk_count.restype = i64
    L.tz_tenzor_hash_name.argtypes = [C.c_char_p, u]
    L.tz_tenzor_hash_name.restype = C.c_uint64
    L.tz_tenzor_count.argtypes = [P]
    L.tz_tenzor_count.restype = i64


def check(rc: int):
    if rc != TZ_OK:
        raise TenzorError(rc, lib().tz_get_last_error().decode(errors="replace"))
