"""Protobuf wire-format writer for ONNX test fixtures (no `onnx` package in this environment): the
fields of onnx.proto3 that the reader of tenzor_b200/onnx_model.py and the reference's parser.zig
consume.  Test infrastructure only."""
from __future__ import annotations

import struct

import numpy as np


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _ld(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field: int, s: str) -> bytes:
    return _ld(field, s.encode())


def _int(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def tensor(name: str, a: np.ndarray, raw: bool = True) -> bytes:
    a = np.asarray(a)
    dt = {np.dtype(np.float32): 1, np.dtype(np.int64): 7, np.dtype(np.int32): 6}[a.dtype]
    out = b"".join(_int(1, d) for d in a.shape) + _int(2, dt) + _str(8, name)
    if raw:
        out += _ld(9, a.astype(a.dtype.newbyteorder("<")).tobytes())
    elif dt == 1:
        out += _ld(4, b"".join(struct.pack("<f", float(x)) for x in a.ravel()))  # packed float_data
    else:
        out += _ld(7, b"".join(_varint(int(x)) for x in a.ravel()))  # packed int64_data
    return out


def attribute(name: str, v) -> bytes:
    out = _str(1, name)
    if isinstance(v, float):
        return out + _key(2, 5) + struct.pack("<f", v) + _int(20, 1)
    if isinstance(v, int):
        return out + _int(3, v) + _int(20, 2)
    if isinstance(v, str):
        return out + _ld(4, v.encode()) + _int(20, 3)
    if isinstance(v, (list, tuple)):
        return out + _ld(8, b"".join(_varint(int(x)) for x in v)) + _int(20, 7)
    raise TypeError(type(v))


def node(op: str, ins, outs, **attrs) -> bytes:
    out = b"".join(_str(1, i) for i in ins) + b"".join(_str(2, o) for o in outs) + _str(4, op)
    return out + b"".join(_ld(5, attribute(k, v)) for k, v in attrs.items())


def value_info(name: str) -> bytes:
    return _str(1, name)


def model(nodes, initializers: dict, inputs, outputs, opset: int = 20, raw: bool = True) -> bytes:
    g = b"".join(_ld(1, n) for n in nodes) + _str(2, "g")
    g += b"".join(_ld(5, tensor(k, v, raw)) for k, v in initializers.items())
    g += b"".join(_ld(11, value_info(i)) for i in inputs) + b"".join(_ld(12, value_info(o)) for o in outputs)
    return _int(1, 9) + _str(2, "tenzor-b200-tests") + _ld(7, g) + _ld(8, _str(1, "") + _int(2, opset))


def bert_layer(seed: int = 0, vocab: int = 97, seq: int = 24, hidden: int = 64, ffn: int = 128,
               gelu: str = "Gelu", raw: bool = True):
    """A one-sequence, one-head BERT encoder layer as an exporter would write it from the ops of the
    reference's op map: embeddings Gather + Add + LayerNormalization, Q/K/V MatMul + Add, scores by
    Gemm(transB), Softmax, P V MatMul, output projection + residual + LayerNormalization, FFN with
    Gemm bias, GELU (the Gelu op, or the Erf decomposition), residual + LayerNormalization.
    Returns (model bytes, feeds)."""
    rng = np.random.default_rng(seed)
    w = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)
    ones = lambda n: (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    inits = {
        "word": w(vocab, hidden), "pos": w(seq, hidden), "ln0_g": ones(hidden), "ln0_b": w(hidden),
        "wq": w(hidden, hidden) * np.float32(1.0 / np.sqrt(hidden)), "bq": w(hidden),
        "wk": w(hidden, hidden), "bk": w(hidden), "wv": w(hidden, hidden), "bv": w(hidden),
        "wo": w(hidden, hidden), "bo": w(hidden), "ln1_g": ones(hidden), "ln1_b": w(hidden),
        "w1": w(hidden, ffn), "b1": w(ffn), "w2": w(ffn, hidden), "b2": w(hidden),
        "ln2_g": ones(hidden), "ln2_b": w(hidden),
    }
    n = [
        node("Gather", ["word", "ids"], ["e0"], axis=0),
        node("Add", ["e0", "pos"], ["e1"]),
        node("LayerNormalization", ["e1", "ln0_g", "ln0_b"], ["x0"], axis=-1, epsilon=1e-12),
        node("MatMul", ["x0", "wq"], ["q0"]), node("Add", ["q0", "bq"], ["q"]),
        node("MatMul", ["x0", "wk"], ["k0"]), node("Add", ["k0", "bk"], ["k"]),
        node("MatMul", ["x0", "wv"], ["v0"]), node("Add", ["v0", "bv"], ["v"]),
        node("Gemm", ["q", "k"], ["s"], transB=1),
        node("Softmax", ["s"], ["p"], axis=-1),
        node("MatMul", ["p", "v"], ["c"]),
        node("MatMul", ["c", "wo"], ["o0"]), node("Add", ["o0", "bo"], ["o"]),
        node("Add", ["o", "x0"], ["r1"]),
        node("LayerNormalization", ["r1", "ln1_g", "ln1_b"], ["x1"], axis=-1, epsilon=1e-12),
        node("Gemm", ["x1", "w1", "b1"], ["h"]),
    ]
    if gelu == "Gelu":
        n.append(node("Gelu", ["h"], ["g"]))
    else:  # 0.5 * h * (1 + erf(h / sqrt(2))), constants as broadcast rows
        inits.update({"inv_sqrt2": np.full(ffn, 1.0 / np.sqrt(2.0), np.float32), "one": np.ones(ffn, np.float32),
                      "half": np.full(ffn, 0.5, np.float32)})
        n += [node("Mul", ["h", "inv_sqrt2"], ["h1"]), node("Erf", ["h1"], ["h2"]), node("Add", ["h2", "one"], ["h3"]),
              node("Mul", ["h", "h3"], ["h4"]), node("Mul", ["h4", "half"], ["g"])]
    n += [
        node("MatMul", ["g", "w2"], ["f0"]), node("Add", ["f0", "b2"], ["f"]),
        node("Add", ["f", "x1"], ["r2"]),
        node("LayerNormalization", ["r2", "ln2_g", "ln2_b"], ["y"], axis=-1, epsilon=1e-12),
    ]
    feeds = {"ids": rng.integers(0, vocab, seq).astype(np.int64)}
    return model(n, inits, ["ids"], ["y"], raw=raw), feeds
