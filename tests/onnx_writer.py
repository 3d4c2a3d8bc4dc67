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


def bert_layer_exported(seed: int = 0, batch: int = 2, seq: int = 16, hidden: int = 384, heads: int = 12,
                        ffn: int = 1536, vocab: int = 200, max_pos: int = 64, decomposed_ln: bool = False,
                        where_mask: bool = False, raw: bool = True):
    """A batched BERT embedding block + one encoder layer (Arctic-embed-xs sizes by default: hidden
    384, 12 heads of 32, FFN 1536) written the way torch.onnx.export writes a HuggingFace BertModel:
    position / token-type ids sliced to the sequence length from Shape; the additive attention mask
    from Unsqueeze / Cast / Sub / Mul (or Equal / Where); per-head Reshape + Transpose of Q, K, V with
    the target shapes assembled by Shape / Gather / Unsqueeze / Concat; batched MatMul for the scores
    and the context, scaled by Div; exact GELU as the Erf decomposition; LayerNormalization (or, for
    opsets below 17, its ReduceMean / Sub / Pow / Sqrt / Div decomposition); and the CLS row pooled by
    a Gather on axis 1.  Weights N(0, 0.05).  Returns (model bytes, feeds)."""
    rng = np.random.default_rng(seed)
    w = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)
    ones = lambda n: (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    hd = hidden // heads
    i64 = lambda v: np.asarray(v, np.int64)
    f32 = lambda v: np.asarray(v, np.float32)
    inits = {
        "word": w(vocab, hidden), "pos": w(max_pos, hidden), "type": w(2, hidden),
        "position_ids": i64(np.arange(max_pos)[None, :]), "token_type_ids": i64(np.zeros((1, max_pos))),
        "ln_e_g": ones(hidden), "ln_e_b": w(hidden),
        "wq": w(hidden, hidden), "bq": w(hidden), "wk": w(hidden, hidden), "bk": w(hidden),
        "wv": w(hidden, hidden), "bv": w(hidden), "wo": w(hidden, hidden), "bo": w(hidden),
        "ln1_g": ones(hidden), "ln1_b": w(hidden), "w1": w(hidden, ffn), "b1": w(ffn), "w2": w(ffn, hidden),
        "b2": w(hidden), "ln2_g": ones(hidden), "ln2_b": w(hidden),
        "c0": i64([0]), "c1": i64([1]), "s0": i64(0), "s1": i64(1), "c_heads": i64([heads]), "c_hd": i64([hd]),
        "c_hidden": i64([hidden]), "f_one": f32(1.0), "f_min": f32(-3.4028234663852886e38), "f_zero": f32(0.0),
        "f_sqrt_hd": f32(np.sqrt(hd)), "f_sqrt2": f32(1.4142135381698608), "f_half": f32(0.5), "f_two": f32(2.0),
        "f_eps": f32(1e-12),
    }
    n = [
        node("Shape", ["input_ids"], ["ids_shape"]),
        node("Gather", ["ids_shape", "s1"], ["S"], axis=0),
        node("Unsqueeze", ["S"], ["S_u"], axes=[0]),
        node("Slice", ["position_ids", "c0", "S_u", "c1"], ["pos_ids"]),
        node("Slice", ["token_type_ids", "c0", "S_u", "c1"], ["tt_ids"]),
        node("Gather", ["word", "input_ids"], ["we"], axis=0),
        node("Gather", ["type", "tt_ids"], ["te"], axis=0),
        node("Add", ["we", "te"], ["e1"]),
        node("Gather", ["pos", "pos_ids"], ["pe"], axis=0),
        node("Add", ["e1", "pe"], ["e2"]),
    ]

    def layer_norm(x, g, b, y):
        if not decomposed_ln:
            return [node("LayerNormalization", [x, g, b], [y], axis=-1, epsilon=1e-12)]
        return [node("ReduceMean", [x], [y + "_mu"], axes=[-1], keepdims=1),
                node("Sub", [x, y + "_mu"], [y + "_d"]),
                node("Pow", [y + "_d", "f_two"], [y + "_sq"]),
                node("ReduceMean", [y + "_sq"], [y + "_var"], axes=[-1], keepdims=1),
                node("Add", [y + "_var", "f_eps"], [y + "_ve"]),
                node("Sqrt", [y + "_ve"], [y + "_sd"]),
                node("Div", [y + "_d", y + "_sd"], [y + "_n"]),
                node("Mul", [y + "_n", g], [y + "_s"]),
                node("Add", [y + "_s", b], [y])]

    n += layer_norm("e2", "ln_e_g", "ln_e_b", "x0")
    n += [node("Unsqueeze", ["attention_mask"], ["m1"], axes=[1]),
          node("Unsqueeze", ["m1"], ["m2"], axes=[2])]
    if where_mask:  # newer exporters: where(mask == 0, finfo.min, 0)
        n += [node("Equal", ["m2", "c0"], ["m_eq"]),
              node("Where", ["m_eq", "f_min", "f_zero"], ["mask"])]
    else:  # (1 - mask) * finfo.min
        n += [node("Cast", ["m2"], ["m3"], to=1),
              node("Sub", ["f_one", "m3"], ["m4"]),
              node("Mul", ["m4", "f_min"], ["mask"])]
    n += [node("Shape", ["x0"], ["x_shape"]),
          node("Gather", ["x_shape", "s0"], ["B"], axis=0),
          node("Gather", ["x_shape", "s1"], ["S2"], axis=0),
          node("Unsqueeze", ["B"], ["B_u"], axes=[0]),
          node("Unsqueeze", ["S2"], ["S2_u"], axes=[0]),
          node("Concat", ["B_u", "S2_u", "c_heads", "c_hd"], ["head_shape"], axis=0),
          node("Concat", ["B_u", "S2_u", "c_hidden"], ["flat_shape"], axis=0)]
    for nm, perm in (("q", [0, 2, 1, 3]), ("k", [0, 2, 3, 1]), ("v", [0, 2, 1, 3])):
        n += [node("MatMul", ["x0", "w" + nm], [nm + "0"]),
              node("Add", ["b" + nm, nm + "0"], [nm + "1"]),
              node("Reshape", [nm + "1", "head_shape"], [nm + "2"]),
              node("Transpose", [nm + "2"], [nm + "t"], perm=perm)]
    n += [node("MatMul", ["qt", "kt"], ["sc"]),
          node("Div", ["sc", "f_sqrt_hd"], ["sc2"]),
          node("Add", ["sc2", "mask"], ["sc3"]),
          node("Softmax", ["sc3"], ["p"], axis=-1),
          node("MatMul", ["p", "vt"], ["ctx"]),
          node("Transpose", ["ctx"], ["ctx_t"], perm=[0, 2, 1, 3]),
          node("Reshape", ["ctx_t", "flat_shape"], ["c"]),
          node("MatMul", ["c", "wo"], ["o0"]), node("Add", ["o0", "bo"], ["o"]),
          node("Add", ["o", "x0"], ["r1"])]
    n += layer_norm("r1", "ln1_g", "ln1_b", "x1")
    n += [node("MatMul", ["x1", "w1"], ["h0"]), node("Add", ["h0", "b1"], ["h"]),
          node("Div", ["h", "f_sqrt2"], ["g1"]), node("Erf", ["g1"], ["g2"]),
          node("Add", ["g2", "f_one"], ["g3"]), node("Mul", ["h", "g3"], ["g4"]),
          node("Mul", ["g4", "f_half"], ["g"]),
          node("MatMul", ["g", "w2"], ["f0"]), node("Add", ["f0", "b2"], ["f"]),
          node("Add", ["f", "x1"], ["r2"])]
    n += layer_norm("r2", "ln2_g", "ln2_b", "y")
    n += [node("Gather", ["y", "s0"], ["cls"], axis=1)]
    ids = rng.integers(1, vocab, (batch, seq)).astype(np.int64)
    mask = np.ones((batch, seq), np.int64)
    for b in range(batch):  # ragged valid lengths, padding id 0
        L = int(rng.integers(seq // 2, seq + 1))
        mask[b, L:] = 0
        ids[b, L:] = 0
    feeds = {"input_ids": ids, "attention_mask": mask}
    return model(n, inits, ["input_ids", "attention_mask"], ["y", "cls"], opset=17, raw=raw), feeds


def mha_model(seed: int = 0, batch: int = 2, seq: int = 16, hidden: int = 384, num_heads: int = 12,
              with_mask: bool = False):
    """A com.microsoft MultiHeadAttention node over projected Q / K / V (as ORT's transformer optimizer
    fuses an exported attention block), with the num_heads attribute and an optional
    key_padding_mask [B, S].  Returns (model bytes, feeds)."""
    rng = np.random.default_rng(seed)
    w = lambda *s: (rng.standard_normal(s) * 0.05).astype(np.float32)
    inits = {"wq": w(hidden, hidden), "wk": w(hidden, hidden), "wv": w(hidden, hidden)}
    ins = ["q", "k", "v", ""] + (["kpm"] if with_mask else [])
    n = [node("MatMul", ["x", "wq"], ["q"]), node("MatMul", ["x", "wk"], ["k"]), node("MatMul", ["x", "wv"], ["v"]),
         node("MultiHeadAttention", ins, ["o"], num_heads=num_heads)]
    x = rng.standard_normal((batch, seq, hidden)).astype(np.float32)
    feeds = {"x": x}
    graph_in = ["x"]
    if with_mask:
        m = np.ones((batch, seq), np.int64)
        m[0, seq // 2:] = 0
        feeds["kpm"] = m
        graph_in.append("kpm")
    return model(n, inits, graph_in, ["o"], opset=17), feeds
