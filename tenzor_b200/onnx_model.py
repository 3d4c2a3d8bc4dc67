"""Reading an ONNX model file and running it on the CUDA op map (tenzor_b200.onnx_ops).

The reference reads `.onnx` files with its own protobuf decoder (src/onnx/proto.zig, parser.zig:
parseModel 40-100, parseGraphProto 129-196, parseNodeProto 198-251, parseAttributeProto 253-330,
parseTensorProto 332-427) and executes the graph with Executor.run (executor.zig:712-816).  This
module is the same reader on the host, written from the protobuf wire format (varint / 64-bit /
length-delimited / 32-bit fields) and onnx.proto3's field numbers, keeping what a BERT-style graph
needs: the nodes with their attributes, the initializers (raw_data or the typed repeated fields),
and the graph's input and output names.  Unknown fields are skipped, as the reference does.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from .onnx_ops import Node, _c, run_graph

# TensorProto.DataType values used by encoder graphs (onnx.proto3)
_DTYPES = {1: np.float32, 2: np.uint8, 3: np.int8, 5: np.int16, 6: np.int32, 7: np.int64, 9: np.bool_,
           10: np.float16, 11: np.float64, 12: np.uint32, 13: np.uint64}


class OnnxFormatError(ValueError):
    pass


class _Reader:
    """Protobuf wire-format reader over one message's bytes."""

    def __init__(self, data: bytes):
        self.d = memoryview(data)
        self.p = 0

    def more(self) -> bool:
        return self.p < len(self.d)

    def varint(self) -> int:
        v = shift = 0
        while True:
            if self.p >= len(self.d):
                raise OnnxFormatError("truncated varint")
            b = self.d[self.p]
            self.p += 1
            v |= (b & 0x7F) << shift
            if b < 0x80:
                return v
            shift += 7
            if shift > 63:
                raise OnnxFormatError("varint longer than 10 bytes")

    def header(self):
        key = self.varint()
        return key >> 3, key & 7

    def take(self, n: int) -> memoryview:
        if self.p + n > len(self.d):
            raise OnnxFormatError("truncated field")
        out = self.d[self.p:self.p + n]
        self.p += n
        return out

    def bytes_(self) -> bytes:
        return bytes(self.take(self.varint()))

    def skip(self, wire: int):
        if wire == 0:
            self.varint()
        elif wire == 1:
            self.take(8)
        elif wire == 2:
            self.take(self.varint())
        elif wire == 5:
            self.take(4)
        else:
            raise OnnxFormatError(f"unsupported wire type {wire}")


def _signed64(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _packed_or_single(r: _Reader, wire: int, kind: str):
    """Repeated scalar field: packed (wire 2) or one element (wire 0 / 5 / 1)."""
    if wire == 2:
        sub = _Reader(r.bytes_())
        vals = []
        while sub.more():
            if kind == "varint":
                vals.append(_signed64(sub.varint()))
            elif kind == "f32":
                vals.append(struct.unpack("<f", sub.take(4))[0])
            else:
                vals.append(struct.unpack("<d", sub.take(8))[0])
        return vals
    if kind == "varint":
        return [_signed64(r.varint())]
    if kind == "f32":
        return [struct.unpack("<f", r.take(4))[0]]
    return [struct.unpack("<d", r.take(8))[0]]


def _tensor(data: bytes):
    """TensorProto -> (name, numpy array)."""
    r = _Reader(data)
    dims, dtype, name, raw = [], 1, "", None
    floats, int32s, int64s, doubles = [], [], [], []
    while r.more():
        f, w = r.header()
        if f == 1:
            dims += _packed_or_single(r, w, "varint")
        elif f == 2:
            dtype = r.varint()
        elif f == 4:
            floats += _packed_or_single(r, w, "f32")
        elif f == 5:
            int32s += _packed_or_single(r, w, "varint")
        elif f == 7:
            int64s += _packed_or_single(r, w, "varint")
        elif f == 8:
            name = r.bytes_().decode()
        elif f == 9:
            raw = r.bytes_()
        elif f == 10:
            doubles += _packed_or_single(r, w, "f64")
        else:
            r.skip(w)
    if dtype not in _DTYPES:
        raise OnnxFormatError(f"tensor {name}: unsupported data type {dtype}")
    np_t = _DTYPES[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=np.dtype(np_t).newbyteorder("<")).astype(np_t)
    elif floats:
        arr = np.asarray(floats, np.float32)
    elif int64s:
        arr = np.asarray(int64s, np.int64)
    elif doubles:
        arr = np.asarray(doubles, np.float64)
    else:
        arr = np.asarray(int32s, np.int32).astype(np_t)  # int32_data also carries the narrower types
    n = int(np.prod(dims)) if dims else 1
    if arr.size != n:
        raise OnnxFormatError(f"tensor {name}: {arr.size} values for dims {dims}")
    return name, arr.reshape(dims)


def _attribute(data: bytes):
    r = _Reader(data)
    name, val, ints, floats = "", None, [], []
    while r.more():
        f, w = r.header()
        if f == 1:
            name = r.bytes_().decode()
        elif f == 2:
            val = struct.unpack("<f", r.take(4))[0]
        elif f == 3:
            val = _signed64(r.varint())
        elif f == 4:
            val = r.bytes_().decode(errors="replace")
        elif f == 5:
            val = _tensor(r.bytes_())[1]
        elif f == 7:
            floats += _packed_or_single(r, w, "f32")
        elif f == 8:
            ints += _packed_or_single(r, w, "varint")
        else:
            r.skip(w)
    if val is None:
        val = ints if ints else floats
    return name, val


def _node(data: bytes) -> Node:
    r = _Reader(data)
    ins, outs, op, attrs = [], [], "", {}
    while r.more():
        f, w = r.header()
        if f == 1:
            ins.append(r.bytes_().decode())
        elif f == 2:
            outs.append(r.bytes_().decode())
        elif f == 4:
            op = r.bytes_().decode()
        elif f == 5:
            k, v = _attribute(r.bytes_())
            attrs[k] = v
        else:
            r.skip(w)
    return Node(op, ins, outs, attrs)  # an empty name stands for an omitted optional input


def _value_info_name(data: bytes) -> str:
    r = _Reader(data)
    while r.more():
        f, w = r.header()
        if f == 1:
            return r.bytes_().decode()
        r.skip(w)
    return ""


@dataclass
class OnnxModel:
    nodes: list
    initializers: dict            # name -> numpy array
    inputs: list                  # graph inputs that are not initializers
    outputs: list
    opset: dict = field(default_factory=dict)  # domain -> version
    ir_version: int = 0


def parse_model(data: bytes) -> OnnxModel:
    """ModelProto bytes -> OnnxModel (parseModel, parser.zig:40-100)."""
    r = _Reader(data)
    graph, opset, ir = None, {}, 0
    while r.more():
        f, w = r.header()
        if f == 1:
            ir = r.varint()
        elif f == 7:
            graph = r.bytes_()
        elif f == 8:
            sub = _Reader(r.bytes_())
            dom, ver = "", 0
            while sub.more():
                g, ww = sub.header()
                if g == 1:
                    dom = sub.bytes_().decode()
                elif g == 2:
                    ver = sub.varint()
                else:
                    sub.skip(ww)
            opset[dom] = ver
        else:
            r.skip(w)
    if graph is None:
        raise OnnxFormatError("model has no graph")
    g = _Reader(graph)
    nodes, inits, ins, outs = [], {}, [], []
    while g.more():
        f, w = g.header()
        if f == 1:
            nodes.append(_node(g.bytes_()))
        elif f == 5:
            k, v = _tensor(g.bytes_())
            inits[k] = v
        elif f == 11:
            ins.append(_value_info_name(g.bytes_()))
        elif f == 12:
            outs.append(_value_info_name(g.bytes_()))
        else:
            g.skip(w)
    return OnnxModel(nodes, inits, [i for i in ins if i not in inits], outs, opset, ir)


def load(path: str) -> OnnxModel:
    with open(path, "rb") as fh:
        return parse_model(fh.read())


def run(ctx, model: OnnxModel, feeds: dict, spec: bool = False, precision: str = "f32x3"):
    """Executes the model on the device: floating-point initializers and feeds become f32 CUDA
    tensors, integer feeds int64 CUDA tensors, integer initializers stay host arrays (the value model
    of tenzor_b200.onnx_ops), then run_graph walks the nodes.  Returns the outputs."""
    import torch

    def value(a, feed):
        a = np.asarray(a)
        if np.issubdtype(a.dtype, np.floating):
            return torch.from_numpy(_c(a, np.float32)).cuda()
        if feed:  # integer data (ids, masks) go to the device
            return torch.from_numpy(_c(a, np.int64)).cuda()
        return _c(a)  # integer constants (axes, shapes, position ids) stay host metadata
    inits = {k: value(v, False) for k, v in model.initializers.items()}
    missing = [i for i in model.inputs if i not in feeds]
    if missing:
        raise KeyError(f"missing graph inputs {missing}")
    return run_graph(ctx, model.nodes, inits, {k: value(v, True) for k, v in feeds.items()}, model.outputs, spec=spec,
                     precision=precision)
