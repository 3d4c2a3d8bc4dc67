"""safetensors read/write in numpy (mirror of the reference's src/io/safetensors.zig:172-411).

Layout: u64 little-endian header length, a JSON header {name: {dtype, shape, data_offsets}},
then the tensor bytes.  int8 checkpoints carry '<name>.scale' F16 vectors
(quantize_arctic_xs.zig:139).  The model loader in the C library (tz_arctic_load_safetensors)
reads the same files without Python.
"""
from __future__ import annotations

import json
import struct

import numpy as np

_DT = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8, "I32": np.int32,
       "I64": np.int64, "F64": np.float64, "BF16": np.uint16, "U16": np.uint16}
_NAME = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int8): "I8",
         np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32", np.dtype(np.int64): "I64",
         np.dtype(np.float64): "F64"}


def save(path: str, tensors: dict, f16_names=()):
    """Writes name -> array.  Arrays of uint16 listed in `f16_names` (or named '*.scale') are
    stored as F16 bit patterns."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        if a.dtype == np.uint16 and (name in f16_names or name.endswith(".scale")):
            dt = "F16"
        else:
            dt = _NAME[a.dtype]
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def load(path: str) -> dict:
    """name -> array (F16 tensors come back as uint16 bit patterns, the form the C ABI takes)."""
    with open(path, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        s, e = info["data_offsets"]
        dt = _DT[info["dtype"]]
        a = np.frombuffer(raw[base + s:base + e], dtype=dt).reshape(info["shape"]).copy()
        out[name] = a.view(np.uint16) if info["dtype"] == "F16" else a
    return out
