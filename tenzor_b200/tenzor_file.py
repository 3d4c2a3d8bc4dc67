"""The reference's ``.tenzor`` checkpoint format (src/io/tenzor_format.zig).

Layout (tenzor_format.zig:1-13, 66-104): a 64-byte header (magic ``TENZOR\\0\\0``, u32 version 1,
u32 flags, u32 tensor_count, u32 pad, u64 index_offset, u64 data_offset, u32 metadata_size, 20
reserved bytes), the metadata JSON padded to 8 bytes, ``tensor_count`` 48-byte index entries
(u64 FNV-1a hash of the name, u8 dtype, u8 ndim, 2 pad bytes, u32 shape[5], u64 offset into the data
section, u64 size) and the tensor bytes back to back from a 4 KiB-aligned data offset.

``write`` follows TenzorWriter.finish (tenzor_format.zig:365-429) and ``convert_from_safetensors``
convertFromSafetensors (441-485).  Reading goes through the C library (``tz_tenzor_*``: the file is
memory-mapped, as TenzorFile.open does), which is also what ``LeNet.from_tenzor`` and
``ArcticModel.from_tenzor`` use.
"""
from __future__ import annotations

import ctypes as C
import json
import struct

import numpy as np

from . import _lib as L

MAGIC = b"TENZOR\x00\x00"
PAGE = 4096
# DType (tenzor_format.zig:26-38)
DTYPES = {0: np.float32, 1: np.float16, 2: None, 3: np.float64, 4: np.int8, 5: np.int16, 6: np.int32,
          7: np.int64, 8: np.uint8, 9: np.uint16, 10: np.uint32, 11: np.uint64}
_CODE = {np.dtype(v).str: k for k, v in DTYPES.items() if v is not None}


def hash_name(name: str) -> int:
    """hashName (tenzor_format.zig:107-114): FNV-1a 64 of the UTF-8 bytes."""
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _align(v: int, a: int) -> int:
    return (v + a - 1) & ~(a - 1)


def write(path: str, tensors, metadata_json: str = "{}"):
    """Writes ``tensors`` (a dict, or (name, array[, dtype code[, shape]]) tuples in order) as a
    .tenzor file.  An explicit dtype code stores the array's bytes under that code (bf16 as uint16
    data: code 2); with a shape too, the array is raw bytes reinterpreted as that dtype and shape."""
    items = []
    for it in (tensors.items() if isinstance(tensors, dict) else tensors):
        name, arr = it[0], np.asarray(it[1])  # tobytes() below writes C order; keeps 0-d arrays 0-d
        code = it[2] if len(it) > 2 else _CODE.get(arr.dtype.str)
        if len(it) > 3:  # raw bytes with an explicit shape
            arr = arr.view(DTYPES[code] or np.uint16).reshape(it[3])
        if code is None:
            raise ValueError(f"{name}: dtype {arr.dtype} has no .tenzor code")
        if arr.ndim > 5:
            raise ValueError(f"{name}: {arr.ndim} dimensions, the index holds 5")
        items.append((name, arr, code))
    meta = metadata_json.encode()
    index_offset = 64 + _align(len(meta), 8)
    data_offset = _align(index_offset + 48 * len(items), PAGE)
    header = MAGIC + struct.pack("<IIII", 1, 0, len(items), 0) + struct.pack("<QQI", index_offset, data_offset, len(meta))
    header += b"\x00" * (64 - len(header))
    index, off = b"", 0
    for name, arr, code in items:
        shape = list(arr.shape) + [0] * (5 - arr.ndim)
        index += struct.pack("<QBBxx5IQQ", hash_name(name), code, arr.ndim, *shape, off, arr.nbytes)
        off += arr.nbytes
    with open(path, "wb") as f:
        f.write(header)
        f.write(meta + b"\x00" * (index_offset - 64 - len(meta)))
        f.write(index)
        f.write(b"\x00" * (data_offset - index_offset - len(index)))
        for _, arr, _ in items:
            f.write(arr.tobytes())


# safetensors dtype -> .tenzor DType, as convertFromSafetensors maps them (tenzor_format.zig:460-473)
_FROM_ST = {"F32": 0, "F16": 1, "BF16": 2, "F64": 3, "I8": 4, "I16": 5, "I32": 6, "I64": 7, "U8": 8,
            "U16": 9, "U32": 10, "U64": 11, "BOOL": 8}


def convert_from_safetensors(src: str, dst: str):
    """convertFromSafetensors: every tensor keeps its name, its declared dtype and its bytes."""
    with open(src, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    items = []
    for name, info in header.items():
        if name == "__metadata__":
            continue
        s, e = info["data_offsets"]
        code = _FROM_ST[info["dtype"]]
        words = np.frombuffer(raw[8 + n + s:8 + n + e], dtype=np.uint8)
        items.append((name, words, code, tuple(info["shape"])))
    write(dst, items)


class TenzorFile:
    """A memory-mapped .tenzor file (TenzorFile, tenzor_format.zig:117-287), read by the C library."""

    def __init__(self, path: str):
        h = C.c_void_p()
        L.check(L.lib().tz_tenzor_open(path.encode(), C.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            L.lib().tz_tenzor_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __len__(self) -> int:
        return int(L.lib().tz_tenzor_count(self.handle))

    def _array(self, e: L.TenzorEntry) -> np.ndarray:
        dt = DTYPES[e.dtype] or np.uint16  # bf16 comes back as its raw 16-bit words
        shape = tuple(e.shape[i] for i in range(e.ndim))
        buf = (C.c_uint8 * e.bytes).from_address(e.data) if e.bytes else b""
        return np.frombuffer(buf, dtype=dt).reshape(shape).copy()

    def entry(self, i: int) -> dict:
        e = L.TenzorEntry()
        L.check(L.lib().tz_tenzor_entry_at(self.handle, i, C.byref(e)))
        return {"name_hash": e.name_hash, "dtype": e.dtype, "shape": tuple(e.shape[j] for j in range(e.ndim)),
                "bytes": e.bytes}

    def get(self, name: str) -> np.ndarray:
        """getTensor + getData: a copy of the tensor's data (TenzorError TZ_EMISSING if absent)."""
        e = L.TenzorEntry()
        L.check(L.lib().tz_tenzor_find(self.handle, name.encode(), C.byref(e)))
        return self._array(e)

    def metadata(self) -> dict:
        p, n = C.c_char_p(), C.c_uint64()
        L.check(L.lib().tz_tenzor_metadata(self.handle, C.byref(p), C.byref(n)))
        raw = C.string_at(p, n.value) if n.value else b"{}"
        return json.loads(raw.decode())
