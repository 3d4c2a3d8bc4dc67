"""WordPiece tokenizer of the embed path (tz_tokenizer.cpp through the C ABI).

Mirrors the reference's ``Tokenizer`` (src/io/tokenizer.zig:9-266): ``load_vocab`` /
``load_vocab_from_bytes`` (one token per line, id = line index), ``put`` (``vocab.put``, as the
reference's tests build vocabularies), ``encode`` (``[CLS] ... [SEP]`` into a buffer of ``max_len``
ids, tokenizer.zig:77-121) and ``encode_raw`` (no markers, no limit, tokenizer.zig:123-200).  Texts
are ``str`` (UTF-8 encoded) or ``bytes``; the algorithm works on bytes like the reference.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L

UNK_ID, CLS_ID, SEP_ID = 100, 101, 102


def _bytes(text) -> bytes:
    return text.encode("utf-8") if isinstance(text, str) else bytes(text)


class Tokenizer:
    """Host WordPiece vocabulary; thread-safe for concurrent encodes once loaded."""

    def __init__(self):
        h = C.c_void_p()
        L.check(L.lib().tz_tokenizer_create(C.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            L.lib().tz_tokenizer_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_special(self, unk_id: int = UNK_ID, cls_id: int = CLS_ID, sep_id: int = SEP_ID):
        L.check(L.lib().tz_tokenizer_set_special(self.handle, unk_id, cls_id, sep_id))

    def load_vocab(self, path: str):
        L.check(L.lib().tz_tokenizer_load_vocab(self.handle, path.encode()))

    def load_vocab_from_bytes(self, data: bytes):
        data = bytes(data)
        L.check(L.lib().tz_tokenizer_load_vocab_bytes(self.handle, data, len(data)))

    def put(self, token, token_id: int):
        b = _bytes(token)
        L.check(L.lib().tz_tokenizer_put(self.handle, b, len(b), token_id))

    def __len__(self) -> int:
        n = C.c_int64()
        L.check(L.lib().tz_tokenizer_vocab_size(self.handle, C.byref(n)))
        return n.value

    def encode(self, text, max_len: int = 512) -> np.ndarray:
        b = _bytes(text)
        out = np.empty(max_len, np.uint32)
        n = C.c_int64()
        L.check(L.lib().tz_tokenizer_encode(self.handle, b, len(b), out.ctypes.data, max_len, C.byref(n)))
        return out[:n.value].copy()

    def encode_raw(self, text) -> np.ndarray:
        b = _bytes(text)
        n = C.c_int64()
        L.check(L.lib().tz_tokenizer_encode_raw(self.handle, b, len(b), None, 0, C.byref(n)))
        out = np.empty(max(n.value, 1), np.uint32)
        L.check(L.lib().tz_tokenizer_encode_raw(self.handle, b, len(b), out.ctypes.data, out.size, C.byref(n)))
        return out[:n.value].copy()

    def encode_batch(self, texts, max_len: int = 512):
        """encode of every text -> (packed ids uint32 [T], cu_seqlens int32 [n + 1])."""
        bufs = [_bytes(t) for t in texts]
        n = len(bufs)
        ptrs = (C.c_char_p * max(n, 1))(*bufs)
        lens = np.array([len(b) for b in bufs] or [0], np.int64)
        ids = np.empty(max(n * max_len, 1), np.uint32)
        cu = np.empty(n + 1, np.int32)
        L.check(L.lib().tz_tokenizer_encode_batch(self.handle, C.cast(ptrs, C.c_void_p), lens.ctypes.data, n, max_len,
                                                  ids.ctypes.data, cu.ctypes.data, ids.size))
        return ids[:cu[-1]].copy(), cu


def doc_chunk_count(tokens: int) -> int:
    """Chunks of a document of ``tokens`` raw ids (main.zig:806-809)."""
    return int(L.lib().tz_doc_chunk_count(tokens))


def text_args(texts):
    """(bytes list kept alive, char** array, int64 lengths) for the embed entry points."""
    bufs = [_bytes(t) for t in texts]
    ptrs = (C.c_char_p * max(len(bufs), 1))(*bufs)
    lens = np.array([len(b) for b in bufs] or [0], np.int64)
    return bufs, ptrs, lens
