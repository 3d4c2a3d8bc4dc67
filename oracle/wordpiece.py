"""Pure-Python restatement of the reference's WordPiece tokenizer and the embed CLI's long-document
chunking / pooling, as the checker of tz_tokenizer.cpp and tz_arctic_embed_documents.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the oracle.  The product never imports it.

Parity anchors: the reference's own known-answer tests (tokenizer.zig:291-439, mini vocabularies
given inline) pin this restatement exactly; the HuggingFace golden ids of
src/tests/tokenizer_parity_test.zig:15-31 need the real vocab.txt (absent), so they pin it only
through the single-piece words whose vocabulary entry the expected ids imply.
"""
from __future__ import annotations

import numpy as np

UNK, CLS, SEP = 100, 101, 102  # tokenizer.zig:11-13
MAX_WORD = 200                 # tokenizer.zig:14
PUNCT = set(b'!"#$%&\'()*+,-./:;<=>?@[\\]^_`{|}~')  # isPunctuation, tokenizer.zig:272-277
WS = set(b" \t\n\r")                                 # isWhitespace, tokenizer.zig:268-270


def vocab_from_bytes(data: bytes) -> dict:
    """loadVocabFromBytes (tokenizer.zig:53-74)."""
    vocab = {}
    for idx, line in enumerate(data.split(b"\n")):
        if not line:
            continue
        tok = line[:-1] if line.endswith(b"\r") else line
        if tok:
            vocab[tok] = idx
    return vocab


def _lower(word: bytes) -> bytes:  # toLower, tokenizer.zig:279-285 (ASCII only)
    return bytes(c + 32 if 65 <= c <= 90 else c for c in word)


def _word(vocab, word: bytes, out: list, start: int, limit):
    """tokenizeWord (tokenizer.zig:203-266) / tokenizeWordAppend (155-200); `limit` is cap - 1 for
    encode, None for encodeRaw.  Writes into `out` from `start`, returns the new length."""
    def put(i, v):
        if i < len(out):
            out[i] = v
        else:
            out.append(v)
    if len(word) > MAX_WORD:
        put(start, UNK)
        return start + 1
    low = _lower(word)
    pos, cs, first = start, 0, True
    while cs < len(low) and (limit is None or pos < limit):
        found = False
        for ce in range(len(low), cs, -1):
            sub = low[cs:ce] if first else b"##" + low[cs:ce]
            if sub in vocab:
                put(pos, vocab[sub])
                pos += 1
                cs, first, found = ce, False, True
                break
        if not found:
            if limit is None:
                del out[start:]
            put(start, UNK)
            return start + 1
    return pos


def encode(vocab, text: bytes, cap: int = 512) -> list:
    """encode (tokenizer.zig:77-121): [CLS] ... [SEP] within a buffer of `cap` ids."""
    assert cap >= 2
    out = [0] * cap
    out[0] = CLS
    pos, i, n = 1, 0, len(text)
    while i < n and pos < cap - 1:
        while i < n and text[i] in WS:
            i += 1
        if i >= n:
            break
        w0 = i
        while i < n and text[i] not in WS and text[i] not in PUNCT:
            i += 1
        if i > w0:
            pos = _word(vocab, text[w0:i], out, pos, cap - 1)
        if i < n and text[i] in PUNCT:
            if pos < cap - 1:
                out[pos] = vocab.get(text[i:i + 1], UNK)
                pos += 1
            i += 1
    out[pos] = SEP
    return out[:pos + 1]


def encode_raw(vocab, text: bytes) -> list:
    """encodeRaw (tokenizer.zig:123-152)."""
    out: list = []
    i, n = 0, len(text)
    while i < n:
        while i < n and text[i] in WS:
            i += 1
        if i >= n:
            break
        w0 = i
        while i < n and text[i] not in WS and text[i] not in PUNCT:
            i += 1
        if i > w0:
            _word(vocab, text[w0:i], out, len(out), None)
        if i < n and text[i] in PUNCT:
            out.append(vocab.get(text[i:i + 1], UNK))
            i += 1
    return out


CHUNK, OVERLAP = 510, 50  # main.zig:784-785


def chunk_count(tokens: int) -> int:
    """main.zig:806-809 (kept as written: the last chunk may end before the document does)."""
    return 1 if tokens <= CHUNK else 1 + (tokens - CHUNK + OVERLAP - 1) // (CHUNK - OVERLAP)


def document_chunks(raw: list) -> list:
    """[CLS] ids[start, min(start + 510, T)) [SEP] per chunk (main.zig:869-878)."""
    out = []
    for c in range(chunk_count(len(raw))):
        a = c * (CHUNK - OVERLAP)
        b = min(a + CHUNK, len(raw))
        out.append([CLS] + list(raw[a:b]) + [SEP])
    return out


def pool_document(chunk_embeddings: np.ndarray) -> np.ndarray:
    """main.zig:909-925: sum in chunk order, times 1/n, divide by the L2 norm when positive."""
    e = np.asarray(chunk_embeddings, np.float32)
    acc = np.zeros(e.shape[1], np.float32)
    for row in e:
        acc = (acc + row).astype(np.float32)
    acc = (acc * np.float32(np.float32(1.0) / np.float32(len(e)))).astype(np.float32)
    norm = np.float32(np.sqrt(np.float32(np.sum(acc.astype(np.float64) ** 2))))
    return (acc / norm).astype(np.float32) if norm > 0 else acc
