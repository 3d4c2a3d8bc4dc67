"""WordPiece tokenizer (tz_tokenizer.cpp) and the embed CLI's text paths (tz_arctic_embed_texts /
tz_arctic_embed_documents) against the restatement in oracle/wordpiece.py.

CPU: the restatement and the C++ tokenizer on the reference's own known-answer tests
(tokenizer.zig:291-439), on the HuggingFace cases of tokenizer_parity_test.zig:15-31 whose
vocabulary entries the expected ids imply, and on seeded random texts and vocabularies (truncation,
long words, non-ASCII bytes, CRLF vocab files, repeated tokens).  GPU: text batches and long
documents (chunking + device mean pooling) against the oracle forward.
"""
import random

import numpy as np
import pytest

import kats
import wordpiece as W


def _lib_tokenizer(vocab: dict):
    from tenzor_b200.tokenizer import Tokenizer
    t = Tokenizer()
    for k, v in vocab.items():
        t.put(k, v)
    return t


def _bvocab(vocab: dict) -> dict:
    return {k.encode(): v for k, v in vocab.items()}


@pytest.mark.parametrize("case", kats.TOKENIZER, ids=[c[0] for c in kats.TOKENIZER])
def test_reference_known_answers(case):
    _, vocab, text, expected = case
    assert W.encode(_bvocab(vocab), text.encode(), 32) == expected
    t = _lib_tokenizer(vocab)
    assert t.encode(text, 32).tolist() == expected


def _basic_tokens(text: bytes):
    """The basic split of encode (whitespace runs dropped, punctuation bytes alone)."""
    out, i = [], 0
    while i < len(text):
        while i < len(text) and text[i] in W.WS:
            i += 1
        w0 = i
        while i < len(text) and text[i] not in W.WS and text[i] not in W.PUNCT:
            i += 1
        if i > w0:
            out.append(text[w0:i].lower())
        if i < len(text) and text[i] in W.PUNCT:
            out.append(text[i:i + 1])
            i += 1
    return out


def _hf_implied():
    vocab, cases = {}, []
    for text, ids in kats.TOKENIZER_HF:
        toks = _basic_tokens(text.encode())
        if len(toks) != len(ids) - 2:  # a word of several pieces: its split is not implied
            continue
        for tok, i in zip(toks, ids[1:-1]):
            assert vocab.setdefault(tok, i) == i, "the golden cases disagree"
        cases.append((text, ids))
    return vocab, cases


def test_hf_golden_cases_with_implied_vocab():
    vocab, cases = _hf_implied()
    assert len(cases) == 13  # all but "embeddings" and "I love programming in Zig!"
    from tenzor_b200.tokenizer import Tokenizer
    t = Tokenizer()
    for k, v in vocab.items():
        t.put(k, v)
    for text, ids in cases:
        assert W.encode(vocab, text.encode(), 512) == ids, text
        assert t.encode(text, 512).tolist() == ids, text


ALPHABET = b"abcdefghijAB XYZ\t\n\r,.!?-'#_\xc3\xa9\xe2\x82\xac0123"


def _random_vocab(rng, n=300):
    words = set()
    while len(words) < n:
        L = rng.randint(1, 6)
        w = bytes(rng.choice(b"abcdefghij0123\xc3\xa9") for _ in range(L))
        words.add((b"##" + w) if rng.random() < 0.4 else w)
    words |= {b",", b".", b"!", b"#", b"-"}
    return {w: rng.randrange(1000, 30000) for w in sorted(words)}


def _random_text(rng, n):
    parts = []
    for _ in range(n):
        r = rng.random()
        if r < 0.05:
            parts.append(bytes(rng.choice(b"abc") for _ in range(rng.randint(195, 210))))  # around the 200-byte limit
        else:
            parts.append(bytes(rng.choice(ALPHABET) for _ in range(rng.randint(1, 12))))
    return b" ".join(parts)


@pytest.mark.parametrize("seed", range(6))
def test_random_texts_match_restatement(seed):
    rng = random.Random(seed)
    vocab = _random_vocab(rng)
    t = _lib_tokenizer({})
    for k, v in vocab.items():
        t.put(k, v)
    texts = [_random_text(rng, rng.randint(0, 60)) for _ in range(80)]
    for text in texts:
        raw = W.encode_raw(vocab, text)
        assert t.encode_raw(text).tolist() == raw
        for cap in (2, 3, 7, 40, 512):
            assert t.encode(text, cap).tolist() == W.encode(vocab, text, cap), (text, cap)
    ids, cu = t.encode_batch(texts, 64)
    for i, text in enumerate(texts):
        assert ids[cu[i]:cu[i + 1]].tolist() == W.encode(vocab, text, 64)


def test_vocab_file_format(tmp_path):
    # empty lines and a lone "\r" take an index, CRLF is stripped, a repeated token keeps its last index
    data = b"[PAD]\n\n[UNK]\r\n\r\nhello\nworld\r\nhello\n##s\n"
    ref = W.vocab_from_bytes(data)
    assert ref == {b"[PAD]": 0, b"[UNK]": 2, b"hello": 6, b"world": 5, b"##s": 7}
    from tenzor_b200.tokenizer import Tokenizer
    a, b = Tokenizer(), Tokenizer()
    a.load_vocab_from_bytes(data)
    p = tmp_path / "vocab.txt"
    p.write_bytes(data)
    b.load_vocab(str(p))
    assert len(a) == len(b) == 5
    for text in ("hello worlds", "HELLO, world", "hellos"):
        want = W.encode(ref, text.encode(), 16)
        assert a.encode(text, 16).tolist() == want and b.encode(text, 16).tolist() == want


def test_missing_vocab_file_is_an_error(tmp_path):
    from tenzor_b200 import _lib as L
    from tenzor_b200.tokenizer import Tokenizer
    with pytest.raises(L.TenzorError):
        Tokenizer().load_vocab(str(tmp_path / "absent.txt"))


def test_encode_needs_room_for_markers():
    from tenzor_b200 import _lib as L
    t = _lib_tokenizer({"a": 5})
    with pytest.raises(L.TenzorError):
        t.encode("a", 1)
    assert t.encode("", 2).tolist() == [101, 102]
    assert t.encode("a a a", 3).tolist() == [101, 5, 102]


def test_chunk_count_formula():
    from tenzor_b200.tokenizer import doc_chunk_count
    for T in list(range(0, 2000, 7)) + [510, 511, 970, 971, 972, 1431, 1432, 100000]:
        assert doc_chunk_count(T) == W.chunk_count(T)
    # the reference's count, kept as written: 511 raw ids make one chunk, the last id is dropped
    assert W.chunk_count(511) == 1 and W.document_chunks(list(range(511)))[0][-2] == 509


# ---- GPU: text batches and long documents through the model -------------------------------------

MAX_ABS, MIN_COS = 2e-3, 0.9999


def _close(y, ref):
    d = np.abs(y - ref).max()
    c = ((y * ref).sum(1) / np.linalg.norm(y, axis=1) / np.linalg.norm(ref, axis=1)).min()
    assert d <= MAX_ABS and c >= MIN_COS, f"max-abs {d:.3e}, min cos {c:.7f}"


def _doc_vocab(seed=21):
    rng = random.Random(seed)
    vocab = {}
    for i in range(2000):
        w = "".join(rng.choice("abcdefghijklmnop") for _ in range(rng.randint(1, 5)))
        vocab[("##" + w) if rng.random() < 0.3 else w] = rng.randrange(1000, 30000)
    for p in ",.!?":
        vocab[p] = rng.randrange(1000, 30000)
    return vocab


def _doc_text(rng, words):
    return " ".join("".join(rng.choice("abcdefghijklmnopqrstuvwxyzABC,.") for _ in range(rng.randint(1, 8)))
                    for _ in range(words))


@pytest.fixture(scope="module")
def tok_setup(ctx, oracle):
    from tenzor_b200 import synthetic as S
    from tenzor_b200.arctic import ArcticModel
    from tenzor_b200.tokenizer import Tokenizer
    vocab = _doc_vocab()
    t = Tokenizer()
    for k, v in vocab.items():
        t.put(k, v)
    w = S.arctic_weights(77)
    model = ArcticModel.from_checkpoint(ctx, w, "f32")
    ref = oracle.OracleModel(w)
    yield t, {k.encode(): v for k, v in vocab.items()}, model, ref, oracle
    model.close()


def _oracle_embed(ref, oracle, seqs):
    cu = np.zeros(len(seqs) + 1, np.int32)
    cu[1:] = np.cumsum([len(s) for s in seqs])
    return ref.forward(np.concatenate([np.asarray(s, np.uint32) for s in seqs]), cu, oracle.MODE_F32)


@pytest.mark.gpu
def test_embed_texts_vs_oracle(tok_setup):
    t, bv, model, ref, oracle = tok_setup
    rng = random.Random(5)
    texts = [_doc_text(rng, rng.randint(0, 60)) for _ in range(12)] + [_doc_text(rng, 400)]  # the last one truncates at 512
    y = model.embed_texts(t, texts)
    seqs = [W.encode(bv, s.encode(), 512) for s in texts]
    assert len(seqs[-1]) == 512
    _close(y, _oracle_embed(ref, oracle, seqs))


@pytest.mark.gpu
def test_embed_documents_vs_oracle(tok_setup):
    t, bv, model, ref, oracle = tok_setup
    rng = random.Random(9)
    docs = ["", _doc_text(rng, 30), _doc_text(rng, 700), _doc_text(rng, 1500)]
    y = model.embed_documents(t, docs)
    want = []
    for d in docs:
        chunks = W.document_chunks(W.encode_raw(bv, d.encode()))
        want.append(W.pool_document(_oracle_embed(ref, oracle, chunks)))
    assert [W.chunk_count(len(W.encode_raw(bv, d.encode()))) for d in docs][2:] != [1, 1]  # several chunks
    _close(y, np.stack(want))
    assert np.abs(np.linalg.norm(y, axis=1) - 1).max() < 1e-5
