// tz_tokenizer.cpp -- BERT WordPiece tokenizer for the text -> device ids pipeline of the embed path.
//
// Behaviour of the reference's Tokenizer (src/io/tokenizer.zig), byte for byte:
//   * vocabulary: one token per line, the line index is the id; empty lines and a line that is a
//     lone "\r" take an index but no entry; one trailing "\r" is stripped; a repeated token keeps
//     its last index (loadVocabFromBytes, tokenizer.zig:53-74, StringHashMap.put);
//   * basic split (encode, tokenizer.zig:77-121): skip ' ', '\t', '\n', '\r'; a word is a run of
//     bytes that are neither whitespace nor ASCII punctuation (isPunctuation, tokenizer.zig:272-277);
//     each punctuation byte is its own token (its vocab id, else [UNK]);
//   * WordPiece (tokenizeWord, tokenizer.zig:203-266): a word longer than 200 bytes is one [UNK];
//     ASCII A-Z lowercased (toLower, tokenizer.zig:279-285); greedy longest match from the left,
//     continuation pieces prefixed "##"; a word with an unmatched remainder becomes one [UNK]
//     written at the word's first position;
//   * encode writes [CLS] ... [SEP] into a buffer of `cap` ids and stops taking tokens once one slot
//     is left for [SEP] (the loop conditions of tokenizer.zig:89, 227); encodeRaw
//     (tokenizer.zig:123-200) has no markers and no limit.
//   * [UNK] / [CLS] / [SEP] are the fixed ids 100 / 101 / 102 (tokenizer.zig:11-13), not looked up.
// Non-ASCII bytes are ordinary word bytes (no Unicode normalisation, as in the reference).
//
// The vocabulary is an open-addressing hash table over one byte arena (FNV-1a), so lookups of the
// candidate pieces need no allocation.  tz_tokenizer_encode_batch tokenizes many texts on host
// threads and packs them as (ids, cu_seqlens) for tz_arctic_forward / tz_arctic_forward_device.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include "tz_internal.h"

struct tz_tokenizer_s {
    struct Slot {
        uint32_t off = 0, len = 0, id = 0;
        bool used = false;
    };
    std::string arena;
    std::vector<Slot> table = std::vector<Slot>(1024);
    size_t count = 0;
    uint32_t unk_id = 100, cls_id = 101, sep_id = 102;
    size_t max_word_chars = 200;

    static uint64_t hash(const char* p, size_t n) {
        uint64_t h = 1469598103934665603ull;
        for (size_t i = 0; i < n; ++i) h = (h ^ static_cast<uint8_t>(p[i])) * 1099511628211ull;
        return h;
    }
    size_t probe(const char* p, size_t n, bool* found) const {
        const size_t mask = table.size() - 1;
        size_t i = static_cast<size_t>(hash(p, n)) & mask;
        while (table[i].used) {
            const Slot& s = table[i];
            if (s.len == n && memcmp(arena.data() + s.off, p, n) == 0) {
                *found = true;
                return i;
            }
            i = (i + 1) & mask;
        }
        *found = false;
        return i;
    }
    bool get(const char* p, size_t n, uint32_t* id) const {
        bool f = false;
        const size_t i = probe(p, n, &f);
        if (f) *id = table[i].id;
        return f;
    }
    void put(const char* p, size_t n, uint32_t id) {
        if ((count + 1) * 2 > table.size()) {  // keep the load factor at most 1/2
            std::vector<Slot> old;
            old.swap(table);
            table.assign(old.size() * 2, Slot{});
            for (const Slot& s : old)
                if (s.used) {
                    bool f = false;
                    table[probe(arena.data() + s.off, s.len, &f)] = s;
                }
        }
        bool f = false;
        const size_t i = probe(p, n, &f);
        if (f) {
            table[i].id = id;  // StringHashMap.put: the later line wins
            return;
        }
        Slot s;
        s.off = static_cast<uint32_t>(arena.size());
        s.len = static_cast<uint32_t>(n);
        s.id = id;
        s.used = true;
        arena.append(p, n);
        table[i] = s;
        ++count;
    }
    uint32_t lookup_or_unk(const char* p, size_t n) const {
        uint32_t id = unk_id;
        return get(p, n, &id) ? id : unk_id;
    }

    static bool is_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
    static bool is_punct(char c) {
        switch (c) {
            case '!': case '"': case '#': case '$': case '%': case '&': case '\'': case '(': case ')':
            case '*': case '+': case ',': case '-': case '.': case '/': case ':': case ';': case '<':
            case '=': case '>': case '?': case '@': case '[': case '\\': case ']': case '^': case '_':
            case '`': case '{': case '|': case '}': case '~':
                return true;
            default:
                return false;
        }
    }

    // WordPiece of one word, written from output position `start`; another piece is taken only
    // while the position is below `cap_minus_one` (the bounded form of encode).  On an unmatched
    // remainder the pieces written since `start` are replaced by one [UNK].  Returns the new
    // output length.
    template <class Out>
    size_t word_pieces(const char* w, size_t n, Out& out, size_t start, size_t cap_minus_one) const {
        if (n > max_word_chars) {
            out.set(start, unk_id);
            return start + 1;
        }
        char b[2 + 256];  // "##" + the lowercased word; b[cs..cs+2) is rewritten to "##" as cs advances
        b[0] = b[1] = '#';
        for (size_t k = 0; k < n; ++k) b[2 + k] = (w[k] >= 'A' && w[k] <= 'Z') ? static_cast<char>(w[k] + 32) : w[k];
        size_t pos = start, cs = 0;
        bool first = true;
        while (cs < n && pos < cap_minus_one) {
            bool found = false;
            if (!first) b[cs] = b[cs + 1] = '#';  // lower[cs-2..cs) are consumed: the "##" prefix goes there
            for (size_t ce = n; ce > cs; --ce) {
                uint32_t id;
                const bool hit = first ? get(b + 2, ce, &id) : get(b + cs, ce - cs + 2, &id);
                if (hit) {
                    out.set(pos++, id);
                    cs = ce;
                    first = false;
                    found = true;
                    break;
                }
            }
            if (!found) {
                out.truncate(start);
                out.set(start, unk_id);
                return start + 1;
            }
        }
        return pos;
    }

    struct Bounded {  // encode: a caller buffer of cap ids
        uint32_t* o;
        void set(size_t i, uint32_t v) { o[i] = v; }
        void truncate(size_t) {}
    };
    struct Growing {  // encodeRaw: an unbounded list
        std::vector<uint32_t>* v;
        void set(size_t i, uint32_t id) {
            if (i >= v->size()) v->resize(i + 1);
            (*v)[i] = id;
        }
        void truncate(size_t n) { v->resize(n); }
    };

    size_t encode(const char* t, size_t n, uint32_t* out, size_t cap) const {
        Bounded o{out};
        size_t pos = 0;
        out[pos++] = cls_id;
        size_t i = 0;
        while (i < n && pos < cap - 1) {
            while (i < n && is_ws(t[i])) ++i;
            if (i >= n) break;
            const size_t w0 = i;
            while (i < n && !is_ws(t[i]) && !is_punct(t[i])) ++i;
            if (i > w0) pos = word_pieces(t + w0, i - w0, o, pos, cap - 1);
            if (i < n && is_punct(t[i])) {
                if (pos < cap - 1) out[pos++] = lookup_or_unk(t + i, 1);
                ++i;
            }
        }
        out[pos++] = sep_id;
        return pos;
    }

    void encode_raw(const char* t, size_t n, std::vector<uint32_t>* v) const {
        Growing o{v};
        size_t i = 0;
        const size_t no_limit = static_cast<size_t>(-1);
        while (i < n) {
            while (i < n && is_ws(t[i])) ++i;
            if (i >= n) break;
            const size_t w0 = i;
            while (i < n && !is_ws(t[i]) && !is_punct(t[i])) ++i;
            if (i > w0) word_pieces(t + w0, i - w0, o, v->size(), no_limit);
            if (i < n && is_punct(t[i])) {
                v->push_back(lookup_or_unk(t + i, 1));
                ++i;
            }
        }
    }

    void load_bytes(const char* d, size_t n) {
        uint32_t line = 0;
        size_t a = 0;
        while (a <= n) {  // splitScalar('\n'): n + 1 segments for n newlines
            size_t b = a;
            while (b < n && d[b] != '\n') ++b;
            size_t len = b - a;
            if (len > 0) {
                if (d[a + len - 1] == '\r') --len;
                if (len > 0) put(d + a, len, line);
            }
            ++line;
            a = b + 1;
        }
    }
};

namespace {

int check_tok(tz_tokenizer_t t) {
    TZ_CHECK(t, TZ_EINVAL, "tokenizer: null handle");
    return TZ_OK;
}

}  // namespace

namespace tz {

int tokenize_raw(tz_tokenizer_t t, const char* text, int64_t len, std::vector<uint32_t>* ids) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(len >= 0 && (text || len == 0), TZ_EINVAL, "tokenizer: bad text buffer");
    ids->clear();
    t->encode_raw(text, static_cast<size_t>(len), ids);
    return TZ_OK;
}
uint32_t tokenizer_cls(tz_tokenizer_t t) { return t->cls_id; }
uint32_t tokenizer_sep(tz_tokenizer_t t) { return t->sep_id; }

}  // namespace tz

extern "C" {

int tz_tokenizer_create(tz_tokenizer_t* out) {
    TZ_CHECK(out, TZ_EINVAL, "tz_tokenizer_create: null out");
    *out = new tz_tokenizer_s();
    return TZ_OK;
}

int tz_tokenizer_free(tz_tokenizer_t t) {
    delete t;
    return TZ_OK;
}

int tz_tokenizer_set_special(tz_tokenizer_t t, uint32_t unk_id, uint32_t cls_id, uint32_t sep_id) {
    if (int rc = check_tok(t)) return rc;
    t->unk_id = unk_id;
    t->cls_id = cls_id;
    t->sep_id = sep_id;
    return TZ_OK;
}

int tz_tokenizer_put(tz_tokenizer_t t, const char* token, int64_t len, uint32_t id) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(token && len > 0 && len < (int64_t(1) << 30), TZ_EINVAL, "tz_tokenizer_put: empty token");
    t->put(token, static_cast<size_t>(len), id);
    return TZ_OK;
}

int tz_tokenizer_load_vocab_bytes(tz_tokenizer_t t, const char* data, int64_t len) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(len >= 0 && (data || len == 0), TZ_EINVAL, "tz_tokenizer_load_vocab_bytes: bad buffer");
    t->load_bytes(data, static_cast<size_t>(len));
    return TZ_OK;
}

int tz_tokenizer_load_vocab(tz_tokenizer_t t, const char* path) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(path, TZ_EINVAL, "tz_tokenizer_load_vocab: null path");
    std::ifstream f(path, std::ios::binary);
    TZ_CHECK(f.good(), TZ_EINVAL, "tz_tokenizer_load_vocab: cannot open %s", path);
    std::string data((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    t->load_bytes(data.data(), data.size());
    return TZ_OK;
}

int tz_tokenizer_vocab_size(tz_tokenizer_t t, int64_t* n) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(n, TZ_EINVAL, "tz_tokenizer_vocab_size: null out");
    *n = static_cast<int64_t>(t->count);
    return TZ_OK;
}

int tz_tokenizer_encode(tz_tokenizer_t t, const char* text, int64_t len, uint32_t* out, int64_t cap, int64_t* n) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(out && n && cap >= 2 && len >= 0 && (text || len == 0), TZ_EINVAL,
             "tz_tokenizer_encode: needs room for [CLS] and [SEP] (cap %lld)", static_cast<long long>(cap));
    *n = static_cast<int64_t>(t->encode(text, static_cast<size_t>(len), out, static_cast<size_t>(cap)));
    return TZ_OK;
}

int tz_tokenizer_encode_raw(tz_tokenizer_t t, const char* text, int64_t len, uint32_t* out, int64_t cap, int64_t* n) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(n && len >= 0 && (text || len == 0) && cap >= 0, TZ_EINVAL, "tz_tokenizer_encode_raw: bad arguments");
    std::vector<uint32_t> v;
    t->encode_raw(text, static_cast<size_t>(len), &v);
    *n = static_cast<int64_t>(v.size());
    if (!out) return TZ_OK;  // size query
    TZ_CHECK(static_cast<int64_t>(v.size()) <= cap, TZ_EINVAL, "tz_tokenizer_encode_raw: %zu ids, buffer holds %lld",
             v.size(), static_cast<long long>(cap));
    if (!v.empty()) memcpy(out, v.data(), v.size() * sizeof(uint32_t));
    return TZ_OK;
}

int tz_tokenizer_encode_batch(tz_tokenizer_t t, const char* const* texts, const int64_t* lens, int n_texts, int max_len,
                              uint32_t* ids_packed, int32_t* cu_seqlens, int64_t cap_tokens) {
    if (int rc = check_tok(t)) return rc;
    TZ_CHECK(n_texts >= 0 && max_len >= 2 && cu_seqlens && (n_texts == 0 || (texts && lens && ids_packed)), TZ_EINVAL,
             "tz_tokenizer_encode_batch: bad arguments");
    for (int i = 0; i < n_texts; ++i)
        TZ_CHECK(lens[i] >= 0 && (texts[i] || lens[i] == 0), TZ_EINVAL, "tz_tokenizer_encode_batch: text %d", i);
    std::vector<uint32_t> lengths(static_cast<size_t>(n_texts));
    std::vector<uint32_t> scratch(static_cast<size_t>(n_texts) * static_cast<size_t>(max_len));
    auto work = [&](int a, int b) {
        for (int i = a; i < b; ++i)
            lengths[i] = static_cast<uint32_t>(t->encode(texts[i], static_cast<size_t>(lens[i]),
                                                         scratch.data() + static_cast<size_t>(i) * max_len,
                                                         static_cast<size_t>(max_len)));
    };
    const unsigned hw = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
    const int nth = n_texts >= 64 ? static_cast<int>(std::min<unsigned>(hw, static_cast<unsigned>(n_texts / 32))) : 1;
    if (nth <= 1) {
        work(0, n_texts);
    } else {
        std::vector<std::thread> pool;
        const int per = (n_texts + nth - 1) / nth;
        for (int k = 0; k < nth; ++k) {
            const int a = k * per, b = std::min(n_texts, a + per);
            if (a < b) pool.emplace_back(work, a, b);
        }
        for (auto& th : pool) th.join();
    }
    int64_t total = 0;
    cu_seqlens[0] = 0;
    for (int i = 0; i < n_texts; ++i) {
        total += lengths[i];
        TZ_CHECK(total <= cap_tokens && total < (int64_t(1) << 31), TZ_EINVAL,
                 "tz_tokenizer_encode_batch: %lld ids exceed the buffer of %lld", static_cast<long long>(total),
                 static_cast<long long>(cap_tokens));
        cu_seqlens[i + 1] = static_cast<int32_t>(total);
    }
    for (int i = 0; i < n_texts; ++i)
        memcpy(ids_packed + cu_seqlens[i], scratch.data() + static_cast<size_t>(i) * max_len, lengths[i] * sizeof(uint32_t));
    return TZ_OK;
}

}  // extern "C"
