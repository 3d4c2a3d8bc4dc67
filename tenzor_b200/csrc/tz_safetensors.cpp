// tz_safetensors.cpp -- safetensors checkpoint reader for tz_arctic_load_safetensors.
//
// Format (safetensors.zig:172-273): u64 little-endian header length, a JSON header mapping tensor
// names to {"dtype", "shape", "data_offsets": [begin, end]} (plus an optional "__metadata__"), then
// the raw data.  Weight names are resolved by tz_ckpt.h (ModelWeights.fromSafeTensors).
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <string>
#include <vector>

#include "tz_ckpt.h"
#include "tz_internal.h"

namespace {

struct TensorInfo {
    std::string dtype;
    std::vector<int64_t> shape;
    int64_t begin = 0, end = 0;
};

struct Parser {
    const char* p;
    const char* e;
    bool ok = true;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool eat(char c) {
        ws();
        if (p < e && *p == c) {
            ++p;
            return true;
        }
        return false;
    }
    std::string str() {
        ws();
        std::string out;
        if (p >= e || *p != '"') {
            ok = false;
            return out;
        }
        ++p;
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) {
                ++p;
                out.push_back(*p == 'n' ? '\n' : *p);
            } else {
                out.push_back(*p);
            }
            ++p;
        }
        if (p < e) ++p;
        else ok = false;
        return out;
    }
    int64_t num() {
        ws();
        bool neg = false;
        if (p < e && *p == '-') {
            neg = true;
            ++p;
        }
        int64_t v = 0;
        if (p >= e || *p < '0' || *p > '9') ok = false;
        while (p < e && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
        return neg ? -v : v;
    }
    void skip_value() {
        ws();
        if (p >= e) {
            ok = false;
            return;
        }
        if (*p == '"') {
            str();
        } else if (*p == '{') {
            ++p;
            if (eat('}')) return;
            do {
                str();
                if (!eat(':')) { ok = false; return; }
                skip_value();
            } while (ok && eat(','));
            if (!eat('}')) ok = false;
        } else if (*p == '[') {
            ++p;
            if (eat(']')) return;
            do skip_value();
            while (ok && eat(','));
            if (!eat(']')) ok = false;
        } else {
            while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        }
    }
};

bool parse_header(const char* s, size_t n, std::map<std::string, TensorInfo>& out) {
    Parser ps{s, s + n};
    if (!ps.eat('{')) return false;
    if (ps.eat('}')) return true;
    do {
        std::string name = ps.str();
        if (!ps.eat(':')) return false;
        if (name == "__metadata__") {
            ps.skip_value();
            continue;
        }
        TensorInfo ti;
        if (!ps.eat('{')) return false;
        if (!ps.eat('}')) {
            do {
                std::string key = ps.str();
                if (!ps.eat(':')) return false;
                if (key == "dtype") {
                    ti.dtype = ps.str();
                } else if (key == "shape") {
                    if (!ps.eat('[')) return false;
                    if (!ps.eat(']')) {
                        do ti.shape.push_back(ps.num());
                        while (ps.ok && ps.eat(','));
                        if (!ps.eat(']')) return false;
                    }
                } else if (key == "data_offsets") {
                    if (!ps.eat('[')) return false;
                    ti.begin = ps.num();
                    if (!ps.eat(',')) return false;
                    ti.end = ps.num();
                    if (!ps.eat(']')) return false;
                } else {
                    ps.skip_value();
                }
            } while (ps.ok && ps.eat(','));
            if (!ps.eat('}')) return false;
        }
        out[name] = ti;
    } while (ps.ok && ps.eat(','));
    return ps.ok && ps.eat('}');
}

int64_t dtype_size(const std::string& d) {
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F16" || d == "BF16" || d == "I16") return 2;
    if (d == "I8" || d == "U8" || d == "BOOL") return 1;
    if (d == "F64" || d == "I64") return 8;
    return 0;
}

struct Checkpoint {
    std::vector<char> bytes;
    size_t data0 = 0;
    std::map<std::string, TensorInfo> t;

    bool find(const std::string& n, tz::CkptView* v) const {
        auto it = t.find(n);
        if (it == t.end()) return false;
        const TensorInfo& ti = it->second;
        v->dtype = ti.dtype == "F32" ? tz::CK_F32 : ti.dtype == "F16" ? tz::CK_F16 : ti.dtype == "I8" ? tz::CK_I8 : tz::CK_OTHER;
        v->bytes = ti.end - ti.begin;
        v->data = bytes.data() + data0 + ti.begin;
        return true;
    }
};

int read_checkpoint(const char* path, Checkpoint& ck) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) return tz::fail(TZ_EINVAL, "cannot open %s", path);
    const std::streamsize n = f.tellg();
    f.seekg(0);
    if (n < 8) return tz::fail(TZ_EINVAL, "%s: file too small for a safetensors header", path);
    ck.bytes.resize(static_cast<size_t>(n));
    if (!f.read(ck.bytes.data(), n)) return tz::fail(TZ_EINVAL, "%s: read failed", path);
    uint64_t hl = 0;
    for (int i = 7; i >= 0; --i) hl = (hl << 8) | static_cast<unsigned char>(ck.bytes[i]);
    if (hl > static_cast<uint64_t>(n) - 8) return tz::fail(TZ_EINVAL, "%s: header length %llu exceeds the file", path, static_cast<unsigned long long>(hl));
    if (!parse_header(ck.bytes.data() + 8, hl, ck.t)) return tz::fail(TZ_EINVAL, "%s: malformed safetensors header", path);
    ck.data0 = 8 + hl;
    const uint64_t data_bytes = static_cast<uint64_t>(n) - ck.data0;
    for (auto& kv : ck.t) {
        const TensorInfo& ti = kv.second;
        int64_t numel = 1;
        for (int64_t d : ti.shape) numel *= d;
        const int64_t es = dtype_size(ti.dtype);
        if (ti.begin < 0 || ti.end < ti.begin || static_cast<uint64_t>(ti.end) > data_bytes || (es && numel * es != ti.end - ti.begin))
            return tz::fail(TZ_EINVAL, "%s: tensor %s has inconsistent offsets", path, kv.first.c_str());
    }
    return TZ_OK;
}

}  // namespace

extern "C" int tz_arctic_load_safetensors(tz_ctx_t ctx, const char* path, int mode, tz_model_t* out) {
    TZ_CHECK(ctx && path && out, TZ_EINVAL, "tz_arctic_load_safetensors: null argument");
    Checkpoint ck;
    int rc = read_checkpoint(path, ck);
    if (rc) return rc;
    tz_arctic_weights w;
    if ((rc = tz::resolve_arctic(ck, &w))) return rc;
    return tz_arctic_load(ctx, &w, mode, out);
}
