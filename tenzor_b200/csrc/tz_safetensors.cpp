// tz_safetensors.cpp -- safetensors checkpoint reader for tz_arctic_load_safetensors.
//
// Format (safetensors.zig:172-273): u64 little-endian header length, a JSON header mapping tensor
// names to {"dtype", "shape", "data_offsets": [begin, end]} (plus an optional "__metadata__"), then
// the raw data.  Weight names follow ModelWeights.fromSafeTensors (arctic.zig:130-156, 302-339):
// an optional "bert." prefix, LayerNorm ".weight"|".gamma" / ".bias"|".beta", and int8 matrices
// stored as I8 with a "<name>.scale" F16 vector (quantize_arctic_xs.zig:139).
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <string>
#include <vector>

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
    std::string prefix;

    const TensorInfo* get(const std::string& n) const {
        auto it = t.find(n);
        return it == t.end() ? nullptr : &it->second;
    }
    const void* data(const TensorInfo& ti) const { return bytes.data() + data0 + ti.begin; }

    int f32(const std::string& name, int64_t numel, const float** out) const {
        const TensorInfo* ti = get(prefix + name);
        if (!ti) return tz::fail(TZ_EMISSING, "Missing weight: %s%s", prefix.c_str(), name.c_str());
        if (ti->dtype != "F32") return tz::fail(TZ_EINVAL, "Weight %s%s has wrong dtype, expected F32", prefix.c_str(), name.c_str());
        if (ti->end - ti->begin != numel * 4) return tz::fail(TZ_EINVAL, "Weight %s%s has %lld bytes, expected %lld", prefix.c_str(), name.c_str(), static_cast<long long>(ti->end - ti->begin), static_cast<long long>(numel * 4));
        *out = static_cast<const float*>(data(*ti));
        return TZ_OK;
    }
    int f32_alt(const std::string& a, const std::string& b, int64_t numel, const float** out) const {
        if (get(prefix + a)) return f32(a, numel, out);
        return f32(b, numel, out);
    }
    // getMatWeightAlloc (arctic.zig:258-287): F32, or I8 + F16 ".scale".
    int mat(const std::string& name, int64_t rows, int64_t cols, tz_mat_weight* w) const {
        *w = tz_mat_weight{nullptr, nullptr, nullptr};
        const TensorInfo* ti = get(prefix + name);
        if (!ti) return tz::fail(TZ_EMISSING, "Missing weight: %s%s", prefix.c_str(), name.c_str());
        if (ti->dtype == "F32") return f32(name, rows * cols, &w->f32);
        if (ti->dtype == "I8") {
            if (ti->end - ti->begin != rows * cols) return tz::fail(TZ_EINVAL, "Weight %s%s has the wrong size", prefix.c_str(), name.c_str());
            const TensorInfo* si = get(prefix + name + ".scale");
            if (!si) return tz::fail(TZ_EMISSING, "Missing weight: %s%s.scale", prefix.c_str(), name.c_str());
            if (si->dtype != "F16") return tz::fail(TZ_EINVAL, "Weight %s%s.scale has wrong dtype, expected F16", prefix.c_str(), name.c_str());
            if (si->end - si->begin != rows * 2) return tz::fail(TZ_EINVAL, "Weight %s%s.scale has the wrong size", prefix.c_str(), name.c_str());
            w->q8 = static_cast<const int8_t*>(data(*ti));
            w->scale_f16 = static_cast<const uint16_t*>(data(*si));
            return TZ_OK;
        }
        return tz::fail(TZ_EUNSUPPORTED, "Weight %s%s has unsupported dtype %s", prefix.c_str(), name.c_str(), ti->dtype.c_str());
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
    ck.prefix = ck.get("bert.embeddings.word_embeddings.weight") ? "bert." : "";
    return TZ_OK;
}

}  // namespace

extern "C" int tz_arctic_load_safetensors(tz_ctx_t ctx, const char* path, int mode, tz_model_t* out) {
    TZ_CHECK(ctx && path && out, TZ_EINVAL, "tz_arctic_load_safetensors: null argument");
    Checkpoint ck;
    int rc = read_checkpoint(path, ck);
    if (rc) return rc;
    tz_arctic_weights w;
    memset(&w, 0, sizeof w);
    const int64_t H = 384, F = 1536;
    if ((rc = ck.mat("embeddings.word_embeddings.weight", 30522, H, &w.word_embeddings))) return rc;
    if ((rc = ck.mat("embeddings.position_embeddings.weight", 512, H, &w.position_embeddings))) return rc;
    if ((rc = ck.mat("embeddings.token_type_embeddings.weight", 2, H, &w.token_type_embeddings))) return rc;
    if ((rc = ck.f32_alt("embeddings.LayerNorm.weight", "embeddings.LayerNorm.gamma", H, &w.ln_gamma))) return rc;
    if ((rc = ck.f32_alt("embeddings.LayerNorm.bias", "embeddings.LayerNorm.beta", H, &w.ln_beta))) return rc;
    for (int l = 0; l < 6; ++l) {
        const std::string p = "encoder.layer." + std::to_string(l) + ".";
        tz_arctic_layer& L = w.layers[l];
        if ((rc = ck.mat(p + "attention.self.query.weight", H, H, &L.query))) return rc;
        if ((rc = ck.mat(p + "attention.self.key.weight", H, H, &L.key))) return rc;
        if ((rc = ck.mat(p + "attention.self.value.weight", H, H, &L.value))) return rc;
        if ((rc = ck.mat(p + "attention.output.dense.weight", H, H, &L.attn_output))) return rc;
        if ((rc = ck.mat(p + "intermediate.dense.weight", F, H, &L.intermediate))) return rc;
        if ((rc = ck.mat(p + "output.dense.weight", H, F, &L.output))) return rc;
        if ((rc = ck.f32(p + "attention.self.query.bias", H, &L.query_bias))) return rc;
        if ((rc = ck.f32(p + "attention.self.key.bias", H, &L.key_bias))) return rc;
        if ((rc = ck.f32(p + "attention.self.value.bias", H, &L.value_bias))) return rc;
        if ((rc = ck.f32(p + "attention.output.dense.bias", H, &L.attn_output_bias))) return rc;
        if ((rc = ck.f32(p + "intermediate.dense.bias", F, &L.intermediate_bias))) return rc;
        if ((rc = ck.f32(p + "output.dense.bias", H, &L.output_bias))) return rc;
        if ((rc = ck.f32_alt(p + "attention.output.LayerNorm.weight", p + "attention.output.LayerNorm.gamma", H, &L.attn_ln_gamma))) return rc;
        if ((rc = ck.f32_alt(p + "attention.output.LayerNorm.bias", p + "attention.output.LayerNorm.beta", H, &L.attn_ln_beta))) return rc;
        if ((rc = ck.f32_alt(p + "output.LayerNorm.weight", p + "output.LayerNorm.gamma", H, &L.output_ln_gamma))) return rc;
        if ((rc = ck.f32_alt(p + "output.LayerNorm.bias", p + "output.LayerNorm.beta", H, &L.output_ln_beta))) return rc;
    }
    return tz_arctic_load(ctx, &w, mode, out);
}
