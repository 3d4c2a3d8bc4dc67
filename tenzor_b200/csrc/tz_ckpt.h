// tz_ckpt.h -- name resolution of checkpoint files into the loaders' host weight structs, shared by
// the safetensors reader (tz_safetensors.cpp) and the .tenzor reader (tz_tenzor_file.cpp).
//
// A source is any type with `bool find(const std::string& name, tz::CkptView* v) const`.  Arctic
// names follow ModelWeights.fromSafeTensors (arctic.zig:130-156, 302-339): an optional "bert."
// prefix, LayerNorm ".weight"|".gamma" / ".bias"|".beta", and int8 matrices stored as I8 with a
// "<name>.scale" F16 vector (getMatWeightAlloc, arctic.zig:258-287; quantize_arctic_xs.zig:139).
#pragma once

#include <cstdint>
#include <string>

#include "tz_internal.h"

namespace tz {

enum CkptDtype { CK_F32 = 0, CK_F16 = 1, CK_I8 = 2, CK_OTHER = 3 };

struct CkptView {
    int dtype = CK_OTHER;
    int64_t bytes = 0;
    const void* data = nullptr;
};

template <class Src>
struct CkptResolver {
    const Src& src;
    std::string prefix;

    explicit CkptResolver(const Src& s, const std::string& pre = "") : src(s), prefix(pre) {}

    bool has(const std::string& n) const {
        CkptView v;
        return src.find(prefix + n, &v);
    }
    int f32(const std::string& name, int64_t numel, const float** out) const {
        CkptView v;
        if (!src.find(prefix + name, &v)) return fail(TZ_EMISSING, "Missing weight: %s%s", prefix.c_str(), name.c_str());
        if (v.dtype != CK_F32) return fail(TZ_EINVAL, "Weight %s%s has wrong dtype, expected F32", prefix.c_str(), name.c_str());
        if (v.bytes != numel * 4)
            return fail(TZ_EINVAL, "Weight %s%s has %lld bytes, expected %lld", prefix.c_str(), name.c_str(),
                        static_cast<long long>(v.bytes), static_cast<long long>(numel * 4));
        *out = static_cast<const float*>(v.data);
        return TZ_OK;
    }
    int f32_alt(const std::string& a, const std::string& b, int64_t numel, const float** out) const {
        return has(a) ? f32(a, numel, out) : f32(b, numel, out);
    }
    // getMatWeightAlloc (arctic.zig:258-287): F32, or I8 + F16 ".scale".
    int mat(const std::string& name, int64_t rows, int64_t cols, tz_mat_weight* w) const {
        *w = tz_mat_weight{nullptr, nullptr, nullptr};
        CkptView v;
        if (!src.find(prefix + name, &v)) return fail(TZ_EMISSING, "Missing weight: %s%s", prefix.c_str(), name.c_str());
        if (v.dtype == CK_F32) return f32(name, rows * cols, &w->f32);
        if (v.dtype == CK_I8) {
            if (v.bytes != rows * cols) return fail(TZ_EINVAL, "Weight %s%s has the wrong size", prefix.c_str(), name.c_str());
            CkptView s;
            if (!src.find(prefix + name + ".scale", &s))
                return fail(TZ_EMISSING, "Missing weight: %s%s.scale", prefix.c_str(), name.c_str());
            if (s.dtype != CK_F16) return fail(TZ_EINVAL, "Weight %s%s.scale has wrong dtype, expected F16", prefix.c_str(), name.c_str());
            if (s.bytes != rows * 2) return fail(TZ_EINVAL, "Weight %s%s.scale has the wrong size", prefix.c_str(), name.c_str());
            w->q8 = static_cast<const int8_t*>(v.data);
            w->scale_f16 = static_cast<const uint16_t*>(s.data);
            return TZ_OK;
        }
        return fail(TZ_EUNSUPPORTED, "Weight %s%s has an unsupported dtype", prefix.c_str(), name.c_str());
    }
};

// Fills `w` with pointers into the source's memory (valid while the source lives).
template <class Src>
int resolve_arctic(const Src& src, tz_arctic_weights* w) {
    CkptView probe;
    const CkptResolver<Src> ck(src, src.find("bert.embeddings.word_embeddings.weight", &probe) ? "bert." : "");
    *w = tz_arctic_weights{};
    const int64_t H = 384, F = 1536;
    int rc;
    if ((rc = ck.mat("embeddings.word_embeddings.weight", 30522, H, &w->word_embeddings))) return rc;
    if ((rc = ck.mat("embeddings.position_embeddings.weight", 512, H, &w->position_embeddings))) return rc;
    if ((rc = ck.mat("embeddings.token_type_embeddings.weight", 2, H, &w->token_type_embeddings))) return rc;
    if ((rc = ck.f32_alt("embeddings.LayerNorm.weight", "embeddings.LayerNorm.gamma", H, &w->ln_gamma))) return rc;
    if ((rc = ck.f32_alt("embeddings.LayerNorm.bias", "embeddings.LayerNorm.beta", H, &w->ln_beta))) return rc;
    for (int l = 0; l < 6; ++l) {
        const std::string p = "encoder.layer." + std::to_string(l) + ".";
        tz_arctic_layer& L = w->layers[l];
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
    return TZ_OK;
}

}  // namespace tz
