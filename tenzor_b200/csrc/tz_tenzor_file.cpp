// tz_tenzor_file.cpp -- the reference's .tenzor checkpoint format, memory-mapped, and the model
// loaders that read it.
//
// Format (src/io/tenzor_format.zig:1-13, 66-104): a 64-byte header {magic "TENZOR\0\0", u32 version
// = 1, u32 flags, u32 tensor_count, u32 pad, u64 index_offset, u64 data_offset, u32 metadata_size,
// 20 reserved bytes}; the metadata JSON right after it (padded to 8 bytes); tensor_count 48-byte
// index entries {u64 FNV-1a hash of the name, u8 dtype, u8 ndim, 2 pad, u32 shape[5], u64 offset
// into the data section, u64 size}; the data section at a 4 KiB-aligned offset.  Names are stored
// only as hashes, so a tensor is found by hashing the name asked for (getTensor, 224-226).  Files
// are mapped read-only (TenzorFile.open, 140-199) and tensor data is used in place.
//
// Loaders: tz_lenet_load_tenzor reads the names LeNet training checkpoints carry (main.zig:502-511,
// read back by runEval 638-667: conv1_weight, conv1_bias, ..., fc3_bias, all f32);
// tz_arctic_load_tenzor reads a file converted from safetensors (convertFromSafetensors,
// tenzor_format.zig:441-485, which keeps the safetensors names and dtypes), resolved as the
// safetensors loader resolves them (tz_ckpt.h).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "tz_ckpt.h"
#include "tz_internal.h"

struct tz_tenzor_s {
    const uint8_t* map = nullptr;
    size_t size = 0;
    uint32_t count = 0;
    uint64_t index_offset = 0, data_offset = 0;
    uint32_t metadata_size = 0;
    std::vector<tz_tenzor_entry> entries;
    std::unordered_map<uint64_t, size_t> by_hash;  // first entry of each hash (the linear scan's answer)

    bool find(const std::string& name, tz::CkptView* v) const {
        auto it = by_hash.find(tz_tenzor_hash_name(name.data(), name.size()));
        if (it == by_hash.end()) return false;
        const tz_tenzor_entry& e = entries[it->second];
        v->dtype = e.dtype == TZ_DT_F32 ? tz::CK_F32 : e.dtype == TZ_DT_F16 ? tz::CK_F16 : e.dtype == TZ_DT_I8 ? tz::CK_I8 : tz::CK_OTHER;
        v->bytes = static_cast<int64_t>(e.bytes);
        v->data = e.data;
        return true;
    }
};

namespace {

constexpr uint8_t kMagic[8] = {'T', 'E', 'N', 'Z', 'O', 'R', 0, 0};

uint64_t rd64(const uint8_t* p) {
    uint64_t v;
    std::memcpy(&v, p, 8);
    return v;
}
uint32_t rd32(const uint8_t* p) {
    uint32_t v;
    std::memcpy(&v, p, 4);
    return v;
}

int dtype_bytes(int d) {  // DType.byteSize (tenzor_format.zig:39-46)
    switch (d) {
        case TZ_DT_F16: case TZ_DT_BF16: case TZ_DT_I16: case TZ_DT_U16: return 2;
        case TZ_DT_F32: case TZ_DT_I32: case TZ_DT_U32: return 4;
        case TZ_DT_F64: case TZ_DT_I64: case TZ_DT_U64: return 8;
        case TZ_DT_I8: case TZ_DT_U8: return 1;
        default: return 0;
    }
}

void unmap(tz_tenzor_s* f) {
    if (f->map) munmap(const_cast<uint8_t*>(f->map), f->size);
    f->map = nullptr;
}

}  // namespace

extern "C" {

uint64_t tz_tenzor_hash_name(const char* name, size_t len) {  // hashName, tenzor_format.zig:107-114
    uint64_t h = 0xcbf29ce484222325ull;
    for (size_t i = 0; i < len; ++i) {
        h ^= static_cast<uint8_t>(name[i]);
        h *= 0x100000001b3ull;
    }
    return h;
}

int tz_tenzor_open(const char* path, tz_tenzor_t* out) {
    TZ_CHECK(path && out, TZ_EINVAL, "tz_tenzor_open: null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return tz::fail(TZ_EINVAL, "tz_tenzor_open: cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 64) {
        close(fd);
        return tz::fail(TZ_EINVAL, "%s: too small for a .tenzor header (InvalidFormat)", path);
    }
    const size_t size = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return tz::fail(TZ_EINVAL, "%s: mmap failed (MmapFailed)", path);
    tz_tenzor_s* f = new tz_tenzor_s;
    f->map = static_cast<const uint8_t*>(m);
    f->size = size;
    auto bad = [&](const char* why) {
        unmap(f);
        delete f;
        return tz::fail(TZ_EINVAL, "%s: %s", path, why);
    };
    const uint8_t* h = f->map;
    if (std::memcmp(h, kMagic, 8) != 0) return bad("bad magic (InvalidMagic)");
    if (rd32(h + 8) != 1) return bad("unsupported version (UnsupportedVersion)");
    f->count = rd32(h + 16);
    f->index_offset = rd64(h + 24);
    f->data_offset = rd64(h + 32);
    f->metadata_size = rd32(h + 40);
    if (64 + static_cast<uint64_t>(f->metadata_size) > size) return bad("metadata runs past the end of the file");
    if (f->index_offset > size || static_cast<uint64_t>(f->count) * 48 > size - f->index_offset)
        return bad("tensor index runs past the end of the file");
    if (f->data_offset > size) return bad("data section starts past the end of the file");
    const uint64_t data_bytes = size - f->data_offset;
    f->entries.resize(f->count);
    for (uint32_t i = 0; i < f->count; ++i) {
        const uint8_t* e = h + f->index_offset + 48ull * i;
        tz_tenzor_entry& t = f->entries[i];
        t.name_hash = rd64(e);
        t.dtype = e[8];
        t.ndim = e[9];
        uint64_t numel = 1;
        for (int d = 0; d < 5; ++d) {
            t.shape[d] = rd32(e + 12 + 4 * d);
            if (d < t.ndim) numel *= t.shape[d];
        }
        const uint64_t off = rd64(e + 32);
        t.bytes = rd64(e + 40);
        if (t.ndim > 5 || dtype_bytes(t.dtype) == 0) return bad("tensor entry with a bad dtype or rank");
        if (off > data_bytes || t.bytes > data_bytes - off) return bad("tensor data runs past the end of the file");
        if (numel * static_cast<uint64_t>(dtype_bytes(t.dtype)) != t.bytes) return bad("tensor size disagrees with its shape");
        t.data = h + f->data_offset + off;
        f->by_hash.emplace(t.name_hash, i);  // keeps the first entry of a repeated hash
    }
    *out = f;
    return TZ_OK;
}

int tz_tenzor_close(tz_tenzor_t f) {
    if (!f) return TZ_OK;
    unmap(f);
    delete f;
    return TZ_OK;
}

int64_t tz_tenzor_count(tz_tenzor_t f) { return f ? static_cast<int64_t>(f->count) : -1; }

int tz_tenzor_entry_at(tz_tenzor_t f, int64_t i, tz_tenzor_entry* out) {
    TZ_CHECK(f && out && i >= 0 && i < static_cast<int64_t>(f->count), TZ_EINVAL, "tz_tenzor_entry_at: bad arguments");
    *out = f->entries[static_cast<size_t>(i)];
    return TZ_OK;
}

int tz_tenzor_find(tz_tenzor_t f, const char* name, tz_tenzor_entry* out) {
    TZ_CHECK(f && name && out, TZ_EINVAL, "tz_tenzor_find: null argument");
    auto it = f->by_hash.find(tz_tenzor_hash_name(name, std::strlen(name)));
    if (it == f->by_hash.end()) return tz::fail(TZ_EMISSING, "tensor %s not in the file", name);
    *out = f->entries[it->second];
    return TZ_OK;
}

int tz_tenzor_metadata(tz_tenzor_t f, const char** json, uint64_t* len) {
    TZ_CHECK(f && json && len, TZ_EINVAL, "tz_tenzor_metadata: null argument");
    *json = reinterpret_cast<const char*>(f->map + 64);
    *len = f->metadata_size;
    return TZ_OK;
}

int tz_lenet_load_tenzor(tz_ctx_t ctx, const char* path, int variant, tz_lenet_t* out) {
    TZ_CHECK(ctx && path && out && (variant == TZ_LENET_REF || variant == TZ_LENET_PAD2), TZ_EINVAL,
             "tz_lenet_load_tenzor: bad arguments");
    *out = nullptr;
    tz_tenzor_t f = nullptr;
    int rc = tz_tenzor_open(path, &f);
    if (rc) return rc;
    const int feat = variant == TZ_LENET_PAD2 ? 400 : 256;
    const tz::CkptResolver<tz_tenzor_s> ck(*f);
    tz_lenet_weights w{};
    if (!(rc = ck.f32("conv1_weight", 6 * 25, &w.conv1_w)) && !(rc = ck.f32("conv1_bias", 6, &w.conv1_b)) &&
        !(rc = ck.f32("conv2_weight", 16 * 25 * 6, &w.conv2_w)) && !(rc = ck.f32("conv2_bias", 16, &w.conv2_b)) &&
        !(rc = ck.f32("fc1_weight", 120LL * feat, &w.fc1_w)) && !(rc = ck.f32("fc1_bias", 120, &w.fc1_b)) &&
        !(rc = ck.f32("fc2_weight", 84 * 120, &w.fc2_w)) && !(rc = ck.f32("fc2_bias", 84, &w.fc2_b)) &&
        !(rc = ck.f32("fc3_weight", 10 * 84, &w.fc3_w)) && !(rc = ck.f32("fc3_bias", 10, &w.fc3_b)))
        rc = tz_lenet_load(ctx, &w, variant, out);
    tz_tenzor_close(f);
    return rc;
}

int tz_arctic_load_tenzor(tz_ctx_t ctx, const char* path, int mode, tz_model_t* out) {
    TZ_CHECK(ctx && path && out, TZ_EINVAL, "tz_arctic_load_tenzor: null argument");
    tz_tenzor_t f = nullptr;
    int rc = tz_tenzor_open(path, &f);
    if (rc) return rc;
    tz_arctic_weights w;
    rc = tz::resolve_arctic(*f, &w);
    if (!rc) rc = tz_arctic_load(ctx, &w, mode, out);
    tz_tenzor_close(f);
    return rc;
}

}  // extern "C"
