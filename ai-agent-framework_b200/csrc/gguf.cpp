#include "gguf.h"

#include <cstdio>
#include <cstring>

#include "../../include/b2decode.h"

namespace b2 {

namespace {
constexpr uint32_t kMagic = 0x46554747;  // "GGUF"
enum : uint32_t {
    VU8 = 0, VI8, VU16, VI16, VU32, VI32, VF32, VBOOL, VSTR, VARR, VU64, VI64, VF64
};

struct Rd {
    FILE* f;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (ok && fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    bool str(std::string* s, bool keep) {
        uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) { ok = false; return false; }  // gguf.go:328-330
        if (keep) {
            s->resize(n);
            if (n && fread(&(*s)[0], 1, n, f) != n) ok = false;
        } else if (n && fseek(f, (long)n, SEEK_CUR) != 0) {
            ok = false;
        }
        return ok;
    }
};

bool read_value(Rd& r, uint32_t t, GgufValue* v, bool keep) {  // gguf.go:346-414
    v->type = t;
    switch (t) {
        case VU8: v->u = r.get<uint8_t>(); break;
        case VI8: v->i = r.get<int8_t>(); break;
        case VU16: v->u = r.get<uint16_t>(); break;
        case VI16: v->i = r.get<int16_t>(); break;
        case VU32: v->u = r.get<uint32_t>(); break;
        case VI32: v->i = r.get<int32_t>(); break;
        case VF32: v->f = r.get<float>(); break;
        case VBOOL: v->u = r.get<uint8_t>() != 0; break;
        case VSTR: r.str(&v->s, keep); break;
        case VU64: v->u = r.get<uint64_t>(); break;
        case VI64: v->i = r.get<int64_t>(); break;
        case VF64: v->f = r.get<double>(); break;
        case VARR: {
            uint32_t et = r.get<uint32_t>();
            uint64_t n = r.get<uint64_t>();
            if (!r.ok) return false;
            v->is_array = true;
            v->arr_len = n;
            v->type = et;
            GgufValue tmp;
            for (uint64_t k = 0; k < n && r.ok; k++) {
                if (!read_value(r, et, &tmp, et == VSTR && n <= 64)) return false;
                if (et == VSTR && n <= 64) v->strs.push_back(tmp.s);
            }
            break;
        }
        default: return false;
    }
    return r.ok;
}
}  // namespace

uint64_t ggml_type_size(uint32_t t) {
    switch (t) {
        case GGML_F32: return 4;
        case GGML_F16: return 2;
        case GGML_Q4_0: return 18;
        case 3: return 20;
        case 6: return 22;
        case 7: return 24;
        case GGML_Q8_0: return 34;
        case 9: return 36;
        case 10: return 84;
        case 11: return 110;
        case 12: return 144;
        case 13: return 176;
        case 14: return 210;
        case 15: return 292;
        case GGML_BF16: return 2;
        default: return 4;
    }
}

uint64_t ggml_block_size(uint32_t t) {
    switch (t) {
        case GGML_F32: case GGML_F16: case GGML_BF16: return 1;
        case GGML_Q4_0: case 3: case 6: case 7: case GGML_Q8_0: case 9: return 32;
        case 10: case 11: case 12: case 13: case 14: case 15: return 256;
        default: return 1;
    }
}

uint64_t GgufTensor::elements() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
}

uint64_t GgufTensor::bytes() const { return elements() * ggml_type_size(type) / ggml_block_size(type); }

const GgufTensor* GgufFile::find(const std::string& name) const {
    for (auto& t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}

bool GgufFile::get_str(const std::string& k, std::string* out) const {
    auto it = meta.find(k);
    if (it == meta.end() || it->second.is_array || it->second.type != VSTR) return false;
    *out = it->second.s;
    return true;
}

bool GgufFile::get_u32(const std::string& k, uint32_t* out) const {
    auto it = meta.find(k);
    if (it == meta.end() || it->second.is_array) return false;
    const GgufValue& v = it->second;
    switch (v.type) {
        case VU32: case VU64: *out = (uint32_t)v.u; return true;
        case VI32: case VI64: *out = (uint32_t)v.i; return true;
        default: return false;
    }
}

bool GgufFile::get_f32(const std::string& k, float* out) const {
    auto it = meta.find(k);
    if (it == meta.end() || it->second.is_array) return false;
    if (it->second.type == VF32 || it->second.type == VF64) {
        *out = (float)it->second.f;
        return true;
    }
    return false;
}

int64_t GgufFile::array_len(const std::string& k) const {
    auto it = meta.find(k);
    if (it == meta.end() || !it->second.is_array) return -1;
    return (int64_t)it->second.arr_len;
}

int gguf_parse(const char* path, GgufFile* g, std::string* err) {
    FILE* f = fopen(path, "rb");
    if (!f) { *err = std::string("open gguf file: ") + path; return B2_ERR_IO; }
    fseek(f, 0, SEEK_END);
    g->file_size = (uint64_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    g->path = path;
    Rd r{f};
    auto fail = [&](const std::string& m) { *err = m; fclose(f); return B2_ERR_FORMAT; };
    uint32_t magic = r.get<uint32_t>();
    if (!r.ok) return fail("read magic: file too short");
    if (magic != kMagic) {
        char b[96];
        snprintf(b, sizeof b, "invalid magic: got 0x%08X, want 0x%08X (GGUF)", magic, kMagic);
        return fail(b);
    }
    g->version = r.get<uint32_t>();
    if (!r.ok || g->version < 2 || g->version > 3)
        return fail("unsupported GGUF version: " + std::to_string(g->version) + " (supported: 2, 3)");
    uint64_t nt = r.get<uint64_t>();
    uint64_t nkv = r.get<uint64_t>();
    if (!r.ok) return fail("read header counts");
    if (nt > (1u << 20) || nkv > (1u << 20)) return fail("implausible tensor/metadata counts");
    for (uint64_t i = 0; i < nkv; i++) {
        std::string key;
        if (!r.str(&key, true)) return fail("read metadata key " + std::to_string(i));
        uint32_t t = r.get<uint32_t>();
        GgufValue v;
        if (!r.ok || !read_value(r, t, &v, true)) return fail("read metadata value for key \"" + key + "\"");
        g->meta[key] = std::move(v);
    }
    g->tensors.resize(nt);
    for (uint64_t i = 0; i < nt; i++) {
        GgufTensor& t = g->tensors[i];
        if (!r.str(&t.name, true)) return fail("read tensor name " + std::to_string(i));
        uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd == 0 || nd > 4) return fail("bad tensor ndims for " + t.name);
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; d++) t.dims[d] = r.get<uint64_t>();
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        if (!r.ok) return fail("read tensor info " + t.name);
    }
    uint64_t pos = (uint64_t)ftell(f);
    fclose(f);
    uint64_t align = 32;
    uint32_t a;
    if (g->get_u32("general.alignment", &a) && a != 0 && (a & (a - 1)) == 0) align = a;
    g->data_offset = (pos + align - 1) / align * align;
    for (auto& t : g->tensors) {
        uint64_t end = g->data_offset + t.offset + t.bytes();
        if (end > g->file_size) {
            *err = "tensor " + t.name + " extends past the end of the file (truncated GGUF)";
            return B2_ERR_FORMAT;
        }
    }
    return B2_OK;
}

}  // namespace b2
