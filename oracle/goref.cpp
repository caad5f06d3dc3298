// goref — CPU restatement of the Local-LLM-Pure-Go decode path.
//
// TEST INFRASTRUCTURE ONLY: the parity oracle and the timed CPU baseline.  The
// product never links or calls this file.
//
// Sources restated (paths relative to the reference project root):
//   Local-LLM-Pure-Go/internal/engine/native/gguf/gguf.go
//   Local-LLM-Pure-Go/internal/engine/native/transformer/transformer.go
//   Local-LLM-Pure-Go/internal/engine/native/bpe/bpe.go (BOS/EOS ids only)
// Float semantics: float32 arithmetic in source order, no contraction
// (-ffp-contract=off), float64 for the transcendentals exactly where Go widens.
// The C library's exp/cos/sin/pow/sqrt stand in for Go's math package; both
// are accurate to about one double ulp, so the float32 results they round to
// agree except when a double lands within an ulp of a float32 rounding
// boundary.

#include "goref.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;

void set_err(const std::string& s) { g_err = s; }

// ---------------------------------------------------------------------------
// gguf.go
// ---------------------------------------------------------------------------

constexpr uint32_t kMagic = 0x46554747;  // gguf.go:25
constexpr int64_t kAlignment = 32;       // gguf.go:26

enum : uint32_t {  // gguf.go:30-44
    TUint8 = 0, TInt8, TUint16, TInt16, TUint32, TInt32, TFloat32, TBool,
    TString, TArray, TUint64, TInt64, TFloat64
};

enum : uint32_t {  // gguf.go:47-72
    GF32 = 0, GF16 = 1, GQ4_0 = 2, GQ4_1 = 3, GQ5_0 = 6, GQ5_1 = 7, GQ8_0 = 8,
    GQ8_1 = 9, GQ2_K = 10, GQ3_K = 11, GQ4_K = 12, GQ5_K = 13, GQ6_K = 14,
    GQ8_K = 15, GBF16 = 30
};

struct Value {
    uint32_t type = 0;
    uint64_t u = 0;      // unsigned / bool payload
    int64_t i = 0;       // signed payload
    double f = 0;        // float payload
    std::string s;
    uint64_t arr_len = 0;  // arrays: only the length is kept (all extractConfig needs)
    bool is_array = false;
};

struct TensorInfo {  // gguf.go:85-91
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t elements() const {  // gguf.go:312-318
        uint64_t n = 1;
        for (auto d : dims) n *= d;
        return n;
    }
};

uint64_t type_size(uint32_t t) {  // gguf.go:422-457
    switch (t) {
        case GF32: return 4;
        case GF16: return 2;
        case GQ4_0: return 18;
        case GQ4_1: return 20;
        case GQ5_0: return 22;
        case GQ5_1: return 24;
        case GQ8_0: return 34;
        case GQ8_1: return 36;
        case GQ2_K: return 84;
        case GQ3_K: return 110;
        case GQ4_K: return 144;
        case GQ5_K: return 176;
        case GQ6_K: return 210;
        case GQ8_K: return 292;
        case GBF16: return 2;
        default: return 4;
    }
}

uint64_t block_size(uint32_t t) {  // gguf.go:460-473
    switch (t) {
        case GF32: case GF16: case GBF16: return 1;
        case GQ4_0: case GQ4_1: case GQ5_0: case GQ5_1: case GQ8_0: case GQ8_1: return 32;
        case GQ2_K: case GQ3_K: case GQ4_K: case GQ5_K: case GQ6_K: case GQ8_K: return 256;
        default: return 1;
    }
}

uint64_t data_size(const TensorInfo& t) {  // gguf.go:273-279
    return t.elements() * type_size(t.type) / block_size(t.type);
}

struct File {
    uint32_t version = 0;
    std::map<std::string, Value> meta;
    std::vector<TensorInfo> tensors;
    int64_t data_offset = 0;
    std::string path;

    const TensorInfo* find(const std::string& name) const {  // gguf.go:263-270
        for (auto& t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
    bool get_string(const std::string& k, std::string* out) const {  // gguf.go:198-206
        auto it = meta.find(k);
        if (it == meta.end() || it->second.type != TString || it->second.is_array) return false;
        *out = it->second.s;
        return true;
    }
    bool get_u32(const std::string& k, uint32_t* out) const {  // gguf.go:209-226
        auto it = meta.find(k);
        if (it == meta.end() || it->second.is_array) return false;
        const Value& v = it->second;
        switch (v.type) {
            case TUint32: case TUint64: *out = (uint32_t)v.u; return true;
            case TInt32: case TInt64: *out = (uint32_t)v.i; return true;
            default: return false;
        }
    }
    bool get_f32(const std::string& k, float* out) const {  // gguf.go:229-241
        auto it = meta.find(k);
        if (it == meta.end() || it->second.is_array) return false;
        const Value& v = it->second;
        if (v.type == TFloat32 || v.type == TFloat64) {
            *out = (float)v.f;
            return true;
        }
        return false;
    }
};

struct Reader {
    FILE* f;
    bool ok = true;
    template <class T> T rd() {
        T v{};
        if (ok && fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
};

bool read_string(Reader& r, std::string* s) {  // gguf.go:322-336
    uint64_t len = r.rd<uint64_t>();
    if (!r.ok) return false;
    if (len > (1u << 20)) { set_err("string too long"); r.ok = false; return false; }
    s->resize(len);
    if (len && fread(&(*s)[0], 1, len, r.f) != len) { r.ok = false; return false; }
    return true;
}

bool read_typed(Reader& r, uint32_t t, Value* v, bool keep) {  // gguf.go:346-414
    v->type = t;
    switch (t) {
        case TUint8: v->u = r.rd<uint8_t>(); break;
        case TInt8: v->i = r.rd<int8_t>(); break;
        case TUint16: v->u = r.rd<uint16_t>(); break;
        case TInt16: v->i = r.rd<int16_t>(); break;
        case TUint32: v->u = r.rd<uint32_t>(); break;
        case TInt32: v->i = r.rd<int32_t>(); break;
        case TFloat32: v->f = r.rd<float>(); break;
        case TBool: v->u = r.rd<uint8_t>() != 0; break;
        case TString: {
            std::string s;
            if (!read_string(r, &s)) return false;
            if (keep) v->s = std::move(s);
            break;
        }
        case TArray: {
            uint32_t et = r.rd<uint32_t>();
            uint64_t n = r.rd<uint64_t>();
            if (!r.ok) return false;
            v->is_array = true;
            v->arr_len = n;
            Value tmp;
            for (uint64_t i = 0; i < n; i++)
                if (!read_typed(r, et, &tmp, false)) return false;
            v->type = et;
            break;
        }
        case TUint64: v->u = r.rd<uint64_t>(); break;
        case TInt64: v->i = r.rd<int64_t>(); break;
        case TFloat64: v->f = r.rd<double>(); break;
        default:
            set_err("unknown value type: " + std::to_string(t));
            return false;
    }
    return r.ok;
}

bool parse(const char* path, File* gf) {  // gguf.go:93-195
    FILE* f = fopen(path, "rb");
    if (!f) { set_err(std::string("open gguf file: ") + path); return false; }
    Reader r{f};
    gf->path = path;
    uint32_t magic = r.rd<uint32_t>();
    if (!r.ok || magic != kMagic) { set_err("invalid magic"); fclose(f); return false; }
    gf->version = r.rd<uint32_t>();
    if (!r.ok || gf->version < 2 || gf->version > 3) {
        set_err("unsupported GGUF version"); fclose(f); return false;
    }
    uint64_t n_tensors = r.rd<uint64_t>();
    uint64_t n_kv = r.rd<uint64_t>();
    if (!r.ok) { set_err("read header"); fclose(f); return false; }
    for (uint64_t i = 0; i < n_kv; i++) {
        std::string key;
        if (!read_string(r, &key)) { if (g_err.empty()) set_err("read metadata key"); fclose(f); return false; }
        uint32_t t = r.rd<uint32_t>();
        Value v;
        if (!r.ok || !read_typed(r, t, &v, true)) {
            if (g_err.empty()) set_err("read metadata value for key " + key);
            fclose(f);
            return false;
        }
        gf->meta[key] = std::move(v);
    }
    gf->tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        TensorInfo& t = gf->tensors[i];
        if (!read_string(r, &t.name)) { set_err("read tensor name"); fclose(f); return false; }
        uint32_t nd = r.rd<uint32_t>();
        if (!r.ok || nd > 8) { set_err("read tensor ndims"); fclose(f); return false; }
        t.dims.resize(nd);
        for (uint32_t j = 0; j < nd; j++) t.dims[j] = r.rd<uint64_t>();
        t.type = r.rd<uint32_t>();
        t.offset = r.rd<uint64_t>();
        if (!r.ok) { set_err("read tensor info"); fclose(f); return false; }
    }
    int64_t pos = ftell(f);
    gf->data_offset = (pos + kAlignment - 1) / kAlignment * kAlignment;  // gguf.go:187-192,416-419
    fclose(f);
    return true;
}

bool read_raw(const File& gf, const TensorInfo& t, std::vector<uint8_t>* out) {  // transformer.go:1148-1156
    FILE* f = fopen(gf.path.c_str(), "rb");
    if (!f) { set_err("open model file"); return false; }
    uint64_t size = data_size(t);
    out->resize(size);
    bool ok = fseek(f, gf.data_offset + (int64_t)t.offset, SEEK_SET) == 0 &&
              (size == 0 || fread(out->data(), 1, size, f) == size);
    fclose(f);
    if (!ok) set_err("read tensor " + t.name);
    return ok;
}

}  // namespace

// gguf.go:616-643 (duplicated at transformer.go:895-919).
extern "C" float goref_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1;
    uint32_t exp = (uint32_t)(h >> 10) & 0x1F;
    uint32_t mant = (uint32_t)h & 0x3FF;
    uint32_t f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign << 31;
        } else {
            exp = 1;
            while ((mant & 0x400) == 0) {
                mant <<= 1;
                exp--;
            }
            mant &= 0x3FF;
            f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        f = (sign << 31) | (0xFFu << 23) | (mant << 13);
    } else {
        f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &f, 4);
    return out;
}

namespace {

inline uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// gguf.go:491-613.  mode picks the Q4_0 element order.
std::vector<float> dequantize(const std::vector<uint8_t>& data, uint32_t type, uint64_t n, int mode) {
    std::vector<float> out(n, 0.0f);
    switch (type) {
        case GF32:  // gguf.go:510-517
            for (uint64_t i = 0; i < n; i++) memcpy(&out[i], &data[i * 4], 4);
            break;
        case GF16:  // gguf.go:519-526
            for (uint64_t i = 0; i < n; i++) out[i] = goref_f16_to_f32(le16(&data[i * 2]));
            break;
        case GBF16: {  // gguf.go:528-536
            for (uint64_t i = 0; i < n; i++) {
                uint32_t bits = (uint32_t)le16(&data[i * 2]) << 16;
                memcpy(&out[i], &bits, 4);
            }
            break;
        }
        case GQ8_0: {  // gguf.go:540-582 (the worker split does not change values)
            uint64_t blocks = (n + 31) / 32;
            for (uint64_t b = 0; b < blocks; b++) {
                uint64_t off = b * 34;
                if (off + 34 > data.size()) break;
                float scale = goref_f16_to_f32(le16(&data[off]));
                for (uint64_t j = 0; j < 32 && b * 32 + j < n; j++)
                    out[b * 32 + j] = scale * (float)(int8_t)data[off + 2 + j];
            }
            break;
        }
        case GQ4_0: {
            for (uint64_t b = 0; b * 32 < n; b++) {
                uint64_t off = b * 18;
                if (off + 18 > data.size()) break;
                float scale = goref_f16_to_f32(le16(&data[off]));
                for (int j = 0; j < 16; j++) {
                    uint8_t byte = data[off + 2 + j];
                    int q0 = (int)(byte & 0x0F) - 8;
                    int q1 = (int)(byte >> 4) - 8;
                    uint64_t i0, i1;
                    if (mode == GOREF_MODE_GO) {  // gguf.go:598-609: interleaved
                        i0 = b * 32 + (uint64_t)j * 2;
                        i1 = i0 + 1;
                    } else {  // ggml layout: low nibble j, high nibble j+16
                        i0 = b * 32 + (uint64_t)j;
                        i1 = i0 + 16;
                    }
                    if (i0 < n) out[i0] = scale * (float)q0;
                    if (i1 < n) out[i1] = scale * (float)q1;
                }
            }
            break;
        }
        default:  // gguf.go:503-506: zero-fill unsupported types
            break;
    }
    return out;
}

// ---------------------------------------------------------------------------
// Worker pool (transformer.go:131-201): NumCPU workers, row chunks.
// ---------------------------------------------------------------------------

class Pool {
   public:
    explicit Pool(int n) : n_(n) {
        for (int i = 1; i < n_; i++) threads_.emplace_back([this, i] { loop(i); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
            gen_++;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    int size() const { return n_; }
    // Runs fn(w) for w in [0, active) and waits.  Worker 0 is the caller.
    void run(int active, const std::function<void(int)>& fn) {
        if (active <= 1) {
            if (active == 1) fn(0);
            return;
        }
        {
            std::lock_guard<std::mutex> g(mu_);
            fn_ = &fn;
            active_ = active;
            pending_ = active - 1;
            gen_++;
        }
        cv_.notify_all();
        fn(0);
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [this] { return pending_ == 0; });
        fn_ = nullptr;
    }

   private:
    void loop(int id) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int)>* fn;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
                if (id >= active_) continue;
                fn = fn_;
            }
            (*fn)(id);
            {
                std::lock_guard<std::mutex> g(mu_);
                if (--pending_ == 0) done_cv_.notify_one();
            }
        }
    }
    int n_;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(int)>* fn_ = nullptr;
    int active_ = 0, pending_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

// transformer.go:810-865 matVecMulQ8Chunk.
void q8_chunk(float* out, const uint8_t* mat, const float* vec, int start, int end, int cols) {
    const int64_t row_bytes = (int64_t)(cols / 32) * 34;  // q8RowBytes, transformer.go:805-807
    const int nb = cols / 32;
    for (int i = start; i < end; i++) {
        const uint8_t* row = mat + (int64_t)i * row_bytes;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = row + (int64_t)b * 34;
            float scale = goref_f16_to_f32(le16(blk));
            const int8_t* q = (const int8_t*)(blk + 2);
            const float* v = vec + b * 32;
            float s0 = (float)q[0] * v[0] + (float)q[1] * v[1] + (float)q[2] * v[2] + (float)q[3] * v[3] +
                       (float)q[4] * v[4] + (float)q[5] * v[5] + (float)q[6] * v[6] + (float)q[7] * v[7];
            float s1 = (float)q[8] * v[8] + (float)q[9] * v[9] + (float)q[10] * v[10] + (float)q[11] * v[11] +
                       (float)q[12] * v[12] + (float)q[13] * v[13] + (float)q[14] * v[14] + (float)q[15] * v[15];
            float s2 = (float)q[16] * v[16] + (float)q[17] * v[17] + (float)q[18] * v[18] + (float)q[19] * v[19] +
                       (float)q[20] * v[20] + (float)q[21] * v[21] + (float)q[22] * v[22] + (float)q[23] * v[23];
            float s3 = (float)q[24] * v[24] + (float)q[25] * v[25] + (float)q[26] * v[26] + (float)q[27] * v[27] +
                       (float)q[28] * v[28] + (float)q[29] * v[29] + (float)q[30] * v[30] + (float)q[31] * v[31];
            sum += scale * (s0 + s1 + s2 + s3);
        }
        out[i] = sum;
    }
}

// The Q8_0 loop of transformer.go:810-865 with ggml Q4_0 blocks: element j of
// the block is (low nibble of byte j) - 8 for j < 16 and (high nibble of byte
// j-16) - 8 for j >= 16; the 8-term partial sums are kept.
void q4_chunk(float* out, const uint8_t* mat, const float* vec, int start, int end, int cols) {
    const int64_t row_bytes = (int64_t)(cols / 32) * 18;
    const int nb = cols / 32;
    for (int i = start; i < end; i++) {
        const uint8_t* row = mat + (int64_t)i * row_bytes;
        float sum = 0.0f;
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = row + (int64_t)b * 18;
            float scale = goref_f16_to_f32(le16(blk));
            float qf[32];
            for (int j = 0; j < 16; j++) {
                qf[j] = (float)((int)(blk[2 + j] & 0x0F) - 8);
                qf[j + 16] = (float)((int)(blk[2 + j] >> 4) - 8);
            }
            const float* v = vec + b * 32;
            float s[4];
            for (int k = 0; k < 4; k++) {
                const float* a = qf + 8 * k;
                const float* c = v + 8 * k;
                s[k] = a[0] * c[0] + a[1] * c[1] + a[2] * c[2] + a[3] * c[3] + a[4] * c[4] + a[5] * c[5] +
                       a[6] * c[6] + a[7] * c[7];
            }
            sum += scale * (s[0] + s[1] + s[2] + s[3]);
        }
        out[i] = sum;
    }
}

// transformer.go:767-784 matVecMulChunk.
void f32_chunk(float* out, const float* mat, const float* vec, int start, int end, int cols) {
    for (int i = start; i < end; i++) {
        float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        const float* row = mat + (int64_t)i * cols;
        int j = 0;
        for (; j + 15 < cols; j += 16) {
            s0 += row[j] * vec[j] + row[j + 1] * vec[j + 1] + row[j + 2] * vec[j + 2] + row[j + 3] * vec[j + 3];
            s1 += row[j + 4] * vec[j + 4] + row[j + 5] * vec[j + 5] + row[j + 6] * vec[j + 6] +
                  row[j + 7] * vec[j + 7];
            s2 += row[j + 8] * vec[j + 8] + row[j + 9] * vec[j + 9] + row[j + 10] * vec[j + 10] +
                  row[j + 11] * vec[j + 11];
            s3 += row[j + 12] * vec[j + 12] + row[j + 13] * vec[j + 13] + row[j + 14] * vec[j + 14] +
                  row[j + 15] * vec[j + 15];
        }
        for (; j < cols; j++) s0 += row[j] * vec[j];
        out[i] = s0 + s1 + s2 + s3;
    }
}

// transformer.go:868-892 matVecMulQ8Pooled / 757-763 matVecMulPooled.
void pooled(Pool& pool, int rows, const std::function<void(int, int)>& chunk) {
    if (rows < 512) {
        chunk(0, rows);
        return;
    }
    int nw = pool.size();
    int cs = (rows + nw - 1) / nw;
    int active = 0;
    for (int w = 0; w < nw; w++) {
        int s = w * cs;
        if (s >= std::min(s + cs, rows)) break;
        active++;
    }
    pool.run(active, [&](int w) {
        int s = w * cs;
        int e = std::min(s + cs, rows);
        chunk(s, e);
    });
}

struct Layer {  // transformer.go:51-76
    std::vector<uint8_t> wq, wk, wv, wo, wg, wu, wd;
    int wq_cols = 0, wk_cols = 0, wv_cols = 0, wo_cols = 0, wg_cols = 0, wu_cols = 0, wd_cols = 0;
    uint32_t wq_t = 0, wk_t = 0, wv_t = 0, wo_t = 0, wg_t = 0, wu_t = 0, wd_t = 0;
    std::vector<float> bq, bk, bv, attn_norm, ffn_norm;
};

}  // namespace

struct goref_model {
    std::unique_ptr<Pool> pool;
    int mode = GOREF_MODE_GO;
    goref_config cfg{};
    std::vector<float> token_embed;  // transformer.go:81
    std::vector<float> output_norm;
    std::vector<uint8_t> output;     // raw lm_head blocks (empty = tied)
    uint32_t output_t = GQ8_0;
    int output_cols = 0;
    std::vector<Layer> layers;
    struct KV {  // transformer.go:88-92
        std::vector<float> k, v;
        int len = 0;
    };
    std::vector<KV> cache;
    std::vector<float> scores;  // inferBuffers.scores [MaxSeqLen]
};

namespace {

// matVecMulQ8Pooled with the mode's type dispatch: the Go engine sends every
// 2-D weight through the Q8_0 loop (transformer.go:627-629, 721-734).
void matvec_w(goref_model* m, float* out, const std::vector<uint8_t>& mat, uint32_t type, const float* vec,
              int rows, int cols) {
    bool q4 = (m->mode == GOREF_MODE_GGML_Q4 && type == GQ4_0);
    pooled(*m->pool, rows, [&](int s, int e) {
        if (q4)
            q4_chunk(out, mat.data(), vec, s, e, cols);
        else
            q8_chunk(out, mat.data(), vec, s, e, cols);
    });
}

}  // namespace

extern "C" {

const char* goref_last_error(void) { return g_err.c_str(); }

void goref_rmsnorm(float* x, const float* w, int32_t n, float eps) {  // transformer.go:922-932
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = (float)(1.0 / std::sqrt((double)(ss / (float)n) + (double)eps));
    for (int i = 0; i < n; i++) x[i] = x[i] * ss * w[i];
}

void goref_rope(float* x, int32_t head_dim, int32_t num_heads, int32_t pos, float theta) {  // 936-951
    for (int h = 0; h < num_heads; h++) {
        for (int i = 0; i < head_dim / 2; i++) {
            float freq = 1.0f / (float)std::pow((double)theta, (double)(2 * i) / (double)head_dim);
            float angle = (float)pos * freq;
            float c = (float)std::cos((double)angle);
            float s = (float)std::sin((double)angle);
            int idx = h * head_dim + 2 * i;
            float x0 = x[idx], x1 = x[idx + 1];
            x[idx] = x0 * c - x1 * s;
            x[idx + 1] = x0 * s + x1 * c;
        }
    }
}

float goref_silu(float x) { return x / (1.0f + (float)std::exp(-(double)x)); }  // 954-956

void goref_softmax(float* x, int32_t n) {  // transformer.go:959-974
    float mx = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = (float)std::exp((double)(x[i] - mx));
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

int32_t goref_argmax(const float* x, int32_t n) {  // transformer.go:1038-1046
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

void goref_matvec_q8_0(const uint8_t* w, const float* x, float* y, int32_t rows, int32_t cols) {
    q8_chunk(y, w, x, 0, rows, cols);
}
void goref_matvec_q4_0(const uint8_t* w, const float* x, float* y, int32_t rows, int32_t cols) {
    q4_chunk(y, w, x, 0, rows, cols);
}
void goref_matvec_f32(const float* w, const float* x, float* y, int32_t rows, int32_t cols) {
    f32_chunk(y, w, x, 0, rows, cols);
}
void goref_matvec_q8_0_mt(goref_model* m, const uint8_t* w, const float* x, float* y, int32_t rows,
                          int32_t cols) {
    pooled(*m->pool, rows, [&](int s, int e) { q8_chunk(y, w, x, s, e, cols); });
}

void goref_attention(const float* q, const float* k, const float* v, float* out, int32_t nh, int32_t nkv,
                     int32_t hd, int32_t ctx) {  // transformer.go:658-685
    int kv_dim = nkv * hd;
    int group = nh / nkv;
    float scale = (float)(1.0 / std::sqrt((double)hd));
    std::vector<float> scores(ctx);
    for (int i = 0; i < nh * hd; i++) out[i] = 0.0f;
    for (int h = 0; h < nh; h++) {
        int kvh = h / group;
        const float* qh = q + h * hd;
        for (int t = 0; t < ctx; t++) {
            const float* kh = k + (int64_t)t * kv_dim + kvh * hd;
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot += qh[d] * kh[d];
            scores[t] = dot * scale;
        }
        goref_softmax(scores.data(), ctx);
        for (int t = 0; t < ctx; t++) {
            const float* vh = v + (int64_t)t * kv_dim + kvh * hd;
            for (int d = 0; d < hd; d++) out[h * hd + d] += scores[t] * vh[d];
        }
    }
}

goref_model* goref_pool_only(int32_t n_threads) {
    auto* m = new goref_model();
    int n = n_threads > 0 ? n_threads : (int)std::max(1u, std::thread::hardware_concurrency());
    m->pool.reset(new Pool(n));
    return m;
}

int32_t goref_num_threads(const goref_model* m) { return m->pool ? m->pool->size() : 0; }

goref_model* goref_load(const char* path, int32_t num_ctx, int32_t n_threads, int32_t mode) {
    g_err.clear();
    File gf;
    if (!parse(path, &gf)) return nullptr;
    auto m = std::unique_ptr<goref_model>(goref_pool_only(n_threads));
    m->mode = mode;
    goref_config& c = m->cfg;

    // transformer.go:1350-1421 extractConfig.
    c.rms_norm_eps = 1e-5f;
    c.rope_theta = 10000.0f;
    std::string arch;
    if (!gf.get_string("general.architecture", &arch)) arch = "llama";
    snprintf(c.arch, sizeof c.arch, "%s", arch.c_str());
    std::string p = arch + ".";
    uint32_t u;
    float fv;
    if (gf.get_u32(p + "embedding_length", &u)) c.hidden_size = (int)u;
    if (gf.get_u32(p + "feed_forward_length", &u)) c.intermediate_size = (int)u;
    if (gf.get_u32(p + "block_count", &u)) c.num_layers = (int)u;
    if (gf.get_u32(p + "attention.head_count", &u)) c.num_heads = (int)u;
    if (gf.get_u32(p + "attention.head_count_kv", &u)) c.num_kv_heads = (int)u;
    else c.num_kv_heads = c.num_heads;
    if (gf.get_u32(p + "context_length", &u)) c.max_seq_len = (int)u;
    else c.max_seq_len = 4096;
    if (gf.get_f32(p + "attention.layer_norm_rms_epsilon", &fv)) c.rms_norm_eps = fv;
    if (gf.get_f32(p + "rope.freq_base", &fv)) c.rope_theta = fv;
    {
        auto it = gf.meta.find("tokenizer.ggml.tokens");
        if (it != gf.meta.end() && it->second.is_array) c.vocab_size = (int)it->second.arr_len;
    }
    if (c.num_heads > 0 && c.hidden_size > 0) c.head_dim = c.hidden_size / c.num_heads;
    if (c.intermediate_size == 0 && c.hidden_size > 0)
        c.intermediate_size = ((c.hidden_size * 8 / 3) + 255) / 256 * 256;
    if (c.hidden_size == 0) { set_err("embedding_length not found in GGUF metadata"); return nullptr; }
    if (c.num_layers == 0) { set_err("block_count not found in GGUF metadata"); return nullptr; }
    // transformer.go:233-235.
    if (num_ctx > 0 && num_ctx < c.max_seq_len) c.max_seq_len = num_ctx;
    // bpe.go:48-49, 105-110.
    c.bos_id = 1;
    c.eos_id = 2;
    if (gf.get_u32("tokenizer.ggml.bos_token_id", &u)) c.bos_id = (int)u;
    if (gf.get_u32("tokenizer.ggml.eos_token_id", &u)) c.eos_id = (int)u;

    // transformer.go:1122-1335 loadWeights.
    auto read_f32 = [&](const std::string& name, std::vector<float>* out) -> bool {
        const TensorInfo* t = gf.find(name);
        if (!t) { set_err("tensor \"" + name + "\" not found"); return false; }
        std::vector<uint8_t> raw;
        if (!read_raw(gf, *t, &raw)) return false;
        *out = dequantize(raw, t->type, t->elements(), m->mode);
        return true;
    };
    auto read_bytes = [&](const std::string& name, std::vector<uint8_t>* out, int* cols, uint32_t* type) -> bool {
        const TensorInfo* t = gf.find(name);
        if (!t) { set_err("tensor \"" + name + "\" not found"); return false; }
        if (!read_raw(gf, *t, out)) return false;
        *cols = (int)t->dims[0];  // GGUF: [cols, rows] (transformer.go:1239)
        *type = t->type;
        return true;
    };
    if (!read_f32("token_embd.weight", &m->token_embed)) return nullptr;
    if (!read_f32("output_norm.weight", &m->output_norm)) return nullptr;
    c.tied = 1;
    if (const TensorInfo* t = gf.find("output.weight")) {
        bool usable = (t->type == GQ8_0) || (m->mode == GOREF_MODE_GGML_Q4 && t->type == GQ4_0);
        if (usable) {  // transformer.go:1178-1180
            if (!read_raw(gf, *t, &m->output)) return nullptr;
            m->output_cols = (int)t->dims[0];
            m->output_t = t->type;
            c.tied = 0;
        }
        // else transformer.go:1181-1189: dropped, the tied fp32 path is used.
    }
    if (c.tied) m->output_cols = c.hidden_size;
    m->layers.resize(c.num_layers);
    for (int i = 0; i < c.num_layers; i++) {
        std::string pre = "blk." + std::to_string(i) + ".";
        Layer& L = m->layers[i];
        if (!read_bytes(pre + "attn_q.weight", &L.wq, &L.wq_cols, &L.wq_t) ||
            !read_bytes(pre + "attn_k.weight", &L.wk, &L.wk_cols, &L.wk_t) ||
            !read_bytes(pre + "attn_v.weight", &L.wv, &L.wv_cols, &L.wv_t) ||
            !read_bytes(pre + "attn_output.weight", &L.wo, &L.wo_cols, &L.wo_t) ||
            !read_bytes(pre + "ffn_gate.weight", &L.wg, &L.wg_cols, &L.wg_t) ||
            !read_bytes(pre + "ffn_up.weight", &L.wu, &L.wu_cols, &L.wu_t) ||
            !read_bytes(pre + "ffn_down.weight", &L.wd, &L.wd_cols, &L.wd_t) ||
            !read_f32(pre + "attn_norm.weight", &L.attn_norm) || !read_f32(pre + "ffn_norm.weight", &L.ffn_norm)) {
            set_err("layer " + std::to_string(i) + ": " + g_err);
            return nullptr;
        }
        // Optional biases (transformer.go:1271-1276, 1298-1301).
        std::string keep = g_err;
        if (!read_f32(pre + "attn_q.bias", &L.bq)) L.bq.clear();
        if (!read_f32(pre + "attn_k.bias", &L.bk)) L.bk.clear();
        if (!read_f32(pre + "attn_v.bias", &L.bv)) L.bv.clear();
        g_err = keep;
    }
    c.weight_type = (int)m->layers[0].wq_t;
    // transformer.go:261-268: KV cache, capacity MaxSeqLen.
    m->cache.resize(c.num_layers);
    int kv_dim = c.num_kv_heads * c.head_dim;
    for (auto& kv : m->cache) {
        kv.k.reserve((size_t)c.max_seq_len * kv_dim);
        kv.v.reserve((size_t)c.max_seq_len * kv_dim);
    }
    m->scores.assign(c.max_seq_len, 0.0f);
    return m.release();
}

void goref_free(goref_model* m) { delete m; }

int goref_get_config(const goref_model* m, goref_config* out) {
    if (!m || !out) return -1;
    *out = m->cfg;
    return 0;
}

void goref_reset(goref_model* m) {  // transformer.go:742-749
    for (auto& kv : m->cache) {
        kv.k.clear();
        kv.v.clear();
        kv.len = 0;
    }
}

int32_t goref_cache_len(const goref_model* m) { return m->cache.empty() ? 0 : m->cache[0].len; }

}  // extern "C"

namespace {

// transformer.go:599-697 selfAttention.
int self_attention(goref_model* m, const float* x, int seq_len, int layer, float* out) {
    const goref_config& c = m->cfg;
    const int hidden = c.hidden_size, hd = c.head_dim, nh = c.num_heads, nkv = c.num_kv_heads;
    const int kv_dim = nkv * hd;
    Layer& L = m->layers[layer];
    auto& kvc = m->cache[layer];
    std::vector<float> q(hidden), k(kv_dim), v(kv_dim), proj(hidden);
    for (int i = 0; i < seq_len * hidden; i++) out[i] = 0.0f;
    for (int pos = 0; pos < seq_len; pos++) {
        const float* xp = x + (int64_t)pos * hidden;
        std::fill(q.begin(), q.end(), 0.0f);
        std::fill(k.begin(), k.end(), 0.0f);
        std::fill(v.begin(), v.end(), 0.0f);
        matvec_w(m, q.data(), L.wq, L.wq_t, xp, hidden, L.wq_cols);
        matvec_w(m, k.data(), L.wk, L.wk_t, xp, kv_dim, L.wk_cols);
        matvec_w(m, v.data(), L.wv, L.wv_t, xp, kv_dim, L.wv_cols);
        if (!L.bq.empty()) for (int i = 0; i < hidden; i++) q[i] += L.bq[i];
        if (!L.bk.empty()) for (int i = 0; i < kv_dim; i++) k[i] += L.bk[i];
        if (!L.bv.empty()) for (int i = 0; i < kv_dim; i++) v[i] += L.bv[i];
        int abs_pos = kvc.len;
        goref_rope(q.data(), hd, nh, abs_pos, c.rope_theta);
        goref_rope(k.data(), hd, nkv, abs_pos, c.rope_theta);
        kvc.k.insert(kvc.k.end(), k.begin(), k.end());
        kvc.v.insert(kvc.v.end(), v.begin(), v.end());
        kvc.len++;
        int cached = kvc.len;
        if (cached > (int)m->scores.size()) {
            set_err("context length exceeded");
            return -1;
        }
        int group = nh / nkv;
        float scale = (float)(1.0 / std::sqrt((double)hd));
        for (int h = 0; h < nh; h++) {
            int kvh = h / group;
            const float* qh = q.data() + h * hd;
            float* sc = m->scores.data();
            for (int t = 0; t < cached; t++) {
                const float* kh = kvc.k.data() + (int64_t)t * kv_dim + kvh * hd;
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot += qh[d] * kh[d];
                sc[t] = dot * scale;
            }
            goref_softmax(sc, cached);
            float* o = out + (int64_t)pos * hidden + h * hd;
            for (int t = 0; t < cached; t++) {
                const float* vh = kvc.v.data() + (int64_t)t * kv_dim + kvh * hd;
                for (int d = 0; d < hd; d++) o[d] += sc[t] * vh[d];
            }
        }
        std::fill(proj.begin(), proj.end(), 0.0f);
        matvec_w(m, proj.data(), L.wo, L.wo_t, out + (int64_t)pos * hidden, hidden, L.wo_cols);
        memcpy(out + (int64_t)pos * hidden, proj.data(), sizeof(float) * hidden);
    }
    return 0;
}

// transformer.go:700-739 feedForward.
void feed_forward(goref_model* m, const float* x, int seq_len, int layer, float* out) {
    const goref_config& c = m->cfg;
    const int hidden = c.hidden_size, inter = c.intermediate_size;
    Layer& L = m->layers[layer];
    std::vector<float> gate(inter), up(inter), down(hidden);
    for (int pos = 0; pos < seq_len; pos++) {
        const float* xp = x + (int64_t)pos * hidden;
        std::fill(gate.begin(), gate.end(), 0.0f);
        std::fill(up.begin(), up.end(), 0.0f);
        matvec_w(m, gate.data(), L.wg, L.wg_t, xp, inter, L.wg_cols);
        matvec_w(m, up.data(), L.wu, L.wu_t, xp, inter, L.wu_cols);
        for (int i = 0; i < inter; i++) gate[i] = goref_silu(gate[i]) * up[i];
        std::fill(down.begin(), down.end(), 0.0f);
        matvec_w(m, down.data(), L.wd, L.wd_t, gate.data(), hidden, L.wd_cols);
        memcpy(out + (int64_t)pos * hidden, down.data(), sizeof(float) * hidden);
    }
}

// transformer.go:519-557 forward, split at the final RMSNorm.
int forward_body(goref_model* m, const int32_t* tokens, int seq_len, std::vector<float>* xout) {
    const goref_config& c = m->cfg;
    const int hidden = c.hidden_size;
    std::vector<float>& x = *xout;
    x.assign((size_t)seq_len * hidden, 0.0f);
    for (int i = 0; i < seq_len; i++) {
        int tok = tokens[i];
        if (tok >= 0 && tok < c.vocab_size)
            memcpy(&x[(size_t)i * hidden], &m->token_embed[(size_t)tok * hidden], sizeof(float) * hidden);
    }
    std::vector<float> normed, attn((size_t)seq_len * hidden), ffn((size_t)seq_len * hidden);
    for (int layer = 0; layer < c.num_layers; layer++) {  // transformerLayer, 560-596
        Layer& L = m->layers[layer];
        normed = x;
        for (int i = 0; i < seq_len; i++) goref_rmsnorm(&normed[(size_t)i * hidden], L.attn_norm.data(), hidden, c.rms_norm_eps);
        if (self_attention(m, normed.data(), seq_len, layer, attn.data()) != 0) return -1;
        for (size_t i = 0; i < x.size(); i++) x[i] += attn[i];
        normed = x;
        for (int i = 0; i < seq_len; i++) goref_rmsnorm(&normed[(size_t)i * hidden], L.ffn_norm.data(), hidden, c.rms_norm_eps);
        feed_forward(m, normed.data(), seq_len, layer, ffn.data());
        for (size_t i = 0; i < x.size(); i++) x[i] += ffn[i];
    }
    for (int i = 0; i < seq_len; i++) goref_rmsnorm(&x[(size_t)i * hidden], m->output_norm.data(), hidden, c.rms_norm_eps);
    return 0;
}

}  // namespace

extern "C" {

int goref_forward_hidden(goref_model* m, const int32_t* tokens, int32_t n, float* hidden) {
    if (!m || n <= 0) return -1;
    std::vector<float> x;
    if (forward_body(m, tokens, n, &x) != 0) return -1;
    memcpy(hidden, &x[(size_t)(n - 1) * m->cfg.hidden_size], sizeof(float) * m->cfg.hidden_size);
    return 0;
}

int goref_forward(goref_model* m, const int32_t* tokens, int32_t n, float* logits) {
    if (!m || n <= 0) return -1;
    const goref_config& c = m->cfg;
    std::vector<float> x;
    if (forward_body(m, tokens, n, &x) != 0) return -1;
    const float* last = &x[(size_t)(n - 1) * c.hidden_size];
    for (int i = 0; i < c.vocab_size; i++) logits[i] = 0.0f;
    if (!m->output.empty()) {  // transformer.go:549-550
        matvec_w(m, logits, m->output, m->output_t, last, c.vocab_size, m->output_cols);
    } else {  // transformer.go:551-554 tied fp32 fallback
        const float* te = m->token_embed.data();
        int hidden = c.hidden_size;
        pooled(*m->pool, c.vocab_size, [&](int s, int e) { f32_chunk(logits, te, last, s, e, hidden); });
    }
    return 0;
}

int32_t goref_sample(float* logits, int32_t n, double temperature, int32_t top_k, double top_p,
                     double repeat_penalty, const int32_t* generated, int32_t n_generated, float r) {
    // transformer.go:981-1036.
    double temp = temperature;
    if (temp <= 0) temp = 1.0;
    if (repeat_penalty > 1 && n_generated > 0) {
        float penalty = (float)repeat_penalty;
        for (int i = 0; i < n_generated; i++) {
            int tok = generated[i];
            if (tok >= 0 && tok < n) {
                if (logits[tok] > 0) logits[tok] /= penalty;
                else logits[tok] *= penalty;
            }
        }
    }
    if (temp < 0.01) return goref_argmax(logits, n);
    for (int i = 0; i < n; i++) logits[i] /= (float)temp;
    struct TP { int idx; float logit; };
    if (top_k > 0 && top_k < n) {  // topKFilter 1053-1069
        std::vector<TP> items(n);
        for (int i = 0; i < n; i++) items[i] = {i, logits[i]};
        std::sort(items.begin(), items.end(), [](const TP& a, const TP& b) { return a.logit > b.logit; });
        float thr = items[top_k - 1].logit;
        for (int i = 0; i < n; i++)
            if (logits[i] < thr) logits[i] = -INFINITY;
    }
    if (top_p > 0 && top_p < 1) {  // topPFilter 1071-1114
        std::vector<TP> items(n);
        for (int i = 0; i < n; i++) items[i] = {i, logits[i]};
        // Go's sort.Slice is not stable; a stable order keeps ties by index.
        std::stable_sort(items.begin(), items.end(), [](const TP& a, const TP& b) { return a.logit > b.logit; });
        std::vector<float> probs(n);
        float mx = items[0].logit;
        float sum = 0.0f;
        for (int i = 0; i < n; i++) {
            probs[i] = (float)std::exp((double)(items[i].logit - mx));
            sum += probs[i];
        }
        for (int i = 0; i < n; i++) probs[i] /= sum;
        float cum = 0.0f;
        int cut = n - 1;
        float p = (float)top_p;
        for (int i = 0; i < n; i++) {
            cum += probs[i];
            if (cum >= p) { cut = i; break; }
        }
        std::vector<char> keep(n, 0);
        for (int i = 0; i <= cut; i++) keep[items[i].idx] = 1;
        for (int i = 0; i < n; i++)
            if (!keep[i]) logits[i] = -INFINITY;
    }
    goref_softmax(logits, n);
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        cum += logits[i];
        if (r <= cum) return i;
    }
    return n - 1;
}

int goref_predict(goref_model* m, const int32_t* prompt, int32_t n_prompt, int32_t max_gen, double temperature,
                  int32_t top_k, double top_p, double repeat_penalty, const int32_t* stop_ids, int32_t n_stop,
                  const float* uniforms, int32_t* out_ids, int32_t* n_out) {
    // transformer.go:325-382.
    goref_reset(m);
    std::vector<int32_t> tokens;
    tokens.push_back(m->cfg.bos_id);
    tokens.insert(tokens.end(), prompt, prompt + n_prompt);
    if (max_gen <= 0) max_gen = 256;
    std::vector<int32_t> generated;
    std::vector<float> logits(m->cfg.vocab_size);
    for (int i = 0; i < max_gen; i++) {
        if (goref_forward(m, tokens.data(), (int)tokens.size(), logits.data()) != 0) return -1;
        float r = uniforms ? uniforms[i] : 0.5f;
        int next = goref_sample(logits.data(), m->cfg.vocab_size, temperature, top_k, top_p, repeat_penalty,
                                generated.data(), (int)generated.size(), r);
        if (next == m->cfg.eos_id) break;
        bool stop = false;
        for (int s = 0; s < n_stop; s++) stop |= (stop_ids[s] == next);
        if (stop) break;
        generated.push_back(next);
        tokens.assign(1, next);
    }
    for (size_t i = 0; i < generated.size(); i++) out_ids[i] = generated[i];
    *n_out = (int32_t)generated.size();
    return 0;
}

int64_t goref_dequant_tensor(const char* path, const char* name, int32_t mode, float* out, int64_t n) {
    File gf;
    if (!parse(path, &gf)) return -1;
    const TensorInfo* t = gf.find(name);
    if (!t) { set_err(std::string("tensor not found: ") + name); return -1; }
    std::vector<uint8_t> raw;
    if (!read_raw(gf, *t, &raw)) return -1;
    std::vector<float> v = dequantize(raw, t->type, t->elements(), mode);
    if ((int64_t)v.size() > n) { set_err("output too small"); return -1; }
    memcpy(out, v.data(), v.size() * sizeof(float));
    return (int64_t)v.size();
}

}  // extern "C"
