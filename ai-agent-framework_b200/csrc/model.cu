// Model load and the per-token drivers.
//
// Load follows transformer.go:215-310 (Engine.Load) and 1122-1335
// (loadWeights) for what is read and how it is interpreted, but nothing is
// dequantised: the Q8_0 / Q4_0 blocks of every weight matrix are uploaded and
// rearranged on the device into the tiled layout of the decode kernel
// (dev.cuh: 8-row tiles, quants and f16 scales in separate regions, the same
// bytes per weight).  Wq, Wk and Wv form one [qd + 2*kvd] x H matrix, the gate
// matrix is followed by the up matrix, every region starts on a 256-byte
// boundary and is padded so 16-byte bulk copies never leave the arena.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "gemm.h"
#include "model.h"
#include "sample.h"
#include "upload.h"

void b2_mvb_release(int dev, cudaStream_t s);

namespace b2 {

// Allocation-failure injection (b2_debug_fail_alloc): the device allocation
// that brings g_fail_left to zero fails.
std::atomic<int> g_fail_left{0};

namespace {

int dev_malloc(void** p, size_t bytes) {
    int left = g_fail_left.load();
    while (left > 0 && !g_fail_left.compare_exchange_weak(left, left - 1)) {
    }
    if (left == 1) {
        *p = nullptr;
        return -1;
    }
    return cudaMalloc(p, bytes) == cudaSuccess ? 0 : -1;
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

constexpr int kWarmTokens = 256;  // the prompt path's warm-up at load: one full chunk

// gguf.go:616-643 float16ToFloat32 (host side, for small F16 vectors).
float f16_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1F, mant = h & 0x3FF, f;
    if (exp == 0) {
        if (mant == 0) {
            f = sign << 31;
        } else {
            exp = 1;
            while ((mant & 0x400) == 0) { mant <<= 1; exp--; }
            mant &= 0x3FF;
            f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
        }
    } else if (exp == 0x1F) {
        f = (sign << 31) | (0xFFu << 23) | (mant << 13);
    } else {
        f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float o;
    memcpy(&o, &f, 4);
    return o;
}

// A weight matrix of the decode kernel: GGUF tensors stacked by rows,
// tiled into the arena at `off`.
struct MatPart {
    std::string name;
    int64_t row0, rows;  // source rows of the tensor that go in
};
struct MatGroup {
    std::vector<MatPart> parts;  // stacked in order
    size_t off;
    int64_t rows, cols;          // the tiled matrix (this rank's share)
    int64_t half_rows = 0;       // gate/up: rows of each part (8-row interleave)
    int64_t cb0 = 0, nb_src = 0; // column blocks [cb0, cb0 + cols / 32) of source rows of nb_src blocks
};

// Row of the stacked source tensors that row r of a tiled matrix holds.  The
// gate/up matrix (half_rows = FF) interleaves them 8 rows at a time, so one
// 16-row tile carries the gate and up rows of the same 8 outputs: tile t =
// gate rows 8t .. 8t+7, then up rows 8t .. 8t+7 (stacked at FF + ...).
__host__ __device__ inline int64_t src_row(int64_t r, int64_t half_rows) {
    if (half_rows == 0) return r;
    return (r >> 4) * 8 + (r & 7) + ((r & 8) ? half_rows : 0);
}

// One thread per (row, block) of the padded matrix: ggml block -> tiled
// quants + scale (padding rows become zero).  Source rows have nb blocks (a
// tensor-parallel column share arrives already cut to its window).
__global__ void repack_kernel(const uint8_t* raw, uint8_t* dst, int64_t rows, int64_t rp, int64_t nb, int qtype,
                              int64_t half_rows) {
    const int bpb = qtype == 8 ? 34 : 18, qb = tile_qb(qtype);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rp * nb; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nb, b = i - r * nb;
        uint8_t* sd = dst + tiled_soff(r, b, nb, rp, qtype);
        if (r >= rows) {
            sd[0] = sd[1] = 0;
            for (int e = 0; e < qb; e++) dst[tiled_qoff(r, b, e, nb, qtype)] = 0;
            continue;
        }
        const uint8_t* src = raw + (src_row(r, half_rows) * nb + b) * bpb;
        sd[0] = src[0];
        sd[1] = src[1];
        for (int e = 0; e < qb; e++) dst[tiled_qoff(r, b, e, nb, qtype)] = src[2 + e];
    }
}

// Element (r, j) of a tiled Q8_0 / Q4_0 matrix (gguf.go:540-582; Q4_0 in
// the ggml element order).
__device__ __forceinline__ float tiled_elem(const uint8_t* base, int64_t r, int64_t j, int64_t nb, int64_t rp, int qtype) {
    const int64_t b = j >> 5;
    const int e = (int)(j & 31);
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(base + tiled_soff(r, b, nb, rp, qtype)));
    if (qtype == 8) return d * (float)(int8_t)base[tiled_qoff(r, b, e, nb, 8)];
    const uint8_t byte = base[tiled_qoff(r, b, e & 15, nb, 2)];
    return d * (float)(((e < 16) ? (byte & 15) : (byte >> 4)) - 8);
}

__global__ void dequant_kernel(TensorLoc t, float* dst) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < t.elements; i += (uint64_t)gridDim.x * blockDim.x) {
        float v;
        if (t.type == 8 || t.type == 2) {
            const int64_t r = (int64_t)(i / (uint64_t)t.cols), j = (int64_t)(i % (uint64_t)t.cols);
            // gate / up halves of the interleaved gate/up matrix (src_row inverse)
            const int64_t tr = t.half ? (r >> 3) * 16 + (r & 7) + (t.half == 2 ? 8 : 0) : t.row0 + r;
            v = tiled_elem(static_cast<const uint8_t*>(t.dev), tr, j, t.cols / 32, t.rp, (int)t.type);
        } else {
            v = static_cast<const float*>(t.dev)[i];
        }
        dst[i] = v;
    }
}

__global__ void embed_mean_kernel(const ModelDev m, const int* toks, int n, float* out) {
    // transformer.go:445-490 Embed: sum rows in order, scale by 1/n, L2 normalise.
    __shared__ float red[32];
    __shared__ float total;
    const float scale = 1.0f / (float)n;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < m.H; j += blockDim.x) {
        float e = 0.0f;
        for (int t = 0; t < n; t++) {
            const int tok = toks[t];
            if (tok < 0 || tok >= m.Vemb) continue;
            e += tiled_elem(m.tok_embd, tok, j, m.H / 32, m.Vp_emb, m.qtype);
        }
        e *= scale;
        out[j] = e;
        ss += e * e;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
        total = (float)sqrt((double)t);
    }
    __syncthreads();
    if (total > 0.0f)
        for (int j = threadIdx.x; j < m.H; j += blockDim.x) out[j] = out[j] / total;
}

}  // namespace

int launch_dequant(const TensorLoc& t, float* dst, cudaStream_t s) {
    int blocks = (int)std::min<uint64_t>((t.elements + 255) / 256, 148 * 16);
    if (blocks < 1) blocks = 1;
    dequant_kernel<<<blocks, 256, 0, s>>>(t, dst);
    return cudaGetLastError() == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

int launch_embed_mean(const b2_model* m, const int* d_tokens, int n, float* d_out, cudaStream_t s) {
    embed_mean_kernel<<<1, 256, 0, s>>>(m->dev, d_tokens, n, d_out);
    return cudaGetLastError() == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

int check_device_status(b2_model* m, std::string* err) {
    int code = 0;
    cudaError_t e = cudaMemcpyAsync(&code, m->dev.err, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
        *err = std::string("CUDA: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    if (code != 0) {
        cudaMemsetAsync(m->dev.err, 0, sizeof(int), m->stream);
        cudaStreamSynchronize(m->stream);
        *err = "device-side wait timed out (bounded wait gave up)";
        return code;
    }
    return B2_OK;
}

// Attention context splits per query head over the `cached` positions before
// the new one: one K/V tile per split while the merge buffer and the grid
// allow it (more q CTAs = a shorter critical path); beyond that a split walks
// several tiles.  The cap keeps CTAs free for the k / v rows.
// The slices rank `rank` of a tp-way model keeps (b2_tp_share_of): heads
// evenly, the FFN by 32-element blocks (the first ranks take the smaller
// shares when the blocks do not divide), the vocabulary by rows.
int tp_share(int H, int nh, int nkv, int FF, int V, int tp, int rank, b2_tp_share* s) {
    if (tp < 1 || rank < 0 || rank >= tp || nh % tp || nkv % tp || H % nh || FF % 32) return B2_ERR_BAD_ARG;
    const int hd = H / nh, nhl = nh / tp, nkvl = nkv / tp;
    const int nbf = FF / 32;
    const int fb0 = (int)((int64_t)rank * nbf / tp), fb1 = (int)((int64_t)(rank + 1) * nbf / tp);
    const int v0 = (int)((int64_t)rank * V / tp), v1 = (int)((int64_t)(rank + 1) * V / tp);
    if (fb1 == fb0 || v1 == v0) return B2_ERR_BAD_ARG;
    s->q_row0 = rank * nhl * hd;
    s->q_rows = nhl * hd;
    s->kv_row0 = rank * nkvl * hd;
    s->kv_rows = nkvl * hd;
    s->ffn_row0 = 32 * fb0;
    s->ffn_rows = 32 * (fb1 - fb0);
    s->vocab_row0 = v0;
    s->vocab_rows = v1 - v0;
    return B2_OK;
}

// Gate/up share of a residual-row owner CTA, in percent of the others' (gu_plan).
constexpr int kGuOwnerPct = 100;

static int splits_for(const b2_model* m, int cached) {
    int s = (cached + m->dev.attn_tile - 1) / m->dev.attn_tile;
    int cap = std::max(1, std::min(m->max_splits, (m->grid - 1) / std::max(1, m->dev.nh)));
    return std::max(1, std::min(s, cap));
}

int run_tokens(b2_model* m, const int32_t* host_tokens, int n, std::string* err) {
    if (n <= 0) { *err = "no tokens"; return B2_ERR_BAD_ARG; }
    if (m->cache_len + n > m->cfg.max_seq_len) {
        *err = "context length exceeded: " + std::to_string(m->cache_len + n) + " > " +
               std::to_string(m->cfg.max_seq_len);
        return B2_ERR_CONTEXT;
    }
    if (prefill_gemm_ok(m, n)) {
        // a prompt: one weight pass per chunk on the tensor cores
        const int rc = prefill_gemm(m, host_tokens, n, m->cache_len, err);
        if (rc) return rc;
        m->cache_len += n;
        return B2_OK;
    }
    if (m->pin_pending) cudaEventSynchronize(m->ev_pin);  // h_pinned may still feed an earlier copy
    memcpy(m->h_pinned, host_tokens, sizeof(int32_t) * n);
    cudaError_t e = cudaMemcpyAsync(m->d_tokens, m->h_pinned, sizeof(int32_t) * n, cudaMemcpyHostToDevice, m->stream);
    if (e != cudaSuccess) { *err = cudaGetErrorString(e); return B2_ERR_CUDA; }
    cudaEventRecord(m->ev_pin, m->stream);
    m->pin_pending = true;
    const int P = kPhasesPerLayer * m->dev.L;
    for (int i = 0; i < n; i++) {
        StepArgs a{};
        a.tok = m->d_tokens + i;
        a.pos = m->cache_len + i;
        a.p_begin = 0;
        // transformer.go:545-555: logits are needed for the last token only.
        a.p_end = (i == n - 1) ? P + m->dev.n_lm : P;
        a.epoch = ++m->epoch;
        a.skew = m->wait_skew;
        m->wait_skew = 0;
        a.splits = splits_for(m, a.pos);
        int rc = launch_decode(m->dev, a, m->grid, m->stream, err);
        if (rc) return rc;
    }
    m->cache_len += n;
    return B2_OK;
}

int run_traced_step(b2_model* m, int32_t token, unsigned long long* d_trace, std::string* err) {
    if (m->cache_len + 1 > m->cfg.max_seq_len) {
        *err = "context length exceeded";
        return B2_ERR_CONTEXT;
    }
    if (m->pin_pending) cudaEventSynchronize(m->ev_pin);
    m->h_pinned[0] = token;
    cudaMemcpyAsync(m->d_tokens, m->h_pinned, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream);
    cudaEventRecord(m->ev_pin, m->stream);
    m->pin_pending = true;
    StepArgs a{};
    a.tok = m->d_tokens;
    a.pos = m->cache_len;
    a.p_begin = 0;
    a.p_end = kPhasesPerLayer * m->dev.L + m->dev.n_lm;
    a.epoch = ++m->epoch;
    a.splits = splits_for(m, a.pos);
    a.trace = d_trace;
    int rc = launch_decode(m->dev, a, m->grid, m->stream, err);
    if (rc) return rc;
    m->cache_len += 1;
    return B2_OK;
}

int run_greedy(b2_model* m, int32_t first, int n_steps, int32_t eos, int32_t* out_ids, int32_t* n_out,
               std::string* err) {
    *n_out = 0;
    if (n_steps <= 0) return B2_OK;
    if (m->cache_len + n_steps > m->cfg.max_seq_len) {
        *err = "context length exceeded: " + std::to_string(m->cache_len + n_steps) + " > " +
               std::to_string(m->cfg.max_seq_len);
        return B2_ERR_CONTEXT;
    }
    if (m->pin_pending) cudaEventSynchronize(m->ev_pin);
    m->h_pinned[0] = first;
    cudaMemcpyAsync(m->d_tokens, m->h_pinned, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream);
    cudaEventRecord(m->ev_pin, m->stream);
    m->pin_pending = true;
    cudaMemsetAsync(m->d_done, 0, sizeof(int), m->stream);
    const int P = kPhasesPerLayer * m->dev.L;
    for (int i = 0; i < n_steps; i++) {
        StepArgs a{};
        a.tok = (i == 0) ? m->d_tokens : m->dev.token;
        a.pos = m->cache_len + i;
        a.p_begin = 0;
        a.p_end = P + m->dev.n_lm;
        a.epoch = ++m->epoch;
        a.skew = m->wait_skew;
        m->wait_skew = 0;
        a.splits = splits_for(m, a.pos);
        a.out_ids = m->d_out_ids;
        a.step = i;
        a.eos = eos;
        a.done = m->d_done;
        int rc = launch_decode(m->dev, a, m->grid, m->stream, err);
        if (rc) return rc;
    }
    cudaError_t e = cudaMemcpyAsync(m->h_pinned, m->d_out_ids, sizeof(int32_t) * n_steps, cudaMemcpyDeviceToHost,
                                    m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) { *err = cudaGetErrorString(e); return B2_ERR_CUDA; }
    int rc = check_device_status(m, err);
    if (rc) return rc;
    // Step i consumed one token at position cache_len + i and produced ids[i].
    // Predict stops before feeding EOS back (transformer.go:355-357), so the
    // cache holds the positions of `first` and every emitted id but the last.
    int k = 0;
    for (; k < n_steps; k++) {
        if (eos >= 0 && m->h_pinned[k] == eos) break;
        out_ids[k] = m->h_pinned[k];
    }
    *n_out = k;
    m->cache_len += (k < n_steps) ? k + 1 : n_steps;
    return B2_OK;
}

}  // namespace b2

using namespace b2;

namespace {

int fail(std::string* err, int code, const std::string& msg) {
    *err = msg;
    return code;
}

}  // namespace

void b2_free_impl(b2_model* m);

int b2_load_impl(const char* path, const b2_load_opts* opts, b2_model** out, std::string* err) {
    *out = nullptr;
    b2_load_opts o{};
    if (opts) o = *opts;
    const int tp = o.tp_size > 1 ? o.tp_size : 1, rank = tp > 1 ? o.tp_rank : 0;
    if (tp > kMaxTp || rank < 0 || rank >= tp)
        return fail(err, B2_ERR_BAD_ARG, "tensor-parallel degree must be 1 .. 8 and the rank below it");
    auto m = new b2_model();
    auto bail = [&](int code, const std::string& msg) {
        *err = msg;
        b2_free_impl(m);
        return code;
    };
    const auto t_load0 = std::chrono::steady_clock::now();
    int rc = gguf_parse(path, &m->gguf, err);
    if (rc) { std::string e = *err; return bail(rc, e); }
    m->load.parse_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t_load0).count();
    const GgufFile& g = m->gguf;
    b2_config& c = m->cfg;

    // transformer.go:1350-1421 extractConfig.
    c.rms_norm_eps = 1e-5f;
    c.rope_theta = 10000.0f;
    std::string arch;
    if (!g.get_str("general.architecture", &arch)) arch = "llama";
    snprintf(c.arch, sizeof c.arch, "%s", arch.c_str());
    const std::string pre = arch + ".";
    uint32_t u;
    float fv;
    if (g.get_u32(pre + "embedding_length", &u)) c.hidden_size = (int)u;
    if (g.get_u32(pre + "feed_forward_length", &u)) c.intermediate_size = (int)u;
    if (g.get_u32(pre + "block_count", &u)) c.num_layers = (int)u;
    if (g.get_u32(pre + "attention.head_count", &u)) c.num_heads = (int)u;
    c.num_kv_heads = g.get_u32(pre + "attention.head_count_kv", &u) ? (int)u : c.num_heads;
    c.max_seq_len = g.get_u32(pre + "context_length", &u) ? (int)u : 4096;
    if (g.get_f32(pre + "attention.layer_norm_rms_epsilon", &fv)) c.rms_norm_eps = fv;
    if (g.get_f32(pre + "rope.freq_base", &fv)) c.rope_theta = fv;
    c.vocab_size = (int)std::max<int64_t>(0, g.array_len("tokenizer.ggml.tokens"));
    if (c.num_heads > 0 && c.hidden_size > 0) c.head_dim = c.hidden_size / c.num_heads;
    if (c.intermediate_size == 0 && c.hidden_size > 0)
        c.intermediate_size = ((c.hidden_size * 8 / 3) + 255) / 256 * 256;
    if (c.hidden_size == 0) return bail(B2_ERR_FORMAT, "embedding_length not found in GGUF metadata");
    if (c.num_layers == 0) return bail(B2_ERR_FORMAT, "block_count not found in GGUF metadata");
    if (o.num_ctx > 0 && o.num_ctx < c.max_seq_len) c.max_seq_len = o.num_ctx;  // transformer.go:233-235
    c.bos_id = g.get_u32("tokenizer.ggml.bos_token_id", &u) ? (int)u : 1;      // bpe.go:48,105
    c.eos_id = g.get_u32("tokenizer.ggml.eos_token_id", &u) ? (int)u : 2;      // bpe.go:49,108

    const int H = c.hidden_size, FF = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
    const int nh = c.num_heads, nkv = c.num_kv_heads, hd = c.head_dim;
    const int qd = nh * hd, kvd = nkv * hd;
    if (V <= 0) return bail(B2_ERR_FORMAT, "tokenizer.ggml.tokens missing: vocab size unknown");
    if (nkv <= 0 || nh % nkv != 0 || hd < 16 || hd > 256 || (hd & (hd - 1)) || H % 32 || FF % 32 || qd % 32)
        return bail(B2_ERR_UNSUPPORTED_TYPE,
                    "unsupported head geometry (need nh % nkv == 0, head_dim a power of two in [16, 256], widths % 32 == 0)");
    if (c.max_seq_len <= 0) return bail(B2_ERR_FORMAT, "context length is zero");

    // Tensor checks (transformer.go:1143-1306 reads the same names).
    auto need = [&](const std::string& name) -> const GgufTensor* { return g.find(name); };
    const GgufTensor* te = need("token_embd.weight");
    if (!te) return bail(B2_ERR_FORMAT, "token_embd: tensor \"token_embd.weight\" not found");
    const uint32_t qt = te->type;
    if (qt != GGML_Q8_0 && qt != GGML_Q4_0)
        return bail(B2_ERR_UNSUPPORTED_TYPE, "token_embd.weight must be Q8_0 or Q4_0");
    auto check_mat = [&](const std::string& name, int cols, int rows, std::string* e) -> bool {
        const GgufTensor* t = g.find(name);
        if (!t) { *e = "tensor \"" + name + "\" not found"; return false; }
        if (t->type != qt) { *e = name + ": all matrices must share one type (Q8_0 or Q4_0)"; return false; }
        if (t->dims.size() != 2 || (int64_t)t->dims[0] != cols || (int64_t)t->dims[1] != rows) {
            *e = name + ": unexpected shape";
            return false;
        }
        return true;
    };
    std::string e2;
    if (!check_mat("token_embd.weight", H, V, &e2)) return bail(B2_ERR_FORMAT, e2);
    const GgufTensor* ow = g.find("output.weight");
    c.tied_embeddings = ow ? 0 : 1;
    if (ow && !check_mat("output.weight", H, V, &e2)) return bail(B2_ERR_UNSUPPORTED_TYPE, e2);
    if (!g.find("output_norm.weight")) return bail(B2_ERR_FORMAT, "output_norm: tensor \"output_norm.weight\" not found");
    c.has_qkv_bias = g.find("blk.0.attn_q.bias") ? 1 : 0;
    for (int l = 0; l < L; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        if (!check_mat(p + "attn_q.weight", H, qd, &e2) || !check_mat(p + "attn_k.weight", H, kvd, &e2) ||
            !check_mat(p + "attn_v.weight", H, kvd, &e2) || !check_mat(p + "attn_output.weight", qd, H, &e2) ||
            !check_mat(p + "ffn_gate.weight", H, FF, &e2) || !check_mat(p + "ffn_up.weight", H, FF, &e2) ||
            !check_mat(p + "ffn_down.weight", FF, H, &e2))
            return bail(B2_ERR_FORMAT, "layer " + std::to_string(l) + ": " + e2);
        for (const char* nm : {"attn_norm.weight", "ffn_norm.weight"})
            if (!g.find(p + nm)) return bail(B2_ERR_FORMAT, "layer " + std::to_string(l) + ": tensor \"" + p + nm + "\" not found");
    }
    c.weight_type = (int)qt;

    // ---------------------------------------------------------- tensor-parallel shares
    // Megatron layout: q / k / v rows and Wo columns by heads, gate / up rows
    // and down columns by FFN 32-blocks (uneven shares allowed), lm_head rows
    // by vocab; norms replicated.  From here on the dims are this rank's (the
    // whole model when tp == 1).
    if (nh % tp || nkv % tp)
        return bail(B2_ERR_UNSUPPORTED_TYPE, "tensor parallelism needs the heads and KV heads divisible by the degree");
    b2_tp_share sh{};
    if (tp_share(H, nh, nkv, FF, V, tp, rank, &sh) != B2_OK)
        return bail(B2_ERR_UNSUPPORTED_TYPE, "tensor-parallel degree too large for this model");
    const int nhl = nh / tp, nkvl = nkv / tp, qdl = sh.q_rows, kvdl = sh.kv_rows;
    const int FFl = sh.ffn_rows, ff0 = sh.ffn_row0, fb0 = ff0 / 32;
    const int v0 = sh.vocab_row0, Vl = sh.vocab_rows;

    // ---------------------------------------------------------- arena plan
    const size_t bpb = qt == GGML_Q8_0 ? 34 : 18;
    const size_t rb_h = H / 32 * bpb, rb_q = qdl / 32 * bpb, rb_f = FFl / 32 * bpb;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o2 = off;
        off += up256(bytes + 16);
        return o2;
    };
    std::vector<MatGroup> groups;
    // f32 vectors: name, arena offset, first element and count of this rank's share
    struct SmallVec { std::string name; size_t off; int64_t e0, n, total; };
    std::vector<SmallVec> small;
    const int qti = qt == GGML_Q8_0 ? 8 : 2;
    auto take_mat = [&](std::vector<MatPart> parts, int64_t rows, int64_t cols, int64_t half_rows = 0,
                        int64_t cb0 = 0, int64_t nb_src = 0) {
        const size_t o2 = take(tiled_bytes(rows, cols, qti));
        groups.push_back({std::move(parts), o2, rows, cols, half_rows, cb0, nb_src ? nb_src : cols / 32});
        return o2;
    };
    // the embedding lookup needs every row; the lm_head only this rank's vocab share
    const size_t off_embd = take_mat({{"token_embd.weight", 0, V}}, V, H);
    size_t off_out = off_embd;
    if (ow) off_out = take_mat({{"output.weight", v0, Vl}}, Vl, H);
    else if (tp > 1) off_out = take_mat({{"token_embd.weight", v0, Vl}}, Vl, H);
    const size_t off_onorm = take((size_t)H * 4);
    small.push_back({"output_norm.weight", off_onorm, 0, H, H});
    struct LOff { size_t qkv, wo, gu, wd, an, fn, b; };
    std::vector<LOff> lo(L);
    for (int l = 0; l < L; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        lo[l].qkv = take_mat({{p + "attn_q.weight", (int64_t)rank * qdl, qdl},
                              {p + "attn_k.weight", (int64_t)rank * kvdl, kvdl},
                              {p + "attn_v.weight", (int64_t)rank * kvdl, kvdl}}, qdl + 2 * kvdl, H);
        // Wo: this rank's heads' input columns; down: its FFN blocks' columns
        lo[l].wo = take_mat({{p + "attn_output.weight", 0, H}}, H, qdl, 0, (int64_t)rank * qdl / 32, qd / 32);
        // gate and up in one matrix of 2*FFl rows, interleaved 8 rows at a time
        lo[l].gu = take_mat({{p + "ffn_gate.weight", ff0, FFl}, {p + "ffn_up.weight", ff0, FFl}}, 2 * FFl, H, FFl);
        lo[l].wd = take_mat({{p + "ffn_down.weight", 0, H}}, H, FFl, 0, fb0, FF / 32);
        lo[l].an = take((size_t)H * 4);
        small.push_back({p + "attn_norm.weight", lo[l].an, 0, H, H});
        lo[l].fn = take((size_t)H * 4);
        small.push_back({p + "ffn_norm.weight", lo[l].fn, 0, H, H});
        lo[l].b = 0;
        if (c.has_qkv_bias) {
            lo[l].b = take((size_t)(qdl + 2 * kvdl) * 4);
            small.push_back({p + "attn_q.bias", lo[l].b, (int64_t)rank * qdl, qdl, qd});
            small.push_back({p + "attn_k.bias", lo[l].b + (size_t)qdl * 4, (int64_t)rank * kvdl, kvdl, kvd});
            small.push_back({p + "attn_v.bias", lo[l].b + (size_t)(qdl + kvdl) * 4, (int64_t)rank * kvdl, kvdl, kvd});
        }
    }
    const size_t weight_end = off;
    const int S = c.max_seq_len;
    const size_t off_cos = take((size_t)S * (hd / 2) * 4);
    const size_t off_sin = take((size_t)S * (hd / 2) * 4);
    const size_t kv_el = o.kv_fp32 ? 4 : 2;
    const size_t off_k = take((size_t)L * S * kvdl * kv_el);
    const size_t off_v = take((size_t)L * S * kvdl * kv_el);

    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0)
        return bail(B2_ERR_CUDA, "no CUDA device available (the engine has no CPU fallback)");
    if (o.device < 0 || o.device >= dev_count) return bail(B2_ERR_BAD_ARG, "device ordinal out of range");
    m->device = o.device;
    cudaSetDevice(m->device);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
    m->grid = sms;

    const size_t off_plans = take((size_t)m->grid * kPlanSlots * sizeof(TPlan));
    const size_t off_llx1 = take((size_t)H * 8);
    const size_t off_llx2 = take((size_t)H * 8);
    const size_t off_llqkv = take((size_t)(qdl + 2 * kvdl) * 8);
    const size_t off_llpart = take((size_t)nhl * kMaxSplits * (hd + 2) * 8);
    const size_t off_llact = take((size_t)FFl * 8);
    const size_t off_lldnp = take((size_t)2 * kDownSplit * H * 8);
    const size_t off_logits = take((size_t)Vl * 4);
    const size_t off_amkey = take(8);
    const size_t off_tok = take(4);
    const size_t off_amctr = take(4);
    const size_t off_err = take(4);
    const size_t off_toks = take((size_t)S * 4);
    const size_t off_ids = take((size_t)S * 4);
    const size_t off_done = take(4);
    // device sampling: the ids generated so far (repetition penalty), the
    // sampler's scratch, the sampled id
    const size_t off_gen = take((size_t)S * 4);
    const size_t off_sexp = take(sample_scratch_bytes(Vl, 1));
    const size_t off_sout = take(4);
    const size_t off_layers = take(sizeof(LayerDev) * L);
    m->arena_bytes = off;
    // the tensor-parallel exchange buffer: its own allocation, so that its IPC
    // mapping covers nothing else and its layout is the same on every rank
    if (tp > 1) {
        m->xch_bytes = xch_bytes(H, tp);
        if (dev_malloc(&m->xch, m->xch_bytes) != 0) {
            m->xch = nullptr;
            return bail(B2_ERR_OOM, "device allocation of the exchange buffer failed");
        }
        cudaMemset(m->xch, 0, m->xch_bytes);
    }

    if (dev_malloc(&m->arena, m->arena_bytes) != 0) {
        m->arena = nullptr;
        return bail(B2_ERR_OOM, "device allocation of " + std::to_string(m->arena_bytes) + " bytes failed");
    }
    uint8_t* A = static_cast<uint8_t*>(m->arena);
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(B2_ERR_CUDA, "stream creation failed");
    cudaEventCreate(&m->ev0);
    cudaEventCreate(&m->ev1);
    cudaEventCreateWithFlags(&m->ev_pin, cudaEventDisableTiming);
    cudaMemsetAsync(A + weight_end, 0, m->arena_bytes - weight_end, m->stream);
    if (cudaMallocHost(&m->h_pinned, sizeof(int32_t) * std::max(S, 16)) != cudaSuccess ||
        cudaMallocHost(&m->h_logits, sizeof(float) * Vl) != cudaSuccess)
        return bail(B2_ERR_OOM, "pinned host allocation failed");

    // ---------------------------------------------------------- upload
    const auto t_up0 = std::chrono::steady_clock::now();
    bool io_ok = true;
    std::string io_err;
    int64_t up_host_ns = 0;
    uint64_t up_bytes = 0;
    int up_threads = 0;
    bool up_mapped = false;
    int64_t up_setup_ns = 0;
    {
        Uploader up(path, m->stream);
        up_setup_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t_up0).count();
        if (!up.ok()) {
            const bool oom = up.error().find("allocation") != std::string::npos;
            return bail(oom ? B2_ERR_OOM : B2_ERR_IO, up.error());
        }
        // Weight matrices: file -> pinned stages -> raw device buffer, then
        // one repack launch per matrix into the arena (the raw buffer is
        // reused by the next matrix only after its repack, stream order).
        // A column share reads only its window of each row from the file.
        size_t raw_max = 0;
        for (const MatGroup& gr : groups) {
            int64_t r = 0;
            for (const MatPart& pt : gr.parts) r += pt.rows;
            raw_max = std::max(raw_max, (size_t)r * (size_t)(gr.cols / 32) * bpb);
        }
        void* raw = nullptr;
        if (dev_malloc(&raw, raw_max) != 0)
            return bail(B2_ERR_OOM, "device allocation of the " + std::to_string(raw_max) + "-byte upload buffer failed");
        for (const MatGroup& gr : groups) {
            size_t dst = 0;
            int64_t row0 = 0;
            for (const MatPart& pt : gr.parts) {
                const std::string& name = pt.name;
                const GgufTensor* t = g.find(name);
                const uint64_t rb_src = (uint64_t)gr.nb_src * bpb;      // source row bytes
                const uint64_t rb = (uint64_t)(gr.cols / 32) * bpb;     // the share's window of a row
                const uint64_t src = g.data_offset + t->offset + (uint64_t)pt.row0 * rb_src + (uint64_t)gr.cb0 * bpb;
                if (!up.to_device_window(src, rb_src, rb, (uint64_t)pt.rows, static_cast<uint8_t*>(raw) + dst)) {
                    io_ok = false;
                    break;
                }
                dst += (uint64_t)pt.rows * rb;
                // this rank's share of the tensor (b2_dequant_tensor decodes it)
                TensorLoc tl{A + gr.off, t->type, (uint64_t)pt.rows * (uint64_t)gr.cols};
                tl.row0 = row0;
                tl.cols = gr.cols;
                tl.rp = tiled_rows(gr.rows);
                tl.half = gr.half_rows ? (row0 == 0 ? 1 : 2) : 0;
                if (!m->tensors.count(name)) m->tensors[name] = tl;
                row0 += pt.rows;
            }
            if (!io_ok) break;
            const int64_t rp = tiled_rows(gr.rows), nbk = gr.cols / 32;
            const int blocks = (int)std::min<int64_t>((rp * nbk + 255) / 256, 148 * 32);
            repack_kernel<<<blocks, 256, 0, m->stream>>>(static_cast<const uint8_t*>(raw), A + gr.off, gr.rows, rp, nbk,
                                                         qti, gr.half_rows);
        }
        if (!up.finish()) io_ok = false;
        cudaStreamSynchronize(m->stream);
        cudaFree(raw);
        // Small vectors (norm gains, biases) as fp32; F16/BF16 widened on the
        // host exactly as gguf.go:510-536 does.
        std::vector<float> buf;
        for (const SmallVec& sv : small) {
            if (!io_ok) break;
            const GgufTensor* t = g.find(sv.name);
            const size_t n = t ? (size_t)t->elements() : 0;
            buf.assign(sv.n, 0.0f);  // an absent optional bias stays zero (transformer.go:632-646)
            if (t) {
                if ((int64_t)n != sv.total) return bail(B2_ERR_FORMAT, sv.name + ": unexpected length");
                std::vector<uint8_t> rawv(t->bytes());
                if (!up.to_host(g.data_offset + t->offset, rawv.size(), rawv.data())) {
                    io_ok = false;
                    break;
                }
                for (int64_t k = 0; k < sv.n; k++) {
                    const size_t i = (size_t)(sv.e0 + k);
                    if (t->type == GGML_F32) memcpy(&buf[k], &rawv[i * 4], 4);
                    else if (t->type == GGML_F16) buf[k] = f16_to_f32((uint16_t)(rawv[2 * i] | (rawv[2 * i + 1] << 8)));
                    else if (t->type == GGML_BF16) { uint32_t bits = (uint32_t)(rawv[2 * i] | (rawv[2 * i + 1] << 8)) << 16; memcpy(&buf[k], &bits, 4); }
                    else return bail(B2_ERR_UNSUPPORTED_TYPE, sv.name + ": vectors must be F32, F16 or BF16");
                }
                m->tensors[sv.name] = TensorLoc{A + sv.off, GGML_F32, (uint64_t)sv.n};
            }
            cudaMemcpyAsync(A + sv.off, buf.data(), buf.size() * 4, cudaMemcpyHostToDevice, m->stream);
            cudaStreamSynchronize(m->stream);
        }
        cudaStreamSynchronize(m->stream);
        if (!io_ok) io_err = up.error().empty() ? "short read while uploading tensors" : up.error();
        up_host_ns = up.host_ns();
        up_bytes = up.bytes();
        up_threads = up.threads();
        up_mapped = up.mapped();
    }
    if (!io_ok) return bail(B2_ERR_IO, io_err);
    m->load.upload_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t_up0).count();
    m->load.host_copy_ns = up_host_ns;
    m->load.bytes_uploaded = (int64_t)up_bytes;
    m->load.host_threads = up_threads;
    m->load.mapped = up_mapped ? 1 : 0;
    m->load.setup_ns = up_setup_ns;

    // RoPE table with the Go formula (transformer.go:939-942): freq in float64
    // pow rounded to float32, angle in float32, cos/sin in float64 rounded.
    {
        std::vector<float> cs((size_t)S * (hd / 2)), sn((size_t)S * (hd / 2));
        for (int i = 0; i < hd / 2; i++) {
            const float freq = 1.0f / (float)std::pow((double)c.rope_theta, (double)(2 * i) / (double)hd);
            for (int p = 0; p < S; p++) {
                const float ang = (float)p * freq;
                cs[(size_t)p * (hd / 2) + i] = (float)std::cos((double)ang);
                sn[(size_t)p * (hd / 2) + i] = (float)std::sin((double)ang);
            }
        }
        cudaMemcpy(A + off_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(A + off_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    }

    // ---------------------------------------------------------- device view
    ModelDev& d = m->dev;
    d.H = H; d.FF = FFl; d.V = Vl; d.L = L; d.nh = nhl; d.nkv = nkvl; d.hd = hd; d.qd = qdl; d.kvd = kvdl;
    d.max_seq = S;
    d.qtype = (int)qt;
    d.rb_h = (int)rb_h; d.rb_q = (int)rb_q; d.rb_f = (int)rb_f;
    d.eps = c.rms_norm_eps;
    d.kv_fp32 = o.kv_fp32 ? 1 : 0;
    d.Vp = (int)tiled_rows(Vl);
    d.Vemb = V;
    d.Vp_emb = (int)tiled_rows(V);
    d.v_off = v0;
    d.tp = tp;
    d.tp_rank = rank;
    d.nbx = std::max(std::max(H, qdl), FFl) / 32;
    d.tok_embd = A + off_embd;
    d.lm_head = A + off_out;
    d.out_norm = reinterpret_cast<const float*>(A + off_onorm);
    d.rope_cos = reinterpret_cast<const float*>(A + off_cos);
    d.rope_sin = reinterpret_cast<const float*>(A + off_sin);
    d.kcache = A + off_k;
    d.vcache = A + off_v;
    d.ll_x1 = reinterpret_cast<uint2*>(A + off_llx1);
    d.ll_x2 = reinterpret_cast<uint2*>(A + off_llx2);
    d.ll_qkv = reinterpret_cast<uint2*>(A + off_llqkv);
    d.ll_part = reinterpret_cast<uint2*>(A + off_llpart);
    d.ll_act = reinterpret_cast<uint2*>(A + off_llact);
    d.ll_dnp = reinterpret_cast<uint2*>(A + off_lldnp);
    d.logits = reinterpret_cast<float*>(A + off_logits);
    d.am_key = reinterpret_cast<unsigned long long*>(A + off_amkey);
    d.token = reinterpret_cast<int*>(A + off_tok);
    d.am_ctr = reinterpret_cast<unsigned*>(A + off_amctr);
    d.err = reinterpret_cast<int*>(A + off_err);
    m->d_tokens = reinterpret_cast<int*>(A + off_toks);
    m->d_out_ids = reinterpret_cast<int*>(A + off_ids);
    m->d_done = reinterpret_cast<int*>(A + off_done);
    m->d_gen = reinterpret_cast<int*>(A + off_gen);
    m->d_sample_ws = A + off_sexp;
    m->d_sample_out = reinterpret_cast<int*>(A + off_sout);
    m->layers_host.resize(L);
    for (int l = 0; l < L; l++) {
        LayerDev& ld = m->layers_host[l];
        ld.wqkv = A + lo[l].qkv;
        ld.wo = A + lo[l].wo;
        ld.wgu = A + lo[l].gu;
        ld.wd = A + lo[l].wd;
        ld.attn_norm = reinterpret_cast<const float*>(A + lo[l].an);
        ld.ffn_norm = reinterpret_cast<const float*>(A + lo[l].fn);
        ld.bqkv = c.has_qkv_bias ? reinterpret_cast<const float*>(A + lo[l].b) : nullptr;
    }
    m->d_layers = reinterpret_cast<LayerDev*>(A + off_layers);
    cudaMemcpy(m->d_layers, m->layers_host.data(), sizeof(LayerDev) * L, cudaMemcpyHostToDevice);
    d.layers = m->d_layers;

    // Shared-memory geometry: the ring of weight slots plus the QA phase's
    // attention scratch (xs: q, the per-warp partials and merge weights, the
    // new position's words, one K and one Vl tile); the phase inputs go
    // straight into the int8 planes.
    const int kv_es = o.kv_fp32 ? 4 : 2;
    const int tile = std::max(1, std::min(kMaxAttnTile, kAttnTileBytes / (hd * kv_es)));
    const int attn_need = hd + kConsumerWarps * (hd + 2) + 16 + 4 * hd +
                          (tile * (hd * kv_es + 16) + tile * hd * kv_es) / 4;
    const int base_xs = attn_need;
    // q CTAs (nhl per split) must leave at least one CTA for the k / v rows
    const int split_cap = std::max(1, std::min(kMaxSplits, (m->grid - 1) / nhl));
    const int slot = 8192;
    // Outputs one CTA keeps per phase (all K-slices): from the same work plan
    // the kernel uses, over every CTA (and every split count for the QA phase).
    const int qb = tile_qb(qti);
    const int tbb1 = kTileRows * qb + 2 * kTileRows;
    auto ybuf_need = [&](int rows, int nbk, bool own) {
        const int tiles = (int)(tiled_rows(rows) / kTileRows);
        int need = 0;
        for (int cta = 0; cta < m->grid; cta++) {
            const TPlan pl = own ? own_plan(tiles, nbk, tbb1, cta, m->grid, slot, kConsumerWarps)
                                 : tile_plan(tiles, nbk, tbb1, cta, m->grid, slot, kConsumerWarps);
            need = std::max(need, pl.nks * kTileRows * pl.n);
        }
        return need;
    };
    // QA rows: fused with the attention (each q CTA computes its head's q) unless
    // one head's q rows are a large matrix share (> 256 tile-blocks: e.g. head
    // dim 128 over K = 4096), then spread over all CTAs and handed on
    const int qa_dist = (hd / kTileRows) * (H / 32) > 256 ? 1 : 0;
    int qa_need = 0, qa_rows = 0;
    for (int S = 1; S <= split_cap; S++)
        for (int cta = 0; cta < m->grid; cta++) {
            int u0 = 0, n = 0;
            qa_tiles(nhl, hd, qdl, kvdl, S, cta, m->grid, &u0, &n, qa_dist);
            const TPlan pl = tile_plan_range(u0, n, H / 32, tbb1, slot, kConsumerWarps);
            qa_need = std::max(qa_need, pl.nks * kTileRows * pl.n);
            qa_rows = std::max(qa_rows, kTileRows * n);
        }
    // The lm_head's share of a CTA, cut into n_lm consecutive sub-phases: the
    // K-slice results of one sub-phase must fit the phase buffer.
    const int lm_tiles = (int)(tiled_rows(Vl) / kTileRows);
    auto lm_plan = [&](int cta, int sub, int n_lm) {
        const int u0 = (int)((long long)cta * lm_tiles / m->grid);
        const int n = (int)((long long)(cta + 1) * lm_tiles / m->grid) - u0;
        const int a = u0 + (int)((long long)sub * n / n_lm), b = u0 + (int)((long long)(sub + 1) * n / n_lm);
        return tile_plan_range(a, b - a, H / 32, tbb1, slot, kConsumerWarps);
    };
    auto lm_need = [&](int n_lm) {
        int need = 0;
        for (int cta = 0; cta < m->grid; cta++)
            for (int sub = 0; sub < n_lm; sub++) {
                const TPlan pl = lm_plan(cta, sub, n_lm);
                need = std::max(need, pl.nks * kTileRows * pl.n);
            }
        return need;
    };
    // even phases (QA, gate/up, LM head) and odd phases (Wo, down) alternate
    // between two buffers, so the next phase's dots may start before this
    // phase's epilogue ends
    int gu_need = 0;
    for (int cta = 0; cta < m->grid; cta++) {
        const TPlan pl = gu_plan(2 * FFl / kTileRows, H / 32, tbb1, cta, m->grid, slot, kConsumerWarps, H / kTileRows,
                                 kGuOwnerPct);
        gu_need = std::max(gu_need, pl.nks * kTileRows * pl.n);
    }
    const int even_layers = std::max(qa_need, gu_need);
    // the down phase split over K on one GPU when the grid has two CTAs per
    // residual tile and the QA / LM gathers can poll the partials with one
    // thread per quarter-block (dn_split_plan)
    const int h_tiles = H / kTileRows;
    const int dn_split = (tp == 1 && kDownSplit * h_tiles <= m->grid && (FFl / 32) % kDownSplit == 0 &&
                          4 * (H / 32) <= kConsumerWarps * 32) ? kDownSplit : 1;
    int dn_need = 0;
    for (int cta = 0; cta < m->grid; cta++) {
        const TPlan pl = dn_split > 1 ? dn_split_plan(h_tiles, FFl / 32, tbb1, cta, m->grid, slot, kConsumerWarps)
                                      : own_plan(h_tiles, FFl / 32, tbb1, cta, m->grid, slot, kConsumerWarps);
        dn_need = std::max(dn_need, pl.nks * kTileRows * pl.n);
    }
    const int ybuf_odd = (std::max(ybuf_need(H, qdl / 32, true), dn_need) + 31) & ~31;
    const int cfloats = cb_floats(hd);
    const int xs = (base_xs + 31) & ~31, max_splits = split_cap;
    auto ring_slots = [&](int ybuf_total) {
        int n = 0;
        while (n < 32 &&
               smem_offsets(n + 1, slot, xs, ybuf_total, cfloats, std::max(std::max(H, qdl), FFl) / 32, L).total <= 232448u)
            n++;
        return n;
    };
    // fewest lm_head sub-phases that leave 8 ring slots (each one more costs a
    // gather of the final norm's input)
    int n_lm = 1, ybuf_even = 0, ns = 0;
    for (int k = 1; k <= kMaxLmSub; k++) {
        const int ev = (std::max(even_layers, lm_need(k)) + 31) & ~31;
        const int nsk = ring_slots(ev + ybuf_odd);
        if (k == 1 || nsk > ns) {
            n_lm = k;
            ybuf_even = ev;
            ns = nsk;
        }
        if (ns >= 8) break;
    }
    const int ybuf = ybuf_even + ybuf_odd;
    const auto rows_per_cta = [&](int rows) {
        return kTileRows * (int)((tiled_rows(rows) / kTileRows + m->grid - 1) / m->grid);
    };
    if (ns < 2) return bail(B2_ERR_UNSUPPORTED_TYPE, "rows too wide for the shared-memory ring");
    if (rows_per_cta(H) > kMaxOwnRows) return bail(B2_ERR_UNSUPPORTED_TYPE, "hidden size too large for one GPU");
    if (qa_rows > kMaxQkvRows || nhl >= m->grid)
        return bail(B2_ERR_UNSUPPORTED_TYPE, "attention projection too large for one GPU");
    // every CTA's work plans (plan_slot order), so the kernel needs no divisions
    {
        std::vector<TPlan> plans((size_t)m->grid * kPlanSlots, TPlan{0, 0, 1, 1, 1, 0, 0, 0});
        for (int cta = 0; cta < m->grid; cta++) {
            TPlan* pc = plans.data() + (size_t)cta * kPlanSlots;
            pc[plan_slot(PH_WO, 1)] = own_plan(H / kTileRows, qdl / 32, tbb1, cta, m->grid, slot, kConsumerWarps);
            pc[plan_slot(PH_GATEUP, 1)] = gu_plan(2 * FFl / kTileRows, H / 32, tbb1, cta, m->grid, slot, kConsumerWarps,
                                                  H / kTileRows, kGuOwnerPct);
            pc[plan_slot(PH_DOWN, 1)] = dn_split > 1
                ? dn_split_plan(h_tiles, FFl / 32, tbb1, cta, m->grid, slot, kConsumerWarps)
                : own_plan(h_tiles, FFl / 32, tbb1, cta, m->grid, slot, kConsumerWarps);
            for (int sub = 0; sub < n_lm; sub++) pc[plan_slot(PH_LMHEAD, sub)] = lm_plan(cta, sub, n_lm);
            for (int S = 1; S <= kMaxSplits && nhl * S < m->grid; S++) {
                int u0 = 0, n = 0;
                qa_tiles(nhl, hd, qdl, kvdl, S, cta, m->grid, &u0, &n, qa_dist);
                pc[plan_slot(PH_QA, S)] = tile_plan_range(u0, n, H / 32, tbb1, slot, kConsumerWarps);
            }
        }
        cudaMemcpy(A + off_plans, plans.data(), plans.size() * sizeof(TPlan), cudaMemcpyHostToDevice);
        d.plans = reinterpret_cast<const TPlan*>(A + off_plans);
    }
    d.xs_floats = xs;
    d.n_lm = n_lm;
    d.ybuf_floats = ybuf_even;
    d.ybuf_odd = ybuf_odd;
    d.cfloats = cfloats;
    d.attn_tile = tile;
    d.qa_dist = qa_dist;
    d.dn_split = dn_split;
    d.slot_bytes = slot;
    d.nslots = ns;
    m->max_splits = max_splits;

    c.weight_bytes = (int64_t)weight_end;
    c.tp_size = tp;
    c.tp_rank = rank;
    c.vocab_begin = v0;
    c.vocab_local = Vl;
    {
        int64_t layer = (int64_t)(qdl + 2 * kvdl) * rb_h + (int64_t)H * rb_q + (int64_t)2 * FFl * rb_h + (int64_t)H * rb_f;
        int64_t smallb = 4 * (2 * (int64_t)H + (c.has_qkv_bias ? (qdl + 2 * kvdl) : 0));
        c.stream_bytes_per_token = (int64_t)L * (layer + smallb) + (int64_t)Vl * rb_h + 4 * (int64_t)H;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return bail(B2_ERR_CUDA, std::string("CUDA: ") + cudaGetErrorString(e));
    // The prompt path's one-time costs (its workspace, the GEMM scratch, the
    // first launch of each of its kernels) are paid here, by a warm-up pass of
    // up to kWarmTokens BOS tokens at position 0; the cache stays empty (the
    // next prompt overwrites those positions before anything reads them).  On
    // failure the prompt path makes its workspace again when first used.
    const int n_warm = std::min(kWarmTokens, S);
    if (prefill_gemm_ok(m, n_warm)) {
        const std::vector<int32_t> warm(n_warm, c.bos_id >= 0 && c.bos_id < c.vocab_size ? c.bos_id : 0);
        std::string e2;
        if (prefill_gemm(m, warm.data(), n_warm, 0, &e2) != B2_OK) free_prefill_ws(m);
        m->cache_len = 0;
    }
    m->load.total_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t_load0).count();
    *out = m;
    return B2_OK;
}

void b2_free_impl(b2_model* m) {
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    b2::free_prefill_ws(m);
    for (int p = 0; p < kMaxTp; p++)
        if (m->xch_peer[p] && m->xch_peer[p] != m->xch) cudaIpcCloseMemHandle(m->xch_peer[p]);
    if (m->xch) cudaFree(m->xch);
    if (m->arena) cudaFree(m->arena);
    if (m->h_pinned) cudaFreeHost(m->h_pinned);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->ev0) cudaEventDestroy(m->ev0);
    if (m->ev1) cudaEventDestroy(m->ev1);
    if (m->ev_pin) cudaEventDestroy(m->ev_pin);
    if (m->stream) {
        // the per-stream scratch of the products that ran on this stream
        b2_gemm_release(m->device, m->stream);
        b2_mvb_release(m->device, m->stream);
        cudaStreamDestroy(m->stream);
    }
    delete m;
}

namespace b2 {

// Tensor parallelism: the IPC handle of this rank's exchange buffer, and the
// mapping of every rank's buffer (handles in rank order, 64 bytes each).
int b2_tp_handle_impl(const b2_model* m, void* out, std::string* err) {
    if (m->dev.tp < 2 || !m->xch) { *err = "not a tensor-parallel model"; return B2_ERR_BAD_ARG; }
    cudaSetDevice(m->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, m->xch);
    if (e != cudaSuccess) { *err = std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e); return B2_ERR_CUDA; }
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(out, &h, sizeof h);
    return B2_OK;
}

int b2_tp_connect_impl(b2_model* m, const void* handles, std::string* err) {
    const int tp = m->dev.tp;
    if (tp < 2 || !m->xch) { *err = "not a tensor-parallel model"; return B2_ERR_BAD_ARG; }
    if (m->tp_connected) { *err = "already connected"; return B2_ERR_BAD_ARG; }
    cudaSetDevice(m->device);
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int p = 0; p < tp; p++) {
        if (p == m->dev.tp_rank) {
            m->xch_peer[p] = m->xch;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + 64 * p, sizeof h);
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            *err = "cudaIpcOpenMemHandle (rank " + std::to_string(p) + "): " + cudaGetErrorString(e);
            for (int q = 0; q < p; q++)
                if (m->xch_peer[q] && m->xch_peer[q] != m->xch) cudaIpcCloseMemHandle(m->xch_peer[q]);
            for (int q = 0; q < kMaxTp; q++) m->xch_peer[q] = nullptr;
            return B2_ERR_CUDA;
        }
        m->xch_peer[p] = ptr;
    }
    for (int p = 0; p < tp; p++) m->dev.xpeer[p] = static_cast<uint8_t*>(m->xch_peer[p]);
    m->tp_connected = true;
    return B2_OK;
}

}  // namespace b2
