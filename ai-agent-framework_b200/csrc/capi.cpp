// The exported C ABI (include/b2decode.h) and the host side of the engine
// loop: Predict / PredictStream / sample / Embed on token ids.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "gemm.h"
#include "model.h"
#include "sample.h"

int b2_load_impl(const char* path, const b2_load_opts* opts, b2_model** out, std::string* err);
void b2_free_impl(b2_model* m);
int b2_matvec_impl(int qtype, const void* w, const float* x, float* y, int rows, int cols, cudaStream_t s,
                   std::string* err);
int b2_matvec_batch_impl(int qtype, const void* w, const float* x, float* y, int rows, int cols, int nvec,
                         cudaStream_t s, std::string* err);
int b2_tiled_matvec_batch_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols,
                               const float* x, float* y, int nvec, cudaStream_t s, std::string* err);
int b2_batch_create_impl(b2_model* m, int B, b2_batch** out, std::string* err);
void b2_batch_free_impl(b2_batch* bt);
int b2_batch_prefill_impl(b2_batch* bt, int slot, const int32_t* prompt, int n, int32_t* next_out, std::string* err);
int b2_batch_step_impl(b2_batch* bt, const int32_t* tokens, int32_t* next_out, std::string* err);
int b2_batch_logits_impl(const b2_batch* bt, float* out, std::string* err);
int b2_batch_use_graph_impl(b2_batch* bt, int on);
int b2_attention_impl(const float* q, const uint16_t* k, const uint16_t* v, float* out, int batch, int nh, int nkv,
                      int hd, int ctx, cudaStream_t s, std::string* err);
int b2_attention_noalloc_impl(const float* q, const uint16_t* k, const uint16_t* v, float* out, int batch, int nh,
                              int nkv, int hd, int ctx, cudaStream_t s, std::string* err);

namespace {

thread_local std::string g_last_error;

int ret(int code, const std::string& msg = "") {
    if (code != B2_OK) g_last_error = msg.empty() ? "error" : msg;
    return code;
}

bool cuda_ok(cudaError_t e, std::string* err) {
    if (e == cudaSuccess) return true;
    *err = std::string("CUDA: ") + cudaGetErrorString(e);
    return false;
}

int sync_and_check(b2_model* m, std::string* err) {
    if (!cuda_ok(cudaStreamSynchronize(m->stream), err)) return B2_ERR_CUDA;
    return b2::check_device_status(m, err);
}

// transformer.go:981-1036 sample().
int32_t sample_impl(float* logits, int32_t n, const b2_sample_opts& o, const int32_t* generated, int32_t ng, float r) {
    double temp = o.temperature;
    if (temp <= 0) temp = 1.0;
    if (o.repeat_penalty > 1 && ng > 0) {
        const float pen = (float)o.repeat_penalty;
        for (int i = 0; i < ng; i++) {
            const int t = generated[i];
            if (t >= 0 && t < n) {
                if (logits[t] > 0) logits[t] /= pen;
                else logits[t] *= pen;
            }
        }
    }
    auto argmax = [&]() {  // transformer.go:1038-1046
        int best = 0;
        for (int i = 1; i < n; i++)
            if (logits[i] > logits[best]) best = i;
        return best;
    };
    if (temp < 0.01) return argmax();
    for (int i = 0; i < n; i++) logits[i] /= (float)temp;
    struct TP { int idx; float logit; };
    if (o.top_k > 0 && o.top_k < n) {  // topKFilter 1053-1069: only the k-th value matters
        std::vector<float> v(logits, logits + n);
        std::nth_element(v.begin(), v.begin() + (o.top_k - 1), v.end(), std::greater<float>());
        const float thr = v[o.top_k - 1];
        for (int i = 0; i < n; i++)
            if (logits[i] < thr) logits[i] = -INFINITY;
    }
    if (o.top_p > 0 && o.top_p < 1) {  // topPFilter 1071-1114
        std::vector<TP> items(n);
        for (int i = 0; i < n; i++) items[i] = {i, logits[i]};
        std::stable_sort(items.begin(), items.end(), [](const TP& a, const TP& b) { return a.logit > b.logit; });
        std::vector<float> probs(n);
        const float mx = items[0].logit;
        float sum = 0.0f;
        for (int i = 0; i < n; i++) {
            probs[i] = (float)std::exp((double)(items[i].logit - mx));
            sum += probs[i];
        }
        for (int i = 0; i < n; i++) probs[i] /= sum;
        float cum = 0.0f;
        int cut = n - 1;
        const float p = (float)o.top_p;
        for (int i = 0; i < n; i++) {
            cum += probs[i];
            if (cum >= p) { cut = i; break; }
        }
        std::vector<char> keep(n, 0);
        for (int i = 0; i <= cut; i++) keep[items[i].idx] = 1;
        for (int i = 0; i < n; i++)
            if (!keep[i]) logits[i] = -INFINITY;
    }
    // softmax (transformer.go:959-974) and the multinomial draw (1027-1035)
    float mx = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > mx) mx = logits[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        logits[i] = (float)std::exp((double)(logits[i] - mx));
        sum += logits[i];
    }
    for (int i = 0; i < n; i++) logits[i] /= sum;
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        cum += logits[i];
        if (r <= cum) return i;
    }
    return n - 1;
}

b2_sample_opts default_opts() {
    b2_sample_opts o{};
    o.temperature = 0.0;
    o.repeat_penalty = 1.0;
    return o;
}

bool is_greedy(const b2_sample_opts& o) {
    const double t = o.temperature <= 0 ? 1.0 : o.temperature;
    return t < 0.01 && !(o.repeat_penalty > 1);
}

float uniform01(std::mt19937_64& g) { return (float)((g() >> 40) * (1.0 / 16777216.0)); }

// The options as transformer.go:981-1004 decides them, for the device sampler.
void sample_opts_to_args(const b2_sample_opts& o, b2::SampleArgs* a) {
    const double temp = o.temperature <= 0 ? 1.0 : o.temperature;
    a->greedy = temp < 0.01 ? 1 : 0;
    a->temp = (float)temp;
    a->pen = o.repeat_penalty > 1 ? (float)o.repeat_penalty : 0.0f;
    a->top_k = o.top_k;
    a->top_p = (o.top_p > 0 && o.top_p < 1) ? (float)o.top_p : 0.0f;
}

// One engine step's sample, on the device (sample.cu): the logits stay in
// HBM, the ids generated so far are kept in d_gen (the kernel appends the
// one it draws), and 4 bytes come back.
int sample_from_device(b2_model* m, const b2_sample_opts& o, const std::vector<int32_t>& generated, int32_t* next,
                       std::string* err) {
    const int V = m->cfg.vocab_size;
    if (m->cfg.tp_size > 1) {
        *err = "sampling needs the whole vocabulary's logits: greedy only on a tensor-parallel model";
        return B2_ERR_BAD_ARG;
    }
    b2::SampleArgs a{};
    sample_opts_to_args(o, &a);
    a.logits = m->dev.logits;
    a.ld = V;
    a.n = V;
    a.scratch = m->d_sample_ws;
    a.err = m->dev.err;
    a.gen = m->d_gen;
    a.gen_ld = m->dev.max_seq;
    a.gen_append = m->d_gen;
    a.gen_cap = m->dev.max_seq;
    a.out = m->d_sample_out;
    a.ngen[0] = (int)std::min<size_t>(generated.size(), (size_t)m->dev.max_seq);
    a.r[0] = uniform01(m->st.rng);
    int rc = b2::launch_sample(a, 1, m->stream, err);
    if (rc) return rc;
    if (!cuda_ok(cudaMemcpyAsync(m->h_pinned, m->d_sample_out, sizeof(int32_t), cudaMemcpyDeviceToHost, m->stream), err))
        return B2_ERR_CUDA;
    rc = sync_and_check(m, err);
    if (rc) return rc;
    *next = m->h_pinned[0];
    return B2_OK;
}

int read_token(b2_model* m, int32_t* next, std::string* err) {
    if (!cuda_ok(cudaMemcpyAsync(m->h_pinned, m->dev.token, sizeof(int32_t), cudaMemcpyDeviceToHost, m->stream), err))
        return B2_ERR_CUDA;
    int rc = sync_and_check(m, err);
    if (rc) return rc;
    *next = m->h_pinned[0];
    return B2_OK;
}

bool in_stop(const std::vector<int32_t>& stop, int32_t id) {
    return std::find(stop.begin(), stop.end(), id) != stop.end();
}

}  // namespace

extern "C" {

const char* b2_last_error(void) { return g_last_error.c_str(); }

int b2_load(const char* path, const b2_load_opts* opts, b2_model** out) {
    if (!path || !out) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    int rc = b2_load_impl(path, opts, out, &err);
    return ret(rc, err);
}

void b2_free(b2_model* m) { b2_free_impl(m); }

int b2_get_config(const b2_model* m, b2_config* out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out) return ret(B2_ERR_BAD_ARG, "null argument");
    *out = m->cfg;
    return B2_OK;
}

int b2_get_load_stats(const b2_model* m, b2_load_stats* out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out) return ret(B2_ERR_BAD_ARG, "null argument");
    *out = m->load;
    return B2_OK;
}

int b2_reset(b2_model* m) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    m->cache_len = 0;
    m->st = b2::StreamState{};
    return B2_OK;
}

int b2_cache_len(const b2_model* m, int32_t* len_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!len_out) return ret(B2_ERR_BAD_ARG, "null argument");
    *len_out = m->cache_len;
    return B2_OK;
}

int b2_forward(b2_model* m, const int32_t* tokens, int32_t n, float* logits_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!tokens || n <= 0) return ret(B2_ERR_BAD_ARG, "tokens must be non-empty");
    std::string err;
    int rc = b2::run_tokens(m, tokens, n, &err);
    if (rc) return ret(rc, err);
    if (logits_out) {
        const int V = m->cfg.vocab_local;  // the whole vocabulary unless tensor-parallel
        if (!cuda_ok(cudaMemcpyAsync(m->h_logits, m->dev.logits, sizeof(float) * V, cudaMemcpyDeviceToHost, m->stream), &err))
            return ret(B2_ERR_CUDA, err);
        rc = sync_and_check(m, &err);
        if (rc) return ret(rc, err);
        memcpy(logits_out, m->h_logits, sizeof(float) * V);
        return B2_OK;
    }
    rc = sync_and_check(m, &err);
    return ret(rc, err);
}

int b2_forward_argmax(b2_model* m, const int32_t* tokens, int32_t n, int32_t* next_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!tokens || n <= 0 || !next_out) return ret(B2_ERR_BAD_ARG, "tokens must be non-empty");
    std::string err;
    int rc = b2::run_tokens(m, tokens, n, &err);
    if (!rc) rc = read_token(m, next_out, &err);
    return ret(rc, err);
}

int b2_decode_greedy(b2_model* m, int32_t first, int32_t n_steps, int32_t eos, int32_t* out_ids, int32_t* n_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out_ids || !n_out || n_steps < 0) return ret(B2_ERR_BAD_ARG, "bad argument");
    std::string err;
    int rc = b2::run_greedy(m, first, n_steps, eos, out_ids, n_out, &err);
    return ret(rc, err);
}

int32_t b2_sample_logits(float* logits, int32_t n, const b2_sample_opts* opts, const int32_t* generated,
                         int32_t n_generated, float r) {
    if (!logits || n <= 0) return -1;
    b2_sample_opts o = opts ? *opts : default_opts();
    return sample_impl(logits, n, o, generated, generated ? n_generated : 0, r);
}

int64_t b2_sample_scratch_bytes(int32_t n, int32_t rows) {
    if (n <= 0 || rows <= 0 || rows > b2::kSampleMaxRows) return -1;
    return (int64_t)b2::sample_scratch_bytes(n, rows);
}

int b2_sample_device(float* d_logits, int32_t n, int32_t rows, int64_t ld, const b2_sample_opts* opts,
                     const int32_t* d_generated, int64_t gen_ld, const int32_t* n_generated, const float* r,
                     void* d_scratch, int32_t* d_out, void* stream) {
    if (!d_logits || !d_out || !r || !d_scratch || n <= 0 || rows <= 0 || rows > b2::kSampleMaxRows || ld < n)
        return ret(B2_ERR_BAD_ARG, "b2_sample_device: bad argument");
    b2::SampleArgs a{};
    sample_opts_to_args(opts ? *opts : default_opts(), &a);
    a.logits = d_logits;
    a.ld = ld;
    a.n = n;
    a.scratch = static_cast<unsigned char*>(d_scratch);
    a.gen = d_generated;
    a.gen_ld = gen_ld;
    a.out = d_out;
    for (int i = 0; i < rows; i++) {
        a.ngen[i] = (d_generated && n_generated) ? std::max(0, n_generated[i]) : 0;
        a.r[i] = r[i];
    }
    std::string err;
    return ret(b2::launch_sample(a, rows, static_cast<cudaStream_t>(stream), &err), err);
}

int b2_predict(b2_model* m, const int32_t* prompt, int32_t n_prompt, const b2_sample_opts* opts,
               const int32_t* stop_ids, int32_t n_stop, int32_t* out_ids, int32_t max_out, int32_t* n_out,
               b2_timings* timings) {
    // transformer.go:325-382.
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if ((n_prompt > 0 && !prompt) || !out_ids || !n_out || max_out < 0) return ret(B2_ERR_BAD_ARG, "bad argument");
    b2_sample_opts o = opts ? *opts : default_opts();
    const int max_gen = o.num_predict > 0 ? o.num_predict : 256;
    std::vector<int32_t> stop(stop_ids, stop_ids + (stop_ids ? std::max(0, n_stop) : 0));
    std::string err;
    m->cache_len = 0;
    m->st.rng.seed(o.seed);
    std::vector<int32_t> tokens;
    tokens.push_back(m->cfg.bos_id);
    tokens.insert(tokens.end(), prompt, prompt + std::max(0, n_prompt));
    *n_out = 0;
    auto t0 = std::chrono::steady_clock::now();
    int rc = b2::run_tokens(m, tokens.data(), (int)tokens.size(), &err);
    if (rc) return ret(rc, err);
    std::vector<int32_t> generated;
    int32_t next = 0;
    if (is_greedy(o) && stop.empty()) {
        rc = read_token(m, &next, &err);
        if (rc) return ret(rc, err);
        auto t1 = std::chrono::steady_clock::now();
        // Greedy: the rest of the loop runs device-resident.
        if (next != m->cfg.eos_id) {
            generated.push_back(next);
            const int rest = std::min(max_gen, max_out) - 1;
            if (rest > 0) {
                std::vector<int32_t> ids(rest);
                int32_t got = 0;
                rc = b2::run_greedy(m, next, rest, m->cfg.eos_id, ids.data(), &got, &err);
                if (rc) return ret(rc, err);
                generated.insert(generated.end(), ids.begin(), ids.begin() + got);
            }
        }
        auto t2 = std::chrono::steady_clock::now();
        if (timings) {
            timings->prompt_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
            timings->eval_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(t2 - t1).count();
        }
    } else {
        rc = sample_from_device(m, o, generated, &next, &err);
        if (rc) return ret(rc, err);
        auto t1 = std::chrono::steady_clock::now();
        for (int i = 0; i < max_gen && (int)generated.size() < max_out; i++) {
            if (i > 0) {
                rc = b2::run_tokens(m, &generated.back(), 1, &err);
                if (!rc) rc = sample_from_device(m, o, generated, &next, &err);
                if (rc) return ret(rc, err);
            }
            if (next == m->cfg.eos_id || in_stop(stop, next)) break;
            generated.push_back(next);
        }
        auto t2 = std::chrono::steady_clock::now();
        if (timings) {
            timings->prompt_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
            timings->eval_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(t2 - t1).count();
        }
    }
    const int n = std::min<int>((int)generated.size(), max_out);
    std::copy(generated.begin(), generated.begin() + n, out_ids);
    *n_out = n;
    if (timings) {
        timings->prompt_tokens = (int32_t)tokens.size();
        timings->completion_tokens = n;
    }
    return B2_OK;
}

int b2_stream_begin(b2_model* m, const int32_t* prompt, int32_t n_prompt, const b2_sample_opts* opts,
                    const int32_t* stop_ids, int32_t n_stop) {
    // transformer.go:385-402: reset, encode, prepend BOS.
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (n_prompt > 0 && !prompt) return ret(B2_ERR_BAD_ARG, "bad argument");
    b2::StreamState& s = m->st;
    s = b2::StreamState{};
    s.opts = opts ? *opts : default_opts();
    s.rng.seed(s.opts.seed);
    s.max_gen = s.opts.num_predict > 0 ? s.opts.num_predict : 256;
    if (stop_ids && n_stop > 0) s.stop.assign(stop_ids, stop_ids + n_stop);
    m->cache_len = 0;
    std::vector<int32_t> tokens;
    tokens.push_back(m->cfg.bos_id);
    tokens.insert(tokens.end(), prompt, prompt + std::max(0, n_prompt));
    std::string err;
    int rc = b2::run_tokens(m, tokens.data(), (int)tokens.size(), &err);
    if (rc) return ret(rc, err);
    s.active = true;
    s.have_logits = true;
    return B2_OK;
}

int b2_stream_next(b2_model* m, int32_t* token_out, int32_t* done_out) {
    // transformer.go:405-441: one iteration of the streaming loop.
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!token_out || !done_out) return ret(B2_ERR_BAD_ARG, "null argument");
    b2::StreamState& s = m->st;
    *token_out = -1;
    *done_out = 1;
    if (!s.active) return B2_OK;
    std::string err;
    int rc;
    if (s.emitted >= s.max_gen) {
        s.active = false;
        return B2_OK;
    }
    if (!s.have_logits) {
        rc = b2::run_tokens(m, &s.generated.back(), 1, &err);
        if (rc) { s.active = false; return ret(rc, err); }
    }
    int32_t next;
    if (is_greedy(s.opts)) rc = read_token(m, &next, &err);
    else rc = sample_from_device(m, s.opts, s.generated, &next, &err);
    if (rc) { s.active = false; return ret(rc, err); }
    s.have_logits = false;
    if (next == m->cfg.eos_id || in_stop(s.stop, next)) {
        s.active = false;
        return B2_OK;
    }
    s.generated.push_back(next);
    s.emitted++;
    *token_out = next;
    *done_out = 0;
    return B2_OK;
}

int b2_embed(b2_model* m, const int32_t* tokens, int32_t n, float* out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out || n < 0 || (n > 0 && !tokens)) return ret(B2_ERR_BAD_ARG, "bad argument");
    const int H = m->cfg.hidden_size;
    if (n == 0) {  // transformer.go:458-461
        std::fill(out, out + H, 0.0f);
        return B2_OK;
    }
    if (n > m->cfg.max_seq_len) return ret(B2_ERR_BAD_ARG, "too many tokens");
    std::string err;
    if (!cuda_ok(cudaMemcpyAsync(m->d_tokens, tokens, sizeof(int32_t) * n, cudaMemcpyHostToDevice, m->stream), &err))
        return ret(B2_ERR_CUDA, err);
    int rc = b2::launch_embed_mean(m, m->d_tokens, n, m->dev.logits, m->stream);
    if (rc) return ret(rc, "embed launch failed");
    if (!cuda_ok(cudaMemcpyAsync(out, m->dev.logits, sizeof(float) * H, cudaMemcpyDeviceToHost, m->stream), &err))
        return ret(B2_ERR_CUDA, err);
    rc = sync_and_check(m, &err);
    return ret(rc, err);
}

int b2_dequant_tensor(const b2_model* m, const char* name, float* out, int64_t n, int64_t* n_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!name || !out || !n_out) return ret(B2_ERR_BAD_ARG, "null argument");
    auto it = m->tensors.find(name);
    if (it == m->tensors.end()) return ret(B2_ERR_BAD_ARG, std::string("tensor not found: ") + name);
    const b2::TensorLoc& t = it->second;
    if ((int64_t)t.elements > n) return ret(B2_ERR_BAD_ARG, "output buffer too small");
    std::string err;
    float* d = nullptr;
    if (!cuda_ok(cudaMalloc(&d, sizeof(float) * t.elements), &err)) return ret(B2_ERR_OOM, err);
    int rc = b2::launch_dequant(t, d, m->stream);
    if (!rc && !cuda_ok(cudaMemcpyAsync(out, d, sizeof(float) * t.elements, cudaMemcpyDeviceToHost, m->stream), &err))
        rc = B2_ERR_CUDA;
    if (!rc && !cuda_ok(cudaStreamSynchronize(m->stream), &err)) rc = B2_ERR_CUDA;
    cudaFree(d);
    if (rc) return ret(rc, err.empty() ? "dequant failed" : err);
    *n_out = (int64_t)t.elements;
    return B2_OK;
}

int b2_matvec(int32_t qtype, const void* w, const float* x, float* y, int32_t rows, int32_t cols, void* stream) {
    if (!w || !x || !y || rows <= 0 || cols <= 0 || cols % 32) return ret(B2_ERR_BAD_ARG, "bad matvec arguments");
    if (qtype != 8 && qtype != 2) return ret(B2_ERR_UNSUPPORTED_TYPE, "qtype must be 8 (Q8_0) or 2 (Q4_0)");
    std::string err;
    int rc = b2_matvec_impl(qtype, w, x, y, rows, cols, static_cast<cudaStream_t>(stream), &err);
    return ret(rc, err);
}

int b2_matvec_batch(int32_t qtype, const void* w, const float* x, float* y, int32_t rows, int32_t cols,
                    int32_t nvec, void* stream) {
    if (!w || !x || !y || rows <= 0 || cols <= 0) return ret(B2_ERR_BAD_ARG, "bad matvec arguments");
    if (cols % 256) return ret(B2_ERR_BAD_ARG, "batched matvec needs cols to be a multiple of 256");
    if (nvec < 1 || nvec > 16) return ret(B2_ERR_BAD_ARG, "batched matvec takes 1 to 16 vectors");
    if (qtype != 8 && qtype != 2) return ret(B2_ERR_UNSUPPORTED_TYPE, "qtype must be 8 (Q8_0) or 2 (Q4_0)");
    std::string err;
    int rc = b2_matvec_batch_impl(qtype, w, x, y, rows, cols, nvec, static_cast<cudaStream_t>(stream), &err);
    return ret(rc, err);
}

int b2_model_matvec(const b2_model* m, const char* name, const float* x, float* y, int32_t nvec, void* stream) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!name || !x || !y) return ret(B2_ERR_BAD_ARG, "null argument");
    if (nvec < 1 || nvec > 16) return ret(B2_ERR_BAD_ARG, "batched matvec takes 1 to 16 vectors");
    auto it = m->tensors.find(name);
    if (it == m->tensors.end()) return ret(B2_ERR_BAD_ARG, std::string("tensor not found: ") + name);
    const b2::TensorLoc& t = it->second;
    if (t.type != 8 && t.type != 2) return ret(B2_ERR_UNSUPPORTED_TYPE, std::string(name) + " is not a Q8_0 / Q4_0 matrix");
    if (t.half) return ret(B2_ERR_BAD_ARG, std::string(name) + ": gate and up rows are interleaved in the resident matrix");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != m->device)
        return ret(B2_ERR_BAD_ARG, "the model's device must be the current device");
    std::string err;
    const int rows = (int)(t.elements / (uint64_t)t.cols);
    int rc = b2_tiled_matvec_batch_impl((int)t.type, t.dev, t.rp, t.row0, rows, (int)t.cols, x, y, nvec,
                                        stream ? static_cast<cudaStream_t>(stream) : m->stream, &err);
    return ret(rc, err);
}

int b2_model_gemm(const b2_model* m, const char* name, const float* x, float* y, int32_t ntok, void* stream) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!name || !x || !y) return ret(B2_ERR_BAD_ARG, "null argument");
    if (ntok < 1) return ret(B2_ERR_BAD_ARG, "at least one token");
    auto it = m->tensors.find(name);
    if (it == m->tensors.end()) return ret(B2_ERR_BAD_ARG, std::string("tensor not found: ") + name);
    const b2::TensorLoc& t = it->second;
    if (t.type != 8 && t.type != 2) return ret(B2_ERR_UNSUPPORTED_TYPE, std::string(name) + " is not a Q8_0 / Q4_0 matrix");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != m->device)
        return ret(B2_ERR_BAD_ARG, "the model's device must be the current device");
    std::string err;
    const int rows = (int)(t.elements / (uint64_t)t.cols);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m->stream;
    int rc = t.half ? b2_tiled_gemm_half_impl((int)t.type, t.dev, t.rp, t.half, rows, (int)t.cols, x, y, ntok, s, &err)
                    : b2_tiled_gemm_impl((int)t.type, t.dev, t.rp, t.row0, rows, (int)t.cols, x, y, ntok, s, &err);
    return ret(rc, err);
}

int b2_batch_create(b2_model* m, int32_t batch, b2_batch** out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out) return ret(B2_ERR_BAD_ARG, "null argument");
    *out = nullptr;
    std::string err;
    return ret(b2_batch_create_impl(m, batch, out, &err), err);
}

void b2_batch_free(b2_batch* b) { b2_batch_free_impl(b); }

int b2_batch_prefill(b2_batch* b, int32_t slot, const int32_t* prompt, int32_t n, int32_t* next_out) {
    if (!b) return ret(B2_ERR_NOT_LOADED, "no batch");
    if (!prompt || !next_out) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    return ret(b2_batch_prefill_impl(b, slot, prompt, n, next_out, &err), err);
}

int b2_batch_step(b2_batch* b, const int32_t* tokens, int32_t* next_out) {
    if (!b) return ret(B2_ERR_NOT_LOADED, "no batch");
    if (!tokens || !next_out) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    return ret(b2_batch_step_impl(b, tokens, next_out, &err), err);
}

int b2_batch_use_graph(b2_batch* b, int32_t on) {
    if (!b) return ret(B2_ERR_NOT_LOADED, "no batch");
    return b2_batch_use_graph_impl(b, on);
}

int b2_batch_logits(const b2_batch* b, float* out) {
    if (!b) return ret(B2_ERR_NOT_LOADED, "no batch");
    if (!out) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    return ret(b2_batch_logits_impl(b, out, &err), err);
}

int b2_attention_decode(const float* q, const uint16_t* k, const uint16_t* v, float* out, int32_t batch, int32_t nh,
                        int32_t nkv, int32_t hd, int32_t ctx, void* stream) {
    if (!q || !k || !v || !out || batch <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || hd % 8 || ctx <= 0)
        return ret(B2_ERR_BAD_ARG, "bad attention arguments");
    std::string err;
    int rc = b2_attention_impl(q, k, v, out, batch, nh, nkv, hd, ctx, static_cast<cudaStream_t>(stream), &err);
    return ret(rc, err);
}

int b2_trace_step(b2_model* m, int32_t token, int64_t* out_ns, int64_t cap, int32_t* n_phases, int32_t* n_ctas) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!out_ns || !n_phases || !n_ctas) return ret(B2_ERR_BAD_ARG, "null argument");
    const int P = b2::kPhasesPerLayer * m->dev.L + m->dev.n_lm;
    const int64_t need = (int64_t)P * b2::kTraceSlots * m->grid;
    *n_phases = P;
    *n_ctas = m->grid;
    if (cap < need) return ret(B2_ERR_BAD_ARG, "trace buffer too small: need " + std::to_string(need));
    std::string err;
    unsigned long long* d = nullptr;
    if (!cuda_ok(cudaMalloc(&d, need * sizeof(int64_t)), &err)) return ret(B2_ERR_OOM, err);
    cudaMemsetAsync(d, 0, need * sizeof(int64_t), m->stream);
    int rc = b2::run_traced_step(m, token, d, &err);
    if (!rc && !cuda_ok(cudaMemcpyAsync(out_ns, d, need * sizeof(int64_t), cudaMemcpyDeviceToHost, m->stream), &err))
        rc = B2_ERR_CUDA;
    if (!rc) rc = sync_and_check(m, &err);
    cudaFree(d);
    return ret(rc, err);
}

void* b2_stream_handle(const b2_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

int b2_debug_wait_skew(b2_model* m, int32_t skew) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (skew < 0) return ret(B2_ERR_BAD_ARG, "skew must be >= 0");
    m->wait_skew = (unsigned)skew;
    return B2_OK;
}

int b2_tp_share_of(int32_t hidden, int32_t heads, int32_t kv_heads, int32_t ffn, int32_t vocab, int32_t tp,
                   int32_t rank, b2_tp_share* out) {
    if (!out || heads <= 0 || kv_heads <= 0 || hidden <= 0) return ret(B2_ERR_BAD_ARG, "bad model shape");
    const int rc = b2::tp_share(hidden, heads, kv_heads, ffn, vocab, tp, rank, out);
    return ret(rc, rc ? "heads must divide by the degree, the rank lie below it and every share be non-empty" : "");
}

int b2_debug_fail_alloc(int32_t nth) {
    if (nth < 0) return ret(B2_ERR_BAD_ARG, "nth must be >= 0");
    b2::g_fail_left.store(nth);
    return B2_OK;
}

int b2_attention_decode_noalloc(const float* q, const uint16_t* k, const uint16_t* v, float* out, int32_t batch,
                                int32_t nh, int32_t nkv, int32_t hd, int32_t ctx, void* stream) {
    if (!q || !k || !v || !out || batch <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || hd % 8 || ctx <= 0)
        return ret(B2_ERR_BAD_ARG, "bad attention arguments");
    std::string err;
    int rc = b2_attention_noalloc_impl(q, k, v, out, batch, nh, nkv, hd, ctx, static_cast<cudaStream_t>(stream), &err);
    return ret(rc, err);
}

int b2_device_status(b2_model* m) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    std::string err;
    int rc = b2::check_device_status(m, &err);
    return ret(rc, err);
}

int b2_tp_handle(const b2_model* m, void* handle_out) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!handle_out) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    return ret(b2::b2_tp_handle_impl(m, handle_out, &err), err);
}

int b2_tp_connect(b2_model* m, const void* handles) {
    if (!m) return ret(B2_ERR_NOT_LOADED, "no model loaded");
    if (!handles) return ret(B2_ERR_BAD_ARG, "null argument");
    std::string err;
    return ret(b2::b2_tp_connect_impl(m, handles, &err), err);
}

}  // extern "C"
