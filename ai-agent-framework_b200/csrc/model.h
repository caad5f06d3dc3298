// Host-side model object behind the b2_model handle.
#pragma once
#include <atomic>
#include <cuda_runtime.h>

#include <map>
#include <random>
#include <string>
#include <vector>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "gguf.h"

namespace b2 {

struct TensorLoc {
    void* dev = nullptr;     // F32: first element; Q8_0 / Q4_0: base of the tiled matrix
    uint32_t type = 0;       // ggml type as resident (F32 for the small vectors)
    uint64_t elements = 0;
    int64_t row0 = 0;        // first row of this tensor in the tiled matrix
    int64_t cols = 0;        // row length (elements)
    int64_t rp = 0;          // rows of the tiled matrix, rounded up to 8
    int half = 0;            // gate/up matrix: 1 = gate rows, 2 = up rows (8-row interleave)
};

// PredictStream state (transformer.go:385-442) for the iterator form.
struct StreamState {
    bool active = false;
    b2_sample_opts opts{};
    std::vector<int32_t> stop;
    std::vector<int32_t> generated;
    int max_gen = 0;
    int emitted = 0;
    bool have_logits = false;  // prefill done, logits of the last token are current
    std::mt19937_64 rng;
};

// Process-wide hook for tests of the failure paths (fault injection on the
// host: a failing device allocation is simulated, nothing faults the GPU):
// the load's device allocation that brings it from 1 to 0 fails.
extern std::atomic<int> g_fail_left;

// The slices a tensor-parallel rank keeps (b2_tp_share_of; the loader's own).
int tp_share(int H, int nh, int nkv, int FF, int V, int tp, int rank, b2_tp_share* s);

}  // namespace b2

struct b2_model {
    int device = 0;
    b2::GgufFile gguf;
    b2_config cfg{};
    b2::ModelDev dev{};
    std::vector<b2::LayerDev> layers_host;
    b2::LayerDev* d_layers = nullptr;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    std::map<std::string, b2::TensorLoc> tensors;
    cudaStream_t stream = nullptr;
    int grid = 0;
    unsigned epoch = 0;
    int max_splits = 1;        // attention splits the merge buffer can hold
    unsigned wait_skew = 0;    // test hook: extra arrivals the next launch waits for
    int cache_len = 0;
    int* d_tokens = nullptr;   // [max_seq] step inputs
    int* d_out_ids = nullptr;  // [max_seq] greedy outputs
    int* d_done = nullptr;     // [1] EOS seen by the device-resident loop
    int* d_gen = nullptr;      // [max_seq] ids sampled so far (device sampling's penalty list)
    unsigned char* d_sample_ws = nullptr;  // device sampler scratch (sample_scratch_bytes(vocab, 1))
    int* d_sample_out = nullptr;  // [1] the sampled id
    int* h_pinned = nullptr;   // pinned staging for token ids (max_seq ints)
    float* h_logits = nullptr; // pinned staging for logits (vocab floats)
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaEvent_t ev_pin = nullptr;  // last H2D copy out of h_pinned
    bool pin_pending = false;
    b2::StreamState st;
    b2_load_stats load{};  // b2_get_load_stats
    // tensor parallelism: this rank's exchange buffer and the peers' (mapped
    // through CUDA IPC by b2_tp_connect; launches need the connection first)
    void* xch = nullptr;
    size_t xch_bytes = 0;
    void* xch_peer[b2::kMaxTp] = {};
    bool tp_connected = false;
    // activations of the tensor-core prompt prefill (a one-row batch over this
    // model's own KV cache), made on the first long prompt
    b2_batch* prefill_ws = nullptr;
};

namespace b2 {

size_t decode_smem_bytes(const ModelDev& m);
// Prompt prefill on the tensor-core GEMM path (decode_batch.cu): tokens at
// positions pos0 .. pos0 + n - 1 of the model's cache, the last token's
// logits and argmax left where the decode kernel leaves them.  prefill_gemm_ok
// says whether the model can take it (one GPU, fp16 cache, supported shapes).
bool prefill_gemm_ok(const b2_model* m, int n);
int prefill_gemm(b2_model* m, const int32_t* tokens, int n, int pos0, std::string* err);
void free_prefill_ws(b2_model* m);
int launch_decode(const ModelDev& m, const StepArgs& a, int grid, cudaStream_t stream, std::string* err);

// Kernel-level entry points (matvec.cu / attention.cu / model.cu).
int launch_dequant(const TensorLoc& t, float* dst, cudaStream_t s);
int launch_embed_mean(const b2_model* m, const int* d_tokens, int n, float* d_out, cudaStream_t s);

// Runs n tokens through the model from the current cache position (prefill
// when n > 1).  Logits of the last token stay in dev.logits and its argmax in
// dev.token.  Returns B2_* codes.
int run_tokens(b2_model* m, const int32_t* host_tokens, int n, std::string* err);
// Tensor parallelism: this rank's exchange-buffer IPC handle (64 bytes), and
// the mapping of all ranks' buffers from their handles in rank order.
int b2_tp_handle_impl(const b2_model* m, void* out, std::string* err);
int b2_tp_connect_impl(b2_model* m, const void* handles, std::string* err);
// Device-resident greedy loop; see b2_decode_greedy.
int run_greedy(b2_model* m, int32_t first, int n_steps, int32_t eos, int32_t* out_ids, int32_t* n_out,
               std::string* err);
int check_device_status(b2_model* m, std::string* err);
// One decode step (with lm_head) that records the phase trace into d_trace.
int run_traced_step(b2_model* m, int32_t token, unsigned long long* d_trace, std::string* err);

}  // namespace b2
