/*
 * b2decode — B200 (sm_100a) decode engine for GGUF Q8_0 / Q4_0 LLaMA/Qwen2
 * models, a drop-in for the per-token forward pass of the Local-LLM-Pure-Go
 * engine.
 *
 * C ABI: plain pointers and sizes, no C++ or CUDA types.  Every function that
 * can fail returns 0 on success or a negative B2_ERR_* code; the message of
 * the last failure on the calling thread is b2_last_error().  No exception or
 * abort crosses the ABI.  The library owns all device memory of a model.  Host
 * buffers passed in are read or written only during the call.  Calls on one
 * b2_model must be serialised by the caller (the Go engine holds one
 * sync.Mutex per engine, transformer.go:96).
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   Local-LLM-Pure-Go/internal/engine/engine.go:15-39          Engine interface
 *   Local-LLM-Pure-Go/internal/engine/native/transformer/transformer.go
 *   Local-LLM-Pure-Go/internal/engine/native/gguf/gguf.go
 */
#ifndef B2DECODE_H
#define B2DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2_OK 0
#define B2_ERR_IO (-1)               /* file missing or short read */
#define B2_ERR_FORMAT (-2)           /* bad magic/version, truncated or inconsistent GGUF */
#define B2_ERR_UNSUPPORTED_TYPE (-3) /* tensor type the engine cannot run */
#define B2_ERR_OOM (-4)              /* device or host allocation failed */
#define B2_ERR_CUDA (-5)             /* CUDA runtime error */
#define B2_ERR_NCCL (-6)             /* collective failure */
#define B2_ERR_TIMEOUT (-7)          /* a bounded device-side wait gave up */
#define B2_ERR_BAD_ARG (-8)          /* invalid argument */
#define B2_ERR_CONTEXT (-9)          /* position beyond the KV-cache capacity */
#define B2_ERR_NOT_LOADED (-10)      /* model handle is NULL or unloaded */

typedef struct b2_model b2_model;
typedef struct b2_batch b2_batch;

/* engine.go:42-47 LoadOptions, plus device placement. */
typedef struct {
    int32_t num_ctx;    /* LoadOptions.NumCtx: caps context_length when > 0 (transformer.go:233-235) */
    int32_t device;     /* CUDA device ordinal */
    int32_t kv_fp32;    /* 0: fp16 KV cache (default); 1: fp32 KV cache as in the Go engine */
    int32_t tp_size;    /* LoadOptions.NumGPU: tensor-parallel degree (0 or 1: one GPU; up to 8) */
    int32_t tp_rank;    /* this process's rank, 0 .. tp_size - 1 (one process per GPU) */
    int32_t reserved2;
} b2_load_opts;

/* transformer.go:33-46 ModelConfig, plus what loadWeights derives. */
typedef struct {
    char arch[32];
    int32_t vocab_size;
    int32_t hidden_size;
    int32_t intermediate_size;
    int32_t num_layers;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t max_seq_len;       /* min(context_length, num_ctx) */
    float rms_norm_eps;
    float rope_theta;
    int32_t tied_embeddings;   /* 1: lm_head reads token_embd (transformer.go:551-554) */
    int32_t has_qkv_bias;
    int32_t weight_type;       /* ggml type of the layer matrices: 8 = Q8_0, 2 = Q4_0 */
    int32_t bos_id;            /* tokenizer.ggml.bos_token_id (bpe.go:48,105) */
    int32_t eos_id;            /* tokenizer.ggml.eos_token_id (bpe.go:49,108) */
    int64_t weight_bytes;      /* bytes of weights resident in HBM (this rank's) */
    int64_t stream_bytes_per_token; /* algorithmic HBM bytes one B=1 decode token reads (this rank's) */
    int32_t tp_size;           /* tensor-parallel degree and this rank */
    int32_t tp_rank;
    int32_t vocab_begin;       /* this rank's share of the lm_head rows: logits of */
    int32_t vocab_local;       /* vocab ids vocab_begin .. vocab_begin + vocab_local - 1 */
} b2_config;

/* Real phase timings (the Go engine reports fixed 1/3 and 2/3 splits,
 * transformer.go:379-380). */
typedef struct {
    int64_t prompt_ns;
    int64_t eval_ns;
    int32_t prompt_tokens;
    int32_t completion_tokens;
} b2_timings;

/* domain.Options (internal/domain/types.go:142-160) fields used by sample. */
typedef struct {
    double temperature;     /* <= 0 means 1.0; greedy when < 0.01 (transformer.go:982-1004) */
    int32_t top_k;
    double top_p;
    double repeat_penalty;  /* applied when > 1 */
    int32_t num_predict;    /* <= 0 means 256 */
    uint64_t seed;          /* seed of the engine's uniform generator */
} b2_sample_opts;

/* ---- model lifecycle (engine.go Load/Unload/ModelInfo/IsLoaded) ---- */

/* transformer.go:215-310 Engine.Load: parse the GGUF, extract the config,
 * copy every Q8_0/Q4_0 block verbatim into one HBM arena (no host dequant),
 * allocate the KV cache.  opts may be NULL. */
int b2_load(const char* gguf_path, const b2_load_opts* opts, b2_model** out);
/* transformer.go:312-322 Unload. NULL is ignored. */
void b2_free(b2_model* m);
int b2_get_config(const b2_model* m, b2_config* out);

/* Where b2_load's time went (transformer.go:1122-1335 loadWeights reads and
 * dequantises on the host; here the blocks go to HBM as they are): the file
 * is memory-mapped, a pool of host threads copies each 32 MB range into one
 * of four pinned stages while the previous stages' cudaMemcpyAsync run, and
 * the device retiles each matrix. */
typedef struct {
    int64_t total_ns;        /* the whole b2_load */
    int64_t parse_ns;        /* GGUF header, metadata and tensor infos */
    int64_t upload_ns;       /* weight and vector bytes to HBM, retiling included */
    int64_t host_copy_ns;    /* of upload_ns: host threads filling the pinned stages */
    int64_t bytes_uploaded;  /* weight bytes sent through the stages */
    int32_t host_threads;
    int32_t mapped;          /* 1: memory-mapped file; 0: pread */
    int64_t setup_ns;        /* of upload_ns: mapping the file, pinned stages, thread pool */
} b2_load_stats;
int b2_get_load_stats(const b2_model* m, b2_load_stats* out);
/* Message of the last failure on this thread ("" if none). */
const char* b2_last_error(void);

/* ---- forward pass ---- */

/* transformer.go:742-749 resetCache. */
int b2_reset(b2_model* m);
/* Number of cached positions (kvCache.Len, transformer.go:88-92). */
int b2_cache_len(const b2_model* m, int32_t* len_out);

/* transformer.go:519-557 forward: run n tokens (prefill when n > 1) from the
 * current cache position; write the vocab_size logits of the last token to
 * logits_out (may be NULL). */
int b2_forward(b2_model* m, const int32_t* tokens, int32_t n, float* logits_out);
/* forward followed by argmax (transformer.go:1038-1046, first maximum wins)
 * computed on the device. */
int b2_forward_argmax(b2_model* m, const int32_t* tokens, int32_t n, int32_t* next_out);
/* Device-resident greedy loop: feed `first`, then each argmax, n_steps times;
 * stop after emitting eos (eos < 0 disables the stop).  out_ids receives up to
 * n_steps ids, *n_out how many (the eos id itself is not emitted, as in
 * Predict, transformer.go:355-357). */
int b2_decode_greedy(b2_model* m, int32_t first, int32_t n_steps, int32_t eos, int32_t* out_ids,
                     int32_t* n_out);

/* ---- engine loop (engine.go Predict / PredictStream on token ids) ---- */

/* transformer.go:325-382 Predict: reset, prepend BOS, prefill, then up to
 * num_predict steps of forward + sample, stopping at EOS or at any id in
 * stop_ids (the token-id form of isStopToken, transformer.go:1430-1437).
 * Greedy runs device-resident; otherwise each step's logits are sampled on
 * the device by the b2_sample_device sampler (transformer.go:981-1114), with
 * the engine's seeded uniforms, and only the id comes back. */
int b2_predict(b2_model* m, const int32_t* prompt, int32_t n_prompt, const b2_sample_opts* opts,
               const int32_t* stop_ids, int32_t n_stop, int32_t* out_ids, int32_t max_out, int32_t* n_out,
               b2_timings* timings);
/* transformer.go:385-442 PredictStream as an iterator: begin resets and
 * prefills; each next call yields one token id or done=1 (EOS, stop id or
 * num_predict reached). */
int b2_stream_begin(b2_model* m, const int32_t* prompt, int32_t n_prompt, const b2_sample_opts* opts,
                    const int32_t* stop_ids, int32_t n_stop);
int b2_stream_next(b2_model* m, int32_t* token_out, int32_t* done_out);

/* transformer.go:981-1036 sample() on host logits (modified in place), with
 * the caller's uniform r in [0,1) for the multinomial draw. */
int32_t b2_sample_logits(float* logits, int32_t n, const b2_sample_opts* opts, const int32_t* generated,
                         int32_t n_generated, float r);
/* transformer.go:981-1114 sample() on the DEVICE, the sampler b2_predict and
 * b2_stream_next use: rows (<= 64) sequences, row i's logits at
 * d_logits[i * ld .. + n) in device memory (modified in place: penalty,
 * temperature, filtered entries), its generated ids at d_generated[i * gen_ld
 * .. + n_generated[i]) (device; may be NULL without a penalty), its uniform
 * r[i] in [0,1) (host array).  Top-K and top-P are radix selections (no
 * sort) by a group of CTAs per row; the masses are summed exactly in fixed
 * point, so the id equals the host sampler's except where r or top_p lies
 * within the host's float rounding of a cumulative boundary.  d_scratch:
 * b2_sample_scratch_bytes(n, rows) bytes of device memory.  The ids are
 * written to d_out[rows] (device; -1 if a group barrier of the launch ran
 * out); asynchronous on stream (a cudaStream_t; NULL = the legacy default
 * stream). */
int64_t b2_sample_scratch_bytes(int32_t n, int32_t rows);
int b2_sample_device(float* d_logits, int32_t n, int32_t rows, int64_t ld, const b2_sample_opts* opts,
                     const int32_t* d_generated, int64_t gen_ld, const int32_t* n_generated, const float* r,
                     void* d_scratch, int32_t* d_out, void* stream);

/* transformer.go:445-490 Embed: mean of the token_embd rows of the ids,
 * L2-normalised, written to out[hidden_size]. */
int b2_embed(b2_model* m, const int32_t* tokens, int32_t n, float* out);

/* ---- debug / kernel-level entry points ---- */

/* gguf.go:491-508 Dequantize of one named tensor, decoded on the device from
 * the resident blocks (Q4_0 in the ggml element order).  n = capacity of out
 * in floats; returns 0 and writes *n_out elements.  On a tensor-parallel rank
 * a sharded tensor yields this rank's share (its rows, or its columns of each
 * row, in the order of the GGUF tensor). */
int b2_dequant_tensor(const b2_model* m, const char* name, float* out, int64_t n, int64_t* n_out);

/* transformer.go:810-865 matVecMulQ8Chunk over all rows, on the device:
 * y[r] = sum_b d_b * sum_j q_bj * x[32b+j].  w, x, y are DEVICE pointers
 * (GGUF block rows, fp32).  qtype 8 = Q8_0, 2 = Q4_0 (ggml layout).
 * stream is a cudaStream_t (NULL = legacy default stream). */
int b2_matvec(int32_t qtype, const void* w, const float* x, float* y, int32_t rows, int32_t cols,
              void* stream);

/* transformer.go:810-892 (matVecMulQ8Chunk / matVecMulQ8Pooled) for nvec
 * vectors at once, reading the matrix from HBM once: y[v][r] = sum_b d_rb *
 * sum_j q_rbj * x[v][32b+j] for v < nvec.  x [nvec][cols] and y [nvec][rows]
 * fp32, w GGUF block rows (16-byte aligned); all DEVICE pointers.
 * 1 <= nvec <= 16 (vectors 8..15 share the pass over w with 0..7); cols a
 * multiple of 256.  qtype 8 = Q8_0, 2 = Q4_0.  Uses a
 * scratch buffer per (device, stream), grown with cudaMalloc when a call
 * needs more; calls on one stream run in order, calls on different streams
 * use different buffers. */
int b2_matvec_batch(int32_t qtype, const void* w, const float* x, float* y, int32_t rows, int32_t cols,
                    int32_t nvec, void* stream);
/* The same batched dots (transformer.go:810-892 for nvec vectors) over a
 * weight matrix of the loaded model, read from its resident tiled blocks:
 * y[v][r] = sum_j W[r][j] * x[v][j] for the tensor `name` (this rank's share
 * under tensor parallelism, rows and columns as b2_dequant_tensor returns
 * them).  x [nvec][cols], y [nvec][rows] fp32 DEVICE pointers, 1 <= nvec <=
 * 16; the model's device must be current.  stream NULL = the model's own
 * stream.  The gate and up matrices are stored interleaved and are rejected.
 * Shares the per-(device, stream) scratch of b2_matvec_batch. */
int b2_model_matvec(const b2_model* m, const char* name, const float* x, float* y, int32_t nvec, void* stream);
/* The same product for any number of tokens on the tensor cores (tcgen05,
 * TMA-staged tiles): Y = W X for the tensor `name`, x [ntok][cols], y
 * [ntok][rows] fp32 DEVICE pointers, ntok >= 1, cols a multiple of 64.  The
 * weights are decoded to fp16 in shared memory (d * q rounded once) and the
 * activations converted to fp16 with a power-of-two scale per token; products
 * accumulate in fp32.  This is the dense contraction of a prompt's prefill:
 * the batched counterpart of the C++ sibling engine's
 * Local-LLM/include/tensor.h:354-387 mat_mat_mul_tensor (Transformer::
 * forward_batch, Local-LLM/src/transformer.cpp:540-575).  Asynchronous on
 * `stream` (NULL = the model's stream), with a per-(device, stream) scratch
 * grown by cudaMalloc when a call needs more.  The gate and up matrices,
 * stored interleaved, are computed whole and their half gathered (a buffer
 * of ntok x 2 x rows floats allocated on the stream for the call). */
int b2_model_gemm(const b2_model* m, const char* name, const float* x, float* y, int32_t ntok, void* stream);

/* transformer.go:663-685 attention of one query token per sequence over an
 * fp16 KV cache, split over the context with a log-sum-exp merge.
 * q [batch][nh*hd] fp32; k, v [batch][ctx][nkv*hd] fp16 (binary16 bits);
 * out [batch][nh*hd] fp32.  DEVICE pointers.  Asynchronous on `stream`; the
 * split partials live in a scratch kept per (device, stream), grown by
 * cudaMalloc when a call needs more and held until the process exits, so
 * calls on different streams may overlap (a caller that cycles through many
 * short-lived streams holds one buffer per stream it used). */
int b2_attention_decode(const float* q, const uint16_t* k, const uint16_t* v, float* out, int32_t batch,
                        int32_t nh, int32_t nkv, int32_t hd, int32_t ctx, void* stream);

/* b2_attention_decode without any device allocation, for callers that cannot
 * call cudaMalloc: a serving process whose HBM is already fully reserved by
 * its own pools (weights, KV cache), or a per-token path that cannot afford
 * the device-wide synchronisation a cudaMalloc/cudaFree pair can cause.  The
 * split partials use a fixed 2 MiB device array inside the library (held by
 * every GPU that loads it until the process exits); the caller still passes
 * q, k, v and out.  Limit: batch * nh * (hd + 2) <= 524288 floats, larger
 * sizes fail with B2_ERR_BAD_ARG.  The first call on a device looks up the
 * array's device address; make that first call before any stream capture.
 * The address is cached per device for the life of the process: after a
 * caller resets a device (cudaDeviceReset) this entry point must not be
 * called on it again.  All calls share the array, so calls whose kernels
 * overlap on the GPU race.  No counterpart in the reference. */
int b2_attention_decode_noalloc(const float* q, const uint16_t* k, const uint16_t* v, float* out, int32_t batch,
                                int32_t nh, int32_t nkv, int32_t hd, int32_t ctx, void* stream);

/* ---- batched greedy decode (config: Llama-3-8B at batch 16) ----
 *
 * Up to 16 sequences, each with a KV-cache slot of its own (max_seq = the
 * model's num_ctx, fp16), advance one token per b2_batch_step together, each
 * at its own position, so every weight byte is read once per step for all of
 * them: the forward of transformer.go:519-739 and argmax 1038-1046 for B
 * sequences at a time.  b2_batch_prefill runs a slot's prompt into the slot
 * (the model's own single-sequence cache is not touched); next_out is the
 * argmax after the prompt.  b2_batch_step
 * feeds tokens[B] (one per slot, every slot) and writes the B argmax ids;
 * b2_batch_logits copies the logits of the last forward of the batch,
 * [B][vocab_size]: the B rows of the last b2_batch_step, or, after a
 * b2_batch_prefill, the prompt's last token in row 0.  A prompt runs in
 * chunks of up to 256 of its tokens, each one pass over the weights on the
 * tensor cores (b2_model_gemm's product) with the chunk's attention over the
 * slot's cache.  Needs a
 * single-GPU model with the fp16 cache; the model's device must be current.
 * Every batch of a model runs on the model's stream and shares its scratch,
 * so calls on the batches of one model, like calls on the model itself, must
 * be serialised by the caller; batches of different models are independent.
 * A batch is used only while its model is loaded; b2_batch_free may come
 * before or after b2_free of the model.
 * No single counterpart in the reference (its engine runs one sequence). */
int b2_batch_create(b2_model* m, int32_t batch, b2_batch** out);
void b2_batch_free(b2_batch* b);
int b2_batch_prefill(b2_batch* b, int32_t slot, const int32_t* prompt, int32_t n, int32_t* next_out);
int b2_batch_step(b2_batch* b, const int32_t* tokens, int32_t* next_out);
int b2_batch_logits(const b2_batch* b, float* out);
/* on != 0: replay each step's launches from a CUDA graph, captured after the
 * first step that runs with the switch on (and again after the batched
 * matvec's shared scratch has moved); a capture that fails leaves the batch
 * stepping eagerly.  Off by default. */
int b2_batch_use_graph(b2_batch* b, int32_t on);

/* ---- tensor parallelism (engine.go LoadOptions.NumGPU; no counterpart in the
 * Go engine, which runs on CPU cores) ----
 *
 * One process per GPU loads the same GGUF with b2_load_opts.tp_size = N and
 * its own tp_rank: it keeps its heads' q / k / v rows and Wo columns, its
 * share of the FFN (gate / up rows, down columns, at 32-block granularity)
 * and of the lm_head vocab rows.  After Wo and after down every rank writes
 * its partial sums into every rank's exchange buffer over NVLink (peer
 * stores) and sums all ranks' partials in rank order, so the residual stream
 * is identical on every rank; the argmax is taken over all ranks' vocab
 * shares the same way.  Before the first forward call, every rank passes the
 * 64-byte handle from b2_tp_handle to the others (any host channel) and calls
 * b2_tp_connect with all N handles in rank order.  Every rank must then make
 * the same sequence of forward calls with the same tokens.  b2_forward's
 * logits_out receives this rank's vocab share (b2_config.vocab_begin /
 * vocab_local); sampling other than greedy is not available. */
int b2_tp_handle(const b2_model* m, void* handle_out);
int b2_tp_connect(b2_model* m, const void* handles);

/* The slices of the GGUF tensors that rank `rank` of a tp-way tensor-
 * parallel model keeps, as b2_load computes them (host arithmetic, no GPU):
 * query heads and KV heads evenly (rows of attn_q / attn_k / attn_v and
 * their biases, input columns of attn_output), the FFN at 32-element block
 * granularity (rows of ffn_gate / ffn_up, input columns of ffn_down; uneven
 * shares allowed), the lm_head by vocab rows.  Fails with B2_ERR_BAD_ARG
 * when the heads do not divide by tp or a share would be empty.  No
 * reference counterpart (the Go engine runs on CPU cores). */
typedef struct {
    int32_t q_row0, q_rows;          /* attn_q rows; attn_output input columns */
    int32_t kv_row0, kv_rows;        /* attn_k / attn_v rows */
    int32_t ffn_row0, ffn_rows;      /* ffn_gate / ffn_up rows; ffn_down input columns */
    int32_t vocab_row0, vocab_rows;  /* lm_head (output or token_embd) rows */
} b2_tp_share;
int b2_tp_share_of(int32_t hidden, int32_t heads, int32_t kv_heads, int32_t ffn, int32_t vocab, int32_t tp,
                   int32_t rank, b2_tp_share* out);

/* Device-side error code of the last launch on this model (B2_ERR_TIMEOUT
 * after a bounded wait gave up), 0 if none; clears it. */
int b2_device_status(b2_model* m);

/* Phase timeline of one decode step (profiling): runs `token` at the current
 * position like b2_forward_argmax and records globaltimer stamps (ns) for
 * every phase, slot and CTA into out_ns[phase][13][cta]: slots 0-3 = consumer
 * wait start, wait done, input staged, work done; 4-5 = producer first and
 * last weight copy issued (0 when the phase has no weights); 6 = total ns the
 * CTA's consumer warps spent waiting for weight chunks, 7 = how many of those
 * waits took longer than 256 ns; 8 = ns the producer waited for free ring
 * slots, 9 = weight chunks it issued; 10 = consumer rows loop done; 11 = total
 * ns the consumer warps spent in tile dot products; 12 = epilogue constants
 * ready.  cap is the
 * capacity of out_ns in elements.  No reference counterpart (the Go engine
 * only logs durations, transformer.go:305-308). */
int b2_trace_step(b2_model* m, int32_t token, int64_t* out_ns, int64_t cap, int32_t* n_phases, int32_t* n_ctas);

/* The cudaStream_t every launch of this model is issued on (for timing with
 * CUDA events on the launching stream).  No reference counterpart. */
void* b2_stream_handle(const b2_model* m);

/* Test hook for failure detection without a GPU fault: the next decode launch
 * waits for `skew` more grid arrivals than will ever come, so its bounded
 * waits run out (about 2 s) and it reports B2_ERR_TIMEOUT through
 * b2_device_status while the context stays usable.  0 disables.  No
 * reference counterpart. */
int b2_debug_wait_skew(b2_model* m, int32_t skew);

/* Test hook for allocation failures: the nth device allocation that
 * b2_load makes from now on (1 = the next one) fails as if cudaMalloc had
 * returned an error, so the caller sees B2_ERR_OOM and can check that the
 * failed load freed everything it had taken.  The hook disarms itself after
 * firing; 0 disarms it.  Process-wide.  No reference counterpart (the Go
 * engine's allocations cannot fail short of a runtime panic). */
int b2_debug_fail_alloc(int32_t nth);

#ifdef __cplusplus
}
#endif
#endif
