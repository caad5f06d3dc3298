/*
 * goref — CPU restatement of the Local-LLM-Pure-Go decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity oracle for the B200
 * decode engine: tests, the smoke check and the bench's CPU-baseline leg call
 * it as the checker.  The product never links it.
 *
 * Every function follows the Go source it names (paths relative to the
 * reference project root), operation for operation, in float32 with the same
 * left-to-right accumulation order and the same float64 round-trips for
 * transcendentals.  Build with -ffp-contract=off: Go on amd64 never fuses
 * x*y+z, so neither may this code.
 */
#ifndef GOREF_H
#define GOREF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct goref_model goref_model;

/* transformer.go:33-46 ModelConfig (plus the fields loadWeights derives). */
typedef struct {
    char arch[32];
    int32_t vocab_size;
    int32_t hidden_size;
    int32_t intermediate_size;
    int32_t num_layers;
    int32_t num_heads;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t max_seq_len;
    float rms_norm_eps;
    float rope_theta;
    int32_t tied;          /* 1 when lm_head runs over token_embd (transformer.go:549-554) */
    int32_t weight_type;   /* ggml type of blk.0.attn_q.weight */
    int32_t bos_id;        /* bpe.go:48,105 */
    int32_t eos_id;        /* bpe.go:49,108 */
} goref_config;

/* Oracle modes.
 * GOREF_MODE_GO: exactly the Go engine.  2-D weights always go through the
 *   Q8_0 matvec (transformer.go:627-629), a non-Q8_0 output.weight is dropped
 *   (transformer.go:1180-1189) and Q4_0 dequant is the interleaved order of
 *   gguf.go:598-609.  Only meaningful for Q8_0 models.
 * GOREF_MODE_GGML_Q4: the same Go forward math with a correct Q4_0 path in
 *   the ggml block layout (low nibble -> element j, high nibble -> j+16,
 *   value (q-8)*d), applied to matvecs, output.weight and dequant.  For Q8_0
 *   models the two modes are identical. */
#define GOREF_MODE_GO 0
#define GOREF_MODE_GGML_Q4 1

/* transformer.go:215-310 Engine.Load (parse, extractConfig, loadWeights,
 * KV cache).  num_ctx > 0 caps MaxSeqLen (transformer.go:233-235).
 * n_threads <= 0 means one worker per online CPU (transformer.go:210).
 * Returns NULL on failure; goref_last_error() says why. */
goref_model* goref_load(const char* path, int32_t num_ctx, int32_t n_threads, int32_t mode);
void goref_free(goref_model* m);
int goref_get_config(const goref_model* m, goref_config* out);
const char* goref_last_error(void);

/* transformer.go:742-749 resetCache. */
void goref_reset(goref_model* m);
/* Number of cached positions (kvCache.Len). */
int32_t goref_cache_len(const goref_model* m);

/* transformer.go:519-557 forward.  Writes vocab_size logits of the last
 * token.  Returns 0, or -1 when the context is exhausted (the Go engine
 * panics there: scores[:cachedLen] past MaxSeqLen, transformer.go:667). */
int goref_forward(goref_model* m, const int32_t* tokens, int32_t n, float* logits);

/* Layer-truncated forward for spot checks: returns the hidden state after the
 * final RMSNorm instead of logits (hidden_size floats). */
int goref_forward_hidden(goref_model* m, const int32_t* tokens, int32_t n, float* hidden);

/* transformer.go:1038-1046 argmax (first maximum wins). */
int32_t goref_argmax(const float* x, int32_t n);

/* transformer.go:981-1036 sample.  The multinomial draw uses the caller's
 * uniform r in [0,1) instead of the unseeded global rand.Float32 (line 1027).
 * logits is modified in place, as in Go. */
int32_t goref_sample(float* logits, int32_t n, double temperature, int32_t top_k,
                     double top_p, double repeat_penalty, const int32_t* generated,
                     int32_t n_generated, float r);

/* transformer.go:325-382 Predict on token ids: prepend BOS, prefill, then up
 * to max_gen steps of forward + sample, stopping at EOS.  stop_ids stands in
 * for the text stop strings (isStopToken, transformer.go:1430-1437).  uniforms
 * supplies one r per step for non-greedy sampling (may be NULL when greedy). */
int goref_predict(goref_model* m, const int32_t* prompt, int32_t n_prompt, int32_t max_gen,
                  double temperature, int32_t top_k, double top_p, double repeat_penalty,
                  const int32_t* stop_ids, int32_t n_stop, const float* uniforms,
                  int32_t* out_ids, int32_t* n_out);

/* gguf.go:491-508 Dequantize of one named tensor, read from the file
 * (gguf.go:282-300).  mode selects the Q4_0 order (see above).  n is the
 * capacity of out in floats.  Returns element count or -1. */
int64_t goref_dequant_tensor(const char* path, const char* name, int32_t mode, float* out, int64_t n);

/* Kernel-level restatements (row-major GGUF block layout). */
/* transformer.go:810-865 matVecMulQ8Chunk over all rows. */
void goref_matvec_q8_0(const uint8_t* w, const float* x, float* y, int32_t rows, int32_t cols);
/* The same loop with ggml Q4_0 blocks (18 bytes: f16 d, 16 nibble bytes). */
void goref_matvec_q4_0(const uint8_t* w, const float* x, float* y, int32_t rows, int32_t cols);
/* transformer.go:767-784 matVecMulChunk (fp32 weights, 4 accumulators). */
void goref_matvec_f32(const float* w, const float* x, float* y, int32_t rows, int32_t cols);
/* Threaded versions (transformer.go:868-892): serial below 512 rows. */
void goref_matvec_q8_0_mt(goref_model* m, const uint8_t* w, const float* x, float* y, int32_t rows, int32_t cols);

/* transformer.go:663-685: attention of one query token over ctx cached
 * positions.  q [nh*hd]; k, v [ctx][nkv*hd] fp32; out [nh*hd] (overwritten). */
void goref_attention(const float* q, const float* k, const float* v, float* out,
                     int32_t nh, int32_t nkv, int32_t hd, int32_t ctx);

/* transformer.go:922-932, 936-951, 954-956, 959-974, 895-919. */
void goref_rmsnorm(float* x, const float* w, int32_t n, float eps);
void goref_rope(float* x, int32_t head_dim, int32_t num_heads, int32_t pos, float theta);
float goref_silu(float x);
void goref_softmax(float* x, int32_t n);
float goref_f16_to_f32(uint16_t h);

/* A worker pool handle without a model, for timing matvecs alone. */
goref_model* goref_pool_only(int32_t n_threads);
int32_t goref_num_threads(const goref_model* m);

#ifdef __cplusplus
}
#endif
#endif
