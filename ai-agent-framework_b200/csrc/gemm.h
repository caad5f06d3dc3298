// Entry points of the tensor-core GEMM (gemm_tc.cu): Y = W X over resident
// tiled Q8_0 / Q4_0 weights, X tokens x cols, Y tokens x rows (fp32).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

// Split-K partial products left for the consumer: planes [k][ntok][rows]
// (plane = ntok * rows floats apart); the product is their sum in plane
// order.  With k == 1, p is the caller's y.  The planes live in the GEMM's
// per-stream scratch: the next GEMM on the stream reuses them.
struct GemmParts {
    const float* p = nullptr;
    int k = 0;
    size_t plane = 0;
};

// fp32 X [ntok][cols] (16-byte aligned), converted to fp16 with a
// power-of-two scale per token by the call; Y [ntok][rows] complete.
int b2_tiled_gemm_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols, const float* x,
                       float* y, int ntok, cudaStream_t s, std::string* err);
// X already in the GEMM's input form: xh fp16 bits [b2_gemm_pad_tokens(ntok)]
// [cols] (16-byte aligned; rows past ntok are read but their products are
// discarded), each token's values scaled by 2^e so the largest lies in
// [2^14, 2^15), tok_scale[t] = 2^-e.  parts == nullptr: Y complete in y;
// otherwise the split-K partials are left in *parts (and y receives the
// product only when there is one split).
int b2_tiled_gemm_f16_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols,
                           const void* xh, const float* tok_scale, int ntok, float* y, GemmParts* parts,
                           cudaStream_t s, std::string* err);
// fp32 X as b2_tiled_gemm_impl, the split-K partials left in *parts as
// b2_tiled_gemm_f16_impl leaves them.
int b2_tiled_gemm_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols, const float* x,
                       float* y, int ntok, GemmParts* parts, cudaStream_t s, std::string* err);
// Rows of X the GEMM reads for ntok tokens (ntok rounded up to its N tile).
int b2_gemm_pad_tokens(int ntok);
// The gate or up half of an interleaved gate/up matrix (see gemm_tc.cu).
int b2_tiled_gemm_half_impl(int qtype, const void* base, int64_t rp, int half, int rows, int cols, const float* x,
                            float* y, int ntok, cudaStream_t s, std::string* err);
// Device error flag of stream s's GEMM scratch (0 if none); clears it.
int b2_gemm_status(cudaStream_t s);
// Frees the GEMM scratch of stream s on device dev (a stream about to be
// destroyed; nothing of it may still run).
void b2_gemm_release(int dev, cudaStream_t s);
// Changes whenever stream s's GEMM scratch is reallocated.
unsigned long long b2_gemm_scratch_generation(cudaStream_t s);
