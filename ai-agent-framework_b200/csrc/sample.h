// Device-side sampling (sample.cu): transformer.go:981-1114 on device logits.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace b2 {

constexpr int kSampleMaxRows = 64;  // sequences per launch

struct SampleArgs {
    float* logits;            // [rows][ld], modified in place (penalty, temperature, filters)
    long long ld;             // row stride of logits (floats)
    int n;                    // vocabulary size
    unsigned char* scratch;   // sample_scratch_bytes(n, rows): the rows' group state, then exp(logit - max) rows
    const int32_t* gen;       // [rows][gen_ld] ids generated so far (may be null when no penalty)
    long long gen_ld;
    int32_t* gen_append;      // when non-null: the sampled id is written at gen_append[row * gen_ld + ngen[row]]
    int gen_cap;              //   if ngen[row] < gen_cap
    int32_t* out;             // [rows] sampled ids
    // options, decided on the host as transformer.go:981-1004 decides them
    int greedy;               // temperature < 0.01: argmax of the penalised logits
    float temp;               // divisor (<= 0 already mapped to 1)
    float pen;                // repetition penalty, applied when > 1
    int top_k;                // applied when 0 < top_k < n
    float top_p;              // applied when 0 < top_p < 1
    int* err;                 // when non-null: B2_ERR_TIMEOUT if a group barrier ran out
    // set by launch_sample
    int rows, group;          // rows, CTAs per row
    long long e_ld;           // floats between the exp rows
    int ngen[kSampleMaxRows];
    float r[kSampleMaxRows];  // the uniform draw of each row, in [0, 1)
};

// Device scratch the sampler needs for rows rows of n logits.
size_t sample_scratch_bytes(int n, int rows);
// A cooperative launch of `group` CTAs per row (the row's vocabulary split
// between them) on stream s, after a reset of the rows' group state.
// Returns a B2_* code (argument and launch errors; the work is asynchronous).
int launch_sample(const SampleArgs& a, int rows, cudaStream_t s, std::string* err);

}  // namespace b2
