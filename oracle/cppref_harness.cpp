// cppref — C entry points over the reference's C++ sibling engine
// (Local-LLM/src/transformer.cpp), compiled from the reference's own source
// files into oracle/_ref/.  TEST INFRASTRUCTURE ONLY: a second, independently
// written CPU implementation of the same LLaMA/Qwen2 decode math, used to
// cross-check the goref oracle within a tolerance and as an optional CPU
// baseline.  Its summation order and float-precision RoPE differ from the Go
// engine, so it agrees with goref to rounding, not bit for bit.
#include <iostream>
#include <sstream>
#include <cstring>
#include "transformer.h"
#include "dequantize.h"

namespace {
struct Silence {  // the engine logs to stdout; keep test output clean
    std::ostringstream sink;  // constructed before it is installed
    std::streambuf* old;
    Silence() : old(std::cout.rdbuf(sink.rdbuf())) {}
    ~Silence() { std::cout.rdbuf(old); }
};
}

extern "C" {

void* cppref_load(const char* path) {
    Silence s;
    auto* t = new localllm::Transformer();
    if (!t->load_model(path)) { delete t; return nullptr; }
    return t;
}

void cppref_free(void* h) { delete static_cast<localllm::Transformer*>(h); }

int cppref_vocab(void* h) { return static_cast<localllm::Transformer*>(h)->config().vocab_size; }

void cppref_reset(void* h) { static_cast<localllm::Transformer*>(h)->reset(); }

// Transformer::forward(token, pos) (Local-LLM/src/transformer.cpp:354-369).
int cppref_forward(void* h, int token, int pos, float* logits, int n) {
    auto* t = static_cast<localllm::Transformer*>(h);
    const std::vector<float>& l = t->forward(token, pos);
    if ((int)l.size() > n) return -1;
    std::memcpy(logits, l.data(), l.size() * sizeof(float));
    return (int)l.size();
}

// Local-LLM/src/dequantize.cpp dequantize_q4_0 / dequantize_q8_0.
void cppref_dequant_q4_0(const void* src, float* dst, long long n) { localllm::dequantize_q4_0(src, dst, n); }
void cppref_dequant_q8_0(const void* src, float* dst, long long n) { localllm::dequantize_q8_0(src, dst, n); }
// Local-LLM/src/dequantize.cpp vec_dot_q8_0 / vec_dot_q4_0 (one row).
float cppref_vec_dot_q8_0(const void* src, const float* y, long long n) { return localllm::vec_dot_q8_0(src, y, n); }
float cppref_vec_dot_q4_0(const void* src, const float* y, long long n) { return localllm::vec_dot_q4_0(src, y, n); }

}
