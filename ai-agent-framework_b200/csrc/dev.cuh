// Device-side model description and PTX helpers shared by the decode kernels.
#pragma once
#include <stdint.h>
#ifdef __CUDACC__
#include <cuda_fp16.h>
#endif

namespace b2 {

// One decode token is a fixed sequence of phases; phase p of layer l is
// 5*l + k with k below, and the lm_head phase is 5*L.  Each phase is a unit of
// work split over all CTAs; a phase may start only when the previous one is
// complete everywhere (grid barrier), except that weight bytes of later phases
// stream into shared memory ahead of time.
enum PhaseKind : int {
    PH_QKV = 0,     // rmsnorm(x) -> [Wq|Wk|Wv] rows, bias, RoPE, KV-cache append
    PH_ATTN = 1,    // GQA attention of the new query over the cache, split over context
    PH_WO = 2,      // attn_out -> Wo rows, residual add into x
    PH_GATEUP = 3,  // rmsnorm(x) -> gate & up rows, SwiGLU -> act
    PH_DOWN = 4,    // act -> Wd rows, residual add into x
    PH_LMHEAD = 5,  // rmsnorm(x) -> lm_head rows, logits + argmax
    PH_MATVEC = 6,  // plain y = W x (kernel-level entry point)
};

constexpr int kPhasesPerLayer = 5;
constexpr int kConsumerWarps = 8;
constexpr int kThreads = 32 * (kConsumerWarps + 1);  // warp 0 = producer
constexpr int kBarStride = 32;                        // counters 128 B apart
constexpr int kMaxSplits = 16;                        // attention context splits per KV head

struct LayerDev {
    const uint8_t* wqkv;  // [(qd + 2*kvd) rows][rb_h]: Wq rows, then Wk, then Wv
    const uint8_t* wo;    // [H rows][rb_q]
    const uint8_t* wgu;   // [2*FF rows][rb_h]: gate rows, then up rows
    const uint8_t* wd;    // [H rows][rb_f]
    const float* attn_norm;
    const float* ffn_norm;
    const float* bqkv;    // [qd + 2*kvd] or null
};

struct ModelDev {
    int H, FF, V, L, nh, nkv, hd, qd, kvd, max_seq;
    int qtype;            // 8 = Q8_0, 2 = Q4_0 (ggml layout)
    int rb_h, rb_q, rb_f; // row bytes for inputs of width H, qd, FF
    float eps;
    int kv_fp32;
    int slot_bytes, nslots, xs_floats;  // shared-memory ring geometry
    const uint8_t* tok_embd;  // [V rows][rb_h]
    const uint8_t* lm_head;   // tok_embd when tied
    const float* out_norm;
    const float* rope_cos;    // [max_seq][hd/2]
    const float* rope_sin;
    void* kcache;             // [L][max_seq][kvd] fp16 or fp32
    void* vcache;
    const LayerDev* layers;   // device array [L]
    // activations and scratch (device)
    float* x;                 // [H] residual stream
    float* q;                 // [qd]
    float* attn;              // [qd] merged attention output
    float* part;              // [nh][kMaxSplits][hd + 2] split partials (o, m, l)
    unsigned* head_ctr;       // [nkv * kBarStride] split arrival counters
    float* act;               // [FF]
    float* logits;            // [V]
    float* best_val;          // [grid] argmax partials
    int* best_idx;
    int* token;               // [1] last argmax
    unsigned* bar;            // [(5L+1) * kBarStride] phase arrival counters
    int* err;                 // device error flag (B2_ERR_* codes)
};

// Per-launch arguments of the decode kernel.
struct StepArgs {
    const int* tok;      // device pointer to this step's input token
    int pos;             // cache position written by this step
    int p_begin, p_end;  // phase range to run
    unsigned epoch;      // arrival target multiplier for this launch
    unsigned skew;       // added to every wait target (test hook; 0 normally)
    int splits;          // attention context splits per KV head
    int* out_ids;        // argmax also written to out_ids[step] when non-null
    int step;
    int eos;             // with done: an argmax equal to eos sets *done
    int* done;           // device flag; a launch that finds it set does no work
    // PH_MATVEC only
    const uint8_t* mv_w;
    const float* mv_x;
    float* mv_y;
    int mv_rows, mv_cols, mv_rb;
};

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// 1-D bulk copy global -> shared (TMA), completing on an mbarrier.  src, dst
// and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_acq_rel_add(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Four signed bytes -> four exact floats.  (b ^ 0x80) placed in the low
// mantissa byte of 2^23 gives the float 2^23 + b + 128; subtracting
// 2^23 + 128 leaves b exactly.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}

// Four nibbles (0..15, one per byte) -> four exact floats of (nibble - 8).
__device__ __forceinline__ void u4x4_to_f32(uint32_t w, float* f) {
    f[0] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)) - 8388616.0f;
    f[1] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)) - 8388616.0f;
    f[2] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)) - 8388616.0f;
    f[3] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)) - 8388616.0f;
}

#endif  // __CUDACC__

}  // namespace b2
