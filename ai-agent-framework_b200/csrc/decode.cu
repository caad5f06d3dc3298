// The decode step: one cooperative, persistent kernel per token.
//
// Replaces transformer.go:519-739 (forward / transformerLayer / selfAttention /
// feedForward) and the Q8_0 matvec of transformer.go:810-892 for B = 1.
//
// Layout of one CTA (one per SM):
//   warp 0, lane 0   producer: walks the static schedule of weight rows this
//                    CTA owns in every phase of the launch and streams them
//                    with 1-D TMA bulk copies into a ring of shared-memory
//                    slots.  Weights never depend on activations, so the
//                    producer runs ahead across phases, limited by the ring.
//   warps 1..12      consumers, per phase:
//                    1. stage: gather the phase input from the previous
//                       phase's LL words (the poll is the load) into shared
//                       memory, with RMSNorm / embedding decode / attention
//                       split merge fused in; the phase constants (norm gains,
//                       QKV bias, RoPE row) arrive by cp.async during the poll;
//                    2. rows: each warp dequantises its chunks of the CTA's
//                       weight rows in registers and leaves the fp32 dot
//                       products in shared memory (ybuf); nothing else is live
//                       in this loop, so it runs without register spills;
//                    3. epilogue, one thread per output: bias + RoPE + KV
//                       append, SwiGLU, residual add, logits + argmax, and the
//                       LL stores that hand the outputs to the next phase.
//                    The attention phase instead runs one (query head,
//                    context split) per CTA over K/V tiles that cp.async
//                    copies into shared memory while the CTA polls for q.
// Each CTA keeps the residual-stream rows it owns (the same rows in every Wo
// and down phase) in shared memory.  Every wait is bounded (globaltimer) and
// reports B2_ERR_TIMEOUT through the device error flag instead of hanging.
#include <cuda_runtime.h>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "model.h"

namespace b2 {

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;      // 2 s for any consumer wait
constexpr uint64_t kProducerLimitNs = 8000000000ull;  // producer slot waits outlast consumer polls
constexpr int kConsumerThreads = 32 * kConsumerWarps;

struct Geom {
    int kind;
    int layer;
    const uint8_t* w;
    const uint8_t* w2;  // up rows (PH_GATEUP)
    int rb;
    int cols;
    int units;
    int rpu;  // rows per unit
};

__device__ __forceinline__ Geom phase_geom(const ModelDev& m, const StepArgs& a, int p) {
    Geom g{};
    if (a.mv_w) {
        g.kind = PH_MATVEC;
        g.w = a.mv_w;
        g.rb = a.mv_rb;
        g.cols = a.mv_cols;
        g.units = a.mv_rows;
        g.rpu = 1;
        return g;
    }
    if (p == kPhasesPerLayer * m.L) {
        g.kind = PH_LMHEAD;
        g.layer = m.L;
        g.w = m.lm_head;
        g.rb = m.rb_h;
        g.cols = m.H;
        g.units = m.V;
        g.rpu = 1;
        return g;
    }
    g.layer = p / kPhasesPerLayer;
    g.kind = p % kPhasesPerLayer;
    const LayerDev& L = m.layers[g.layer];
    switch (g.kind) {
        case PH_QKV:
            g.w = L.wqkv; g.rb = m.rb_h; g.cols = m.H; g.units = (m.qd + 2 * m.kvd) / 2; g.rpu = 2;
            break;
        case PH_ATTN:
            g.units = m.nh * a.splits;
            break;
        case PH_WO:
            g.w = L.wo; g.rb = m.rb_q; g.cols = m.qd; g.units = m.H; g.rpu = 1;
            break;
        case PH_GATEUP:
            g.w = L.wgu; g.w2 = L.wgu + (size_t)m.FF * m.rb_h; g.rb = m.rb_h; g.cols = m.H; g.units = m.FF;
            g.rpu = 1;
            break;
        default:  // PH_DOWN
            g.w = L.wd; g.rb = m.rb_f; g.cols = m.FF; g.units = m.H; g.rpu = 1;
            break;
    }
    return g;
}

// Static split of a phase's units over the grid and of a CTA's share into
// chunks that fit one ring slot.  Producer and consumers evaluate the same
// function, so they agree on every chunk without communicating.
struct Split {
    int u0, n, cu, nchunks;
};

__device__ __forceinline__ Split cta_split(const Geom& g, int cta, int grid, int slot_bytes) {
    Split s;
    s.u0 = (int)((long long)cta * g.units / grid);
    int u1 = (int)((long long)(cta + 1) * g.units / grid);
    s.n = u1 - s.u0;
    if (g.w == nullptr || s.n <= 0) {
        s.cu = 1;
        s.nchunks = 0;
        return s;
    }
    int per_unit = g.rpu * g.rb * (g.w2 ? 2 : 1);
    int max_units = (slot_bytes - (g.w2 ? 192 : 32)) / per_unit;
    int spread = (s.n + kConsumerWarps - 1) / kConsumerWarps;
    s.cu = max(1, min(max_units, spread));
    s.nchunks = (s.n + s.cu - 1) / s.cu;
    return s;
}

__device__ __forceinline__ void set_err(int* err, int code) { atomicCAS(err, 0, code); }

// Producer: bounded wait for a free ring slot.
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kProducerLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Consumer: bounded wait for chunk gidx to land.  *pstop is the index of the
// first chunk the producer did not issue (it stops early only after an
// error); such chunks are skipped instead of waited for, and every chunk that
// was issued is waited for, so no bulk copy is left in flight at exit.
__device__ __forceinline__ bool chunk_wait(uint64_t* bar, uint32_t parity, unsigned gidx, const volatile unsigned* pstop,
                                           int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (gidx >= *pstop) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ unsigned ll_tag(unsigned epoch, int layer) { return epoch * 256u + (unsigned)layer + 1u; }

// Result of a gather: whether it completed, and the sum of squares of the
// gathered values (for RMSNorm) when asked for.
struct GatherRes {
    float ss;
    int ok;
};

// Gathers LL words src[0 .. n) (n even, src 16-byte aligned) once every word
// carries `tag` and stores the values into shared memory at byte address
// dst: value i goes to float i (us == 0) or to the dot-loop layout of the
// phase input (us values per lane unit, nu units; see xs_index).  Each
// consumer thread polls its own words with 16-byte loads, up to 4 in flight;
// a word whose tag is stale is simply read again.  Bounded: gives up (ok = 0,
// error flag set) after kWaitLimitNs or when another CTA already reported an
// error.  Not inlined: its polling state would otherwise add to the register
// peak of the whole kernel at every one of its call sites.
__device__ __noinline__ GatherRes ll_gather_s(const uint2* src, int n, unsigned tag, int* err, uint32_t dst, int us,
                                              int nu, int want_ss) {
    const int ct = threadIdx.x - 32;
    const int n2 = n >> 1;
    const int ul = us == 32 ? 5 : 4;
    uint64_t t0 = 0;
    float ss = 0.0f;
    for (int base = 0; base < n2; base += kConsumerThreads * 4) {
        uint4 v[4];
        for (;;) {
            bool ok = true;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int i = base + ct + k * kConsumerThreads;
                if (i < n2) {
                    v[k] = ll_load2(src + 2 * i);
                    ok &= (v[k].y == tag) & (v[k].w == tag);
                }
            }
            if (ok) break;
            __nanosleep(64);  // back off: thousands of pollers share these lines
            const uint64_t now = global_ns();
            if (t0 == 0) t0 = now;
            if (now - t0 > kWaitLimitNs) {
                set_err(err, B2_ERR_TIMEOUT);
                return GatherRes{ss, 0};
            }
            if (*(volatile int*)err) return GatherRes{ss, 0};
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int i = base + ct + k * kConsumerThreads;
            if (i < n2) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int j = 2 * i + e;
                    const float val = __uint_as_float(e ? v[k].z : v[k].x);
                    int idx = j;
                    if (us) {
                        const int u = j >> ul, r = j & (us - 1);
                        idx = ((r >> 2) * nu + u) * 4 + (r & 3);
                    }
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst + 4u * (uint32_t)idx), "f"(val) : "memory");
                    if (want_ss) ss += val * val;
                }
            }
        }
    }
    return GatherRes{ss, 1};
}

// Shared-memory layout of the phase input: element j of lane unit u (US
// values per unit) lives in float4 column (j % US) / 4; columns are stored
// one after another, so lane u's k-th float4 is xs4[k * NU + u] and a warp
// reads 32 consecutive float4 per instruction (no bank conflicts).
template <int US>
__device__ __forceinline__ int xs_index(int j, int nu) {
    const int u = j / US, r = j % US;
    return ((r >> 2) * nu + u) * 4 + (r & 3);
}

// ---------------------------------------------------------------------------
// dequantising dot products: two rows against the staged input vector
// ---------------------------------------------------------------------------

// Four consecutive 32-bit words of row data starting at a 2-byte aligned
// shared address (realigned with funnel shifts).
__device__ __forceinline__ void load16(const uint8_t* q, uint32_t* d) {
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(qa & 3) * 8;
    const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3], w4 = wp[4];
    d[0] = __funnelshift_r(w0, w1, sh);
    d[1] = __funnelshift_r(w1, w2, sh);
    d[2] = __funnelshift_r(w2, w3, sh);
    d[3] = __funnelshift_r(w3, w4, sh);
}

// 16 int8 (4 words) . 16 floats -> fp32x2 partial (short dependency chains).
__device__ __forceinline__ unsigned long long q8_dot16(const uint32_t* d, const float4* x) {
    const unsigned long long sub = f2_pack(-8388736.0f, -8388736.0f);
    unsigned long long acc[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        unsigned long long p01, p23;
        bytes_to_f2(d[k] ^ 0x80808080u, sub, p01, p23);
        acc[k] = f2_mul(p01, f2_pack(x[k].x, x[k].y));
        acc[k] = f2_fma(p23, f2_pack(x[k].z, x[k].w), acc[k]);
    }
    return f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
}

// Q8_0: lane unit = half a block (16 values); block = [f16 d][32 x int8].
__device__ __forceinline__ void dot2_q8(const uint8_t* r0, const uint8_t* r1, bool two, const float* xs, int cols,
                                        int lane, float& out0, float& out1) {
    const int nu = cols >> 4;
    const float4* xv = reinterpret_cast<const float4*>(xs);
    unsigned long long a0 = f2_pack(0.0f, 0.0f), a1 = a0;
    for (int u = lane; u < nu; u += 32) {
        const int b = u >> 1, h = u & 1;
        float4 x[4];
#pragma unroll
        for (int k = 0; k < 4; k++) x[k] = xv[k * nu + u];
        uint32_t d[4];
        const uint8_t* p0 = r0 + 34 * b;
        load16(p0 + 2 + 16 * h, d);
        const float s0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p0));
        a0 = f2_fma(f2_pack(s0, s0), q8_dot16(d, x), a0);
        if (two) {
            const uint8_t* p1 = r1 + 34 * b;
            load16(p1 + 2 + 16 * h, d);
            const float s1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p1));
            a1 = f2_fma(f2_pack(s1, s1), q8_dot16(d, x), a1);
        }
    }
    const float2 f0 = f2_unpack(a0), f1 = f2_unpack(a1);
    out0 = f0.x + f0.y;
    out1 = f1.x + f1.y;
}

// One Q4_0 block (16 bytes: low nibble = element j, high nibble = j + 16)
// dotted with 32 floats (x[0..7] = elements 0..31).
__device__ __forceinline__ unsigned long long q4_dot32(const uint32_t* d, const float4* x) {
    const unsigned long long sub = f2_pack(-8388616.0f, -8388616.0f);
    unsigned long long acc[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        unsigned long long l01, l23, h01, h23;
        bytes_to_f2(d[k] & 0x0F0F0F0Fu, sub, l01, l23);
        bytes_to_f2((d[k] >> 4) & 0x0F0F0F0Fu, sub, h01, h23);
        acc[k] = f2_mul(l01, f2_pack(x[k].x, x[k].y));
        acc[k] = f2_fma(l23, f2_pack(x[k].z, x[k].w), acc[k]);
        acc[k] = f2_fma(h01, f2_pack(x[4 + k].x, x[4 + k].y), acc[k]);
        acc[k] = f2_fma(h23, f2_pack(x[4 + k].z, x[4 + k].w), acc[k]);
    }
    return f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
}

// Q4_0: lane unit = one block (32 values).
__device__ __forceinline__ void dot2_q4(const uint8_t* r0, const uint8_t* r1, bool two, const float* xs, int cols,
                                        int lane, float& out0, float& out1) {
    const int nu = cols >> 5;
    const float4* xv = reinterpret_cast<const float4*>(xs);
    unsigned long long a0 = f2_pack(0.0f, 0.0f), a1 = a0;
    for (int u = lane; u < nu; u += 32) {
        float4 x[8];
#pragma unroll
        for (int k = 0; k < 8; k++) x[k] = xv[k * nu + u];
        uint32_t d[4];
        const uint8_t* p0 = r0 + 18 * u;
        load16(p0 + 2, d);
        const float s0 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p0));
        a0 = f2_fma(f2_pack(s0, s0), q4_dot32(d, x), a0);
        if (two) {
            const uint8_t* p1 = r1 + 18 * u;
            load16(p1 + 2, d);
            const float s1 = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p1));
            a1 = f2_fma(f2_pack(s1, s1), q4_dot32(d, x), a1);
        }
    }
    const float2 f0 = f2_unpack(a0), f1 = f2_unpack(a1);
    out0 = f0.x + f0.y;
    out1 = f1.x + f1.y;
}

// transformer.go:525-531 + gguf.go:540-613: element j of token_embd row tok,
// decoded from its block (out-of-range ids embed to zero).
__device__ __forceinline__ float embed_elem(const ModelDev& m, int tok, int j) {
    if (tok < 0 || tok >= m.V) return 0.0f;
    const uint8_t* row = m.tok_embd + (size_t)tok * m.rb_h;
    const int b = j >> 5, e = j & 31;
    if (m.qtype == 8) {
        const uint8_t* p = row + 34 * b;
        float d = f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
        return d * (float)(int8_t)p[2 + e];
    }
    const uint8_t* p = row + 18 * b;
    float d = f16_bits_to_f32((uint16_t)(p[0] | (p[1] << 8)));
    uint8_t byte = p[2 + (e & 15)];
    int nib = (e < 16) ? (byte & 15) : (byte >> 4);
    return d * (float)(nib - 8);
}

struct Best {
    float v;
    int i;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// Sums a0 over the warp into lane 0 and a1 into lane 16 (6 shuffles).
__device__ __forceinline__ float warp_sum2(float a0, float a1, int lane) {
    const float t0 = __shfl_xor_sync(0xffffffffu, a0, 16);
    const float t1 = __shfl_xor_sync(0xffffffffu, a1, 16);
    float v = (lane & 16) ? a1 + t1 : a0 + t0;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide (consumer threads) max / sum through warp shuffles and red[].
__device__ __forceinline__ float block_max(float v, float* red, int cw) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[cw] = v;
    named_bar_sync(1, kConsumerThreads);
    float r = red[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; w++) r = fmaxf(r, red[w]);
    named_bar_sync(1, kConsumerThreads);
    return r;
}
__device__ __forceinline__ float block_sum(float v, float* red, int cw) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[cw] = v;
    named_bar_sync(1, kConsumerThreads);
    float r = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; w++) r += red[w];
    named_bar_sync(1, kConsumerThreads);
    return r;
}

// Offsets in the constant buffer (floats).
__device__ __forceinline__ int cb_bias(const ModelDev& m) { return m.H; }
__device__ __forceinline__ int cb_cos(const ModelDev& m) { return m.H + kMaxQkvRows + 4; }
__device__ __forceinline__ int cb_sin(const ModelDev& m) { return m.H + kMaxQkvRows + 4 + m.hd / 2; }

// The attention phase, transformer.go:658-685, for one query head over one
// slice [t0, t1) of the context.  Cached K and V rows of a tile go to shared
// memory by cp.async; the first tile's copies are issued before the poll for
// q, so they overlap the QKV phase.  The new position's k and v come from the
// QKV phase's LL words (its cache stores are not ordered with them).  Scores:
// one thread per position; weighted V sum: thread (chunk vc, group vg) sums 8
// dims over positions vg, vg + ngrp, ...; online softmax across tiles.  The
// result is o / l (one split) or the split partial (o, m, l).  Not inlined,
// so its tiles and gathers do not raise the kernel's register peak.
template <bool F32>
__device__ __noinline__ int attn_phase(const uint2* qsrc, const uint2* ksrc, const uint2* vsrc, const uint8_t* kg,
                                       const uint8_t* vg, uint32_t gs, int hd, int TP, int t0, int t1, int pos,
                                       unsigned tag_here, unsigned tag_out, uint2* out, int split_out, int* err,
                                       uint32_t xs_off, uint32_t red_off, int alive) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int ES = F32 ? 4 : 2;
    const int ct = threadIdx.x - 32, lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 1;
    float* xs = reinterpret_cast<float*>(smem + xs_off);
    float* red = reinterpret_cast<float*>(smem + red_off);
    const int rowb = hd * ES, KS = rowb + 16;  // K rows padded: no bank conflicts across positions
    float* aq = xs;                    // [hd] q
    float* akc = aq + hd;              // [hd] k of the new position
    float* avc = akc + hd;             // [hd] v of the new position
    float* ao = avc + hd;              // [hd] running output
    float* asc = ao + hd;              // [TP] probabilities of the tile
    float* avred = asc + TP;           // [kConsumerWarps][hd] per-warp V sums
    uint8_t* ktile = reinterpret_cast<uint8_t*>(avred + kConsumerWarps * hd);  // [TP][KS]
    uint8_t* vtile = ktile + (size_t)TP * KS;                                   // [TP][rowb]
    const int pieces = rowb / 16;
    auto load_tile = [&](int tb, int nt) {
        for (int i = ct; i < nt * pieces; i += kConsumerThreads) {
            const int t = i / pieces, c = i - t * pieces;
            if (tb + t == pos) continue;
            cp_async16(ktile + (size_t)t * KS + c * 16, kg + (size_t)(tb + t) * gs + c * 16);
            cp_async16(vtile + (size_t)t * rowb + c * 16, vg + (size_t)(tb + t) * gs + c * 16);
        }
        cp_async_commit();
    };
    if (t1 > t0) load_tile(t0, min(TP, t1 - t0));

    if (alive) alive = ll_gather_s(qsrc, hd, tag_here, err, smem_u32(aq), 0, 0, 0).ok;
    if (alive && pos >= t0 && pos < t1) {
        alive = ll_gather_s(ksrc, hd, tag_here, err, smem_u32(akc), 0, 0, 0).ok;
        if (alive) alive = ll_gather_s(vsrc, hd, tag_here, err, smem_u32(avc), 0, 0, 0).ok;
    }
    for (int i = ct; i < hd; i += kConsumerThreads) ao[i] = 0.0f;
    cp_async_wait();
    named_bar_sync(1, kConsumerThreads);

    const float scale = (float)(1.0 / sqrt((double)hd));
    const int hv = hd / 8, ngrp = kConsumerThreads / hv;
    const int vc = ct % hv, vgi = ct / hv;
    float mrun = -INFINITY, lrun = 0.0f;
    for (int tb = t0; tb < t1; tb += TP) {
        const int nt = min(TP, t1 - tb);
        if (tb != t0) {
            load_tile(tb, nt);
            cp_async_wait();
            named_bar_sync(1, kConsumerThreads);
        }
        // scores (transformer.go:664-671)
        float sv = -INFINITY;
        if (ct < nt) {
            float d0 = 0.0f, d1 = 0.0f;
            if (tb + ct == pos) {
                for (int d = 0; d < hd; d += 2) {
                    d0 = fmaf(aq[d], akc[d], d0);
                    d1 = fmaf(aq[d + 1], akc[d + 1], d1);
                }
            } else if (F32) {
                const float4* kr = reinterpret_cast<const float4*>(ktile + (size_t)ct * KS);
                const float4* q4 = reinterpret_cast<const float4*>(aq);
                for (int i = 0; i < hd / 4; i++) {
                    const float4 k = kr[i], q = q4[i];
                    d0 = fmaf(q.x, k.x, d0);
                    d1 = fmaf(q.y, k.y, d1);
                    d0 = fmaf(q.z, k.z, d0);
                    d1 = fmaf(q.w, k.w, d1);
                }
            } else {
                const uint4* kr = reinterpret_cast<const uint4*>(ktile + (size_t)ct * KS);
                const float4* q4 = reinterpret_cast<const float4*>(aq);
                for (int i = 0; i < hd / 8; i++) {
                    const uint4 ku = kr[i];
                    const __half2* kh = reinterpret_cast<const __half2*>(&ku);
                    const float4 qa = q4[2 * i], qb = q4[2 * i + 1];
                    const float2 f0 = __half22float2(kh[0]), f1 = __half22float2(kh[1]);
                    const float2 f2 = __half22float2(kh[2]), f3 = __half22float2(kh[3]);
                    d0 = fmaf(qa.x, f0.x, d0);
                    d1 = fmaf(qa.y, f0.y, d1);
                    d0 = fmaf(qa.z, f1.x, d0);
                    d1 = fmaf(qa.w, f1.y, d1);
                    d0 = fmaf(qb.x, f2.x, d0);
                    d1 = fmaf(qb.y, f2.y, d1);
                    d0 = fmaf(qb.z, f3.x, d0);
                    d1 = fmaf(qb.w, f3.y, d1);
                }
            }
            sv = (d0 + d1) * scale;
        }
        // online softmax (transformer.go:673-677)
        const float mb = block_max(sv, red, cw);
        const float mnew = fmaxf(mrun, mb);
        const float pv = (ct < nt) ? expf(sv - mnew) : 0.0f;
        if (ct < nt) asc[ct] = pv;
        const float lb = block_sum(pv, red, cw);  // its barriers also publish asc[]
        const float corr = (mrun == -INFINITY) ? 0.0f : expf(mrun - mnew);
        lrun = lrun * corr + lb;
        mrun = mnew;
        // weighted V sum (transformer.go:679-685)
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; e++) acc[e] = 0.0f;
        for (int tl = vgi; tl < nt; tl += ngrp) {
            const float pt = asc[tl];
            float vf[8];
            if (tb + tl == pos) {
#pragma unroll
                for (int e = 0; e < 8; e++) vf[e] = avc[vc * 8 + e];
            } else if (F32) {
                const float4* vr = reinterpret_cast<const float4*>(vtile + (size_t)tl * rowb + vc * 32);
                const float4 x0 = vr[0], x1 = vr[1];
                vf[0] = x0.x; vf[1] = x0.y; vf[2] = x0.z; vf[3] = x0.w;
                vf[4] = x1.x; vf[5] = x1.y; vf[6] = x1.z; vf[7] = x1.w;
            } else {
                const uint4 vu = *reinterpret_cast<const uint4*>(vtile + (size_t)tl * rowb + vc * 16);
                const __half2* vh = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f = __half22float2(vh[e]);
                    vf[2 * e] = f.x;
                    vf[2 * e + 1] = f.y;
                }
            }
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] = fmaf(pt, vf[e], acc[e]);
        }
        // lanes of one warp that share a chunk: lane, lane ^ hv, ...
        for (int o = hv; o < 32; o <<= 1) {
#pragma unroll
            for (int e = 0; e < 8; e++) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
        }
        if (lane < hv) {
#pragma unroll
            for (int e = 0; e < 8; e++) avred[cw * hd + lane * 8 + e] = acc[e];
        }
        named_bar_sync(1, kConsumerThreads);
        for (int d = ct; d < hd; d += kConsumerThreads) {
            float o = ao[d] * corr;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; w++) o += avred[w * hd + d];
            ao[d] = o;
        }
        named_bar_sync(1, kConsumerThreads);
    }
    if (!split_out) {
        for (int d = ct; d < hd; d += kConsumerThreads) ll_store(out + d, ao[d] / lrun, tag_out);
    } else {
        // split partial (o unnormalised, m, l), laid out [head][split][hd + 2]
        for (int i = ct; i < hd + 2; i += kConsumerThreads) {
            const float v = i < hd ? ao[i] : (i == hd ? mrun : lrun);
            ll_store(out + i, v, tag_out);
        }
    }
    return alive;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int QT>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const ModelDev m, const StepArgs a) {
    constexpr int US = QT == 8 ? 16 : 32;  // values per lane unit
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = m.nslots;
    const int SB = m.slot_bytes;
    const SmemOffsets so = smem_offsets(NS, SB, m.xs_floats, m.ybuf_floats, m.cfloats);
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + so.xs);
    float* xres = reinterpret_cast<float*>(smem + so.xres);
    float* ybuf = reinterpret_cast<float*>(smem + so.ybuf);
    float* cb = reinterpret_cast<float*>(smem + so.cbuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + so.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + so.empty);
    float* red = reinterpret_cast<float*>(smem + so.red);
    int* misc = reinterpret_cast<int*>(smem + so.misc);
    volatile unsigned* pstop = reinterpret_cast<volatile unsigned*>(misc + 31);  // first chunk not issued
    volatile int* dead = misc + 30;  // set by any consumer thread whose wait failed

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, grid = gridDim.x;

    // A device-resident greedy loop that already produced EOS does no work.
    if (a.done && *(volatile const int*)a.done) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        *pstop = 0xffffffffu;
        *dead = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == 0) {
        if (lane == 0) {
            unsigned gidx = 0;
            bool ok = true;
            for (int p = a.p_begin; p < a.p_end && ok; p++) {
                Geom g = phase_geom(m, a, p);
                Split s = cta_split(g, cta, grid, SB);
                for (int k = 0; k < s.nchunks && ok; k++, gidx++) {
                    if (a.trace && (k == 0 || k == s.nchunks - 1))
                        a.trace[((size_t)(p - a.p_begin) * kTraceSlots + (k == 0 ? 4 : 5)) * grid + cta] = global_ns();
                    const int slot = gidx % NS;
                    const uint32_t round = gidx / NS;
                    if (*(volatile int*)m.err || !slot_wait(&empty[slot], (round & 1) ^ 1, m.err)) {
                        *pstop = gidx;  // consumers skip chunks from here on
                        ok = false;
                        break;
                    }
                    const int uu0 = s.u0 + k * s.cu;
                    const int nu = min(s.cu, s.n - k * s.cu);
                    const size_t r0 = (size_t)uu0 * g.rpu, nbytes = (size_t)nu * g.rpu * g.rb;
                    const uint8_t* src = g.w + r0 * g.rb;
                    const uint8_t* sal = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
                    const uint32_t len1 = (uint32_t)(((src - sal) + nbytes + 15) & ~size_t(15));
                    uint32_t total = len1, len2 = 0, off2 = 0;
                    const uint8_t* sal2 = nullptr;
                    if (g.w2) {
                        const uint8_t* src2 = g.w2 + r0 * g.rb;
                        sal2 = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src2) & ~uintptr_t(15));
                        len2 = (uint32_t)(((src2 - sal2) + nbytes + 15) & ~size_t(15));
                        off2 = (len1 + 127) & ~127u;
                        total = len1 + len2;
                    }
                    uint8_t* dst = ring + (size_t)slot * SB;
                    mbar_arrive_expect_tx(&full[slot], total);
                    bulk_g2s(dst, sal, len1, &full[slot]);
                    if (g.w2) bulk_g2s(dst + off2, sal2, len2, &full[slot]);
                }
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int cw = warp - 1;              // consumer warp index
    const int ct = threadIdx.x - 32;      // consumer thread index
    unsigned gbase = 0;                   // chunk index of the phase's first chunk
    bool alive = true;
    const int tok = a.mv_w ? 0 : *a.tok;
    const int own0 = (int)((long long)cta * m.H / grid);  // residual rows [own0, own1)
    const int own1 = (int)((long long)(cta + 1) * m.H / grid);
    // Consumer barrier that also makes `alive` uniform across the CTA: a
    // failed wait in any thread stops the work of all (warp collectives in
    // the row loop must never run with part of a warp).
    auto sync_alive = [&]() {
        if (!alive) *dead = 1;
        named_bar_sync(1, kConsumerThreads);
        alive = (*dead == 0);
    };

    for (int p = a.p_begin; p < a.p_end; p++) {
        const Geom g = phase_geom(m, a, p);
        const Split s = cta_split(g, cta, grid, SB);
        const bool has_rows = s.nchunks > 0;
        const size_t tr = (size_t)(p - a.p_begin) * kTraceSlots;
        if (a.trace && ct == 0) a.trace[(tr + 0) * grid + cta] = global_ns();
        const unsigned tag_here = ll_tag(a.epoch, g.layer) + a.skew;
        const unsigned tag_prev = ll_tag(a.epoch, g.layer - 1) + a.skew;

        // 1. stage the phase input
        if (g.kind == PH_QKV && g.layer == 0) {
            // transformer.go:524-531: the residual stream starts at the embedding
            for (int j = own0 + ct; j < own1; j += kConsumerThreads) xres[j - own0] = embed_elem(m, tok, j);
        }
        if ((g.kind == PH_QKV || g.kind == PH_GATEUP || g.kind == PH_LMHEAD) && has_rows) {
            // constants first (they land while the poll below waits)
            const float* nw = g.kind == PH_QKV ? m.layers[g.layer].attn_norm
                            : (g.kind == PH_GATEUP ? m.layers[g.layer].ffn_norm : m.out_norm);
            for (int i = ct; i < m.H / 4; i += kConsumerThreads) cp_async16(cb + 4 * i, nw + 4 * i);
            if (g.kind == PH_QKV) {
                const float* bq = m.layers[g.layer].bqkv;
                const int r0b = (2 * s.u0) & ~3, r1 = 2 * (s.u0 + s.n);
                if (bq)
                    for (int i = ct; i < (r1 - r0b + 3) / 4; i += kConsumerThreads)
                        cp_async16(cb + cb_bias(m) + 4 * i, bq + r0b + 4 * i);
                const int hh = m.hd / 2;
                for (int i = ct; i < hh / 4; i += kConsumerThreads) {
                    cp_async16(cb + cb_cos(m) + 4 * i, m.rope_cos + (size_t)a.pos * hh + 4 * i);
                    cp_async16(cb + cb_sin(m) + 4 * i, m.rope_sin + (size_t)a.pos * hh + 4 * i);
                }
            }
            cp_async_commit();
            // RMSNorm (transformer.go:922-932) fused into the stage
            const int nu_h = m.H / US;
            float ss = 0.0f;
            if (g.kind == PH_QKV && g.layer == 0) {
                for (int j = ct; j < m.H; j += kConsumerThreads) {
                    const float v = embed_elem(m, tok, j);
                    xs[xs_index<US>(j, nu_h)] = v;
                    ss += v * v;
                }
            } else if (alive) {
                const uint2* src = g.kind == PH_GATEUP ? m.ll_x1 : m.ll_x2;
                const unsigned tg = g.kind == PH_GATEUP ? tag_here : tag_prev;
                const GatherRes gr = ll_gather_s(src, m.H, tg, m.err, smem_u32(xs), US, nu_h, 1);
                alive = gr.ok;
                ss = gr.ss;
            }
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
            cp_async_wait();
            const float tot = block_sum(ss, red, cw);  // its barriers also publish cb[]
            const float r = (float)(1.0 / sqrt((double)(tot / (float)m.H) + (double)m.eps));
            for (int j = ct; j < m.H; j += kConsumerThreads) {
                float* px = xs + xs_index<US>(j, nu_h);
                *px = *px * r * cb[j];
            }
        } else if (g.kind == PH_WO && has_rows) {
            const int nu_q = m.qd / US;
            if (a.splits == 1) {
                if (alive)
                    alive = ll_gather_s(m.ll_attn, m.qd, tag_here, m.err, smem_u32(xs), US, nu_q, 0).ok;
                if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
            } else {
                // merge the context splits: o = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M)
                const int S = a.splits, hd = m.hd, W2 = hd + 2;
                float* part = xs + m.qd;  // [nh][S][hd+2] after the qd outputs
                if (alive)
                    alive = ll_gather_s(m.ll_part, m.nh * S * W2, tag_here, m.err, smem_u32(part), 0, 0, 0).ok;
                if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
                named_bar_sync(1, kConsumerThreads);
                for (int i = ct; i < m.qd; i += kConsumerThreads) {
                    const int hh = i / hd, d = i - hh * hd;
                    const float* ph = part + (size_t)hh * S * W2;
                    float M = -INFINITY;
                    for (int s2 = 0; s2 < S; s2++) M = fmaxf(M, ph[s2 * W2 + hd]);
                    float Ls = 0.0f, o = 0.0f;
                    for (int s2 = 0; s2 < S; s2++) {
                        const float ms = ph[s2 * W2 + hd];
                        const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
                        Ls = fmaf(ph[s2 * W2 + hd + 1], w, Ls);
                        o = fmaf(ph[s2 * W2 + d], w, o);
                    }
                    xs[xs_index<US>(i, nu_q)] = o / Ls;
                }
            }
        } else if (g.kind == PH_DOWN && has_rows) {
            const int nu_f = m.FF / US;
            if (alive)
                alive = ll_gather_s(m.ll_act, m.FF, tag_here, m.err, smem_u32(xs), US, nu_f, 0).ok;
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        } else if (g.kind == PH_MATVEC) {
            const int nu = g.cols / US;
            for (int j = ct; j < g.cols; j += kConsumerThreads) xs[xs_index<US>(j, nu)] = a.mv_x[j];
        } else {
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        }
        sync_alive();
        if (a.trace && ct == 0) a.trace[(tr + 2) * grid + cta] = global_ns();

        float* yb = ybuf + (p & 1) * m.ybuf_floats;  // parity buffers: the next phase's
                                                      // dots may start before this epilogue ends
        if (g.kind == PH_ATTN) {
            // 2'. attention, one (query head, split) per CTA
            if (cta < m.nh * a.splits) {
                const int S = a.splits, hd = m.hd;
                const int h = cta / S, sidx = cta - h * S, kvh = h / (m.nh / m.nkv);
                const int ctx = a.pos + 1;
                const int t0 = (int)((long long)sidx * ctx / S), t1 = (int)((long long)(sidx + 1) * ctx / S);
                const int es = m.kv_fp32 ? 4 : 2;
                const size_t lay = ((size_t)g.layer * m.max_seq * m.kvd + (size_t)kvh * hd) * es;
                const uint8_t* kg = reinterpret_cast<const uint8_t*>(m.kcache) + lay;
                const uint8_t* vg = reinterpret_cast<const uint8_t*>(m.vcache) + lay;
                uint2* out = S == 1 ? m.ll_attn + (size_t)h * hd : m.ll_part + ((size_t)h * S + sidx) * (hd + 2);
                const uint2* q = m.ll_qkv + (size_t)h * hd;
                const uint2* kn = m.ll_qkv + m.qd + (size_t)kvh * hd;
                const uint2* vn = kn + m.kvd;
                const unsigned tout = ll_tag(a.epoch, g.layer);
                alive = m.kv_fp32
                            ? attn_phase<true>(q, kn, vn, kg, vg, (uint32_t)(m.kvd * es), hd, m.attn_tile, t0, t1, a.pos,
                                               tag_here, tout, out, S != 1, m.err, so.xs, so.red, alive)
                            : attn_phase<false>(q, kn, vn, kg, vg, (uint32_t)(m.kvd * es), hd, m.attn_tile, t0, t1,
                                                a.pos, tag_here, tout, out, S != 1, m.err, so.xs, so.red, alive);
            }
        } else {
            // 2. rows: dot products of this CTA's weight rows into yb
            const int rbase = g.rpu * s.u0;
            for (int k = 0; k < s.nchunks; k++) {
                const unsigned gidx = gbase + k;
                if ((int)(gidx % kConsumerWarps) != cw) continue;
                const int slot = gidx % NS;
                const bool landed =
                    __all_sync(0xffffffffu, chunk_wait(&full[slot], (gidx / NS) & 1, gidx, pstop, m.err));
                if (!landed) alive = false;
                if (alive) {
                    const uint8_t* dst = ring + (size_t)slot * SB;
                    const int uu0 = s.u0 + k * s.cu;
                    const int nu = min(s.cu, s.n - k * s.cu);
                    const size_t r0 = (size_t)uu0 * g.rpu;
                    const uint8_t* src = g.w + r0 * g.rb;
                    const uint8_t* base1 = dst + (reinterpret_cast<uintptr_t>(src) & 15);
                    const uint8_t* base2 = base1;
                    if (g.w2) {
                        const uintptr_t s2 = reinterpret_cast<uintptr_t>(g.w2 + r0 * g.rb);
                        const uint32_t len1 = (uint32_t)((((uintptr_t)src & 15) + (size_t)nu * g.rb + 15) & ~size_t(15));
                        base2 = dst + ((len1 + 127) & ~127u) + (s2 & 15);
                    }
                    const int nrows = nu * g.rpu;
                    const int npairs = g.w2 ? nrows : (nrows + 1) / 2;
                    for (int pi = 0; pi < npairs; pi++) {
                        const uint8_t *ra, *rb2;
                        bool two;
                        int yi;  // output index of the pair's first row in yb
                        if (g.w2) {
                            ra = base1 + (size_t)pi * g.rb;
                            rb2 = base2 + (size_t)pi * g.rb;
                            two = true;
                            yi = 2 * (uu0 - s.u0 + pi);  // gate, up interleaved
                        } else {
                            ra = base1 + (size_t)(2 * pi) * g.rb;
                            two = (2 * pi + 1) < nrows;
                            rb2 = two ? ra + g.rb : ra;
                            yi = (int)r0 - rbase + 2 * pi;
                        }
                        float a0, a1;
                        if (QT == 8) dot2_q8(ra, rb2, two, xs, g.cols, lane, a0, a1);
                        else dot2_q4(ra, rb2, two, xs, g.cols, lane, a0, a1);
                        const float v = warp_sum2(a0, a1, lane);
                        if (lane == 0) yb[yi] = v;
                        if (lane == 16 && two) yb[yi + 1] = v;
                    }
                }
                __syncwarp();
                if (lane == 0 && landed) mbar_arrive(&empty[slot]);
            }
            gbase += s.nchunks;
        }
        sync_alive();

        // 3. epilogue, one thread per output
        const unsigned tag = ll_tag(a.epoch, g.layer);
        if ((alive && has_rows) || g.kind == PH_LMHEAD) {
            // (every CTA takes part in the argmax, so its arrival counter
            // always completes and resets)
            switch (g.kind) {
                case PH_QKV: {
                    // bias (transformer.go:632-646), RoPE on interleaved pairs
                    // (936-951), KV append (654-656)
                    const bool bias = m.layers[g.layer].bqkv != nullptr;
                    const int bias0 = (2 * s.u0) & ~3;
                    for (int j = ct; j < s.n; j += kConsumerThreads) {
                        const int row = 2 * (s.u0 + j);
                        float a0 = yb[2 * j], a1 = yb[2 * j + 1];
                        if (bias) {
                            a0 += cb[cb_bias(m) + row - bias0];
                            a1 += cb[cb_bias(m) + row + 1 - bias0];
                        }
                        if (row < m.qd + m.kvd) {
                            const int pi2 = (row % m.hd) >> 1;
                            const float rc = cb[cb_cos(m) + pi2], rs = cb[cb_sin(m) + pi2];
                            const float x0 = a0, x1 = a1;
                            a0 = x0 * rc - x1 * rs;
                            a1 = x0 * rs + x1 * rc;
                        }
                        ll_store2(m.ll_qkv + row, a0, a1, tag);
                        if (row >= m.qd) {
                            const bool isk = row < m.qd + m.kvd;
                            const int col = row - m.qd - (isk ? 0 : m.kvd);
                            const size_t off = ((size_t)g.layer * m.max_seq + a.pos) * m.kvd + col;
                            void* cache = isk ? m.kcache : m.vcache;
                            if (m.kv_fp32) {
                                reinterpret_cast<float*>(cache)[off] = a0;
                                reinterpret_cast<float*>(cache)[off + 1] = a1;
                            } else {
                                *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(cache) + off) =
                                    __floats2half2_rn(a0, a1);
                            }
                        }
                    }
                    break;
                }
                case PH_GATEUP:
                    // SwiGLU (transformer.go:725-727, 954-956)
                    for (int j = ct; j < s.n; j += kConsumerThreads) {
                        const float gv = yb[2 * j], uv = yb[2 * j + 1];
                        ll_store(m.ll_act + s.u0 + j, gv / (1.0f + expf(-gv)) * uv, tag);
                    }
                    break;
                case PH_WO:
                case PH_DOWN: {
                    // residual (transformer.go:576-578, 591-593); the rows are
                    // exactly the residual rows this CTA owns
                    uint2* dstll = g.kind == PH_WO ? m.ll_x1 : m.ll_x2;
                    for (int j = ct; j < s.n; j += kConsumerThreads) {
                        const int row = s.u0 + j;
                        const float xr = xres[row - own0] + yb[j];
                        xres[row - own0] = xr;
                        ll_store(dstll + row, xr, tag);
                    }
                    break;
                }
                case PH_LMHEAD: {
                    // logits + argmax, first maximum wins (transformer.go:1038-1046)
                    Best best{-INFINITY, 0x7fffffff};
                    for (int j = ct; alive && j < s.n; j += kConsumerThreads) {
                        const int row = s.u0 + j;
                        const float v = yb[j];
                        m.logits[row] = v;
                        if (better(v, row, best.v, best.i)) { best.v = v; best.i = row; }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
                        const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
                        if (better(ov, oi, best.v, best.i)) { best.v = ov; best.i = oi; }
                    }
                    if (lane == 0) { red[cw] = best.v; misc[4 + cw] = best.i; }
                    named_bar_sync(1, kConsumerThreads);
                    if (ct == 0) {
                        Best b{red[0], misc[4]};
                        for (int w = 1; w < kConsumerWarps; w++)
                            if (better(red[w], misc[4 + w], b.v, b.i)) { b.v = red[w]; b.i = misc[4 + w]; }
                        m.best_val[cta] = b.v;
                        m.best_idx[cta] = b.i;
                        __threadfence();
                        const unsigned old = atom_acq_rel_add(m.am_ctr, 1u);
                        if (old == (unsigned)(grid - 1)) {
                            Best f{-INFINITY, 0x7fffffff};
                            for (int c2 = 0; c2 < grid; c2++) {
                                const float v = __ldcg(m.best_val + c2);
                                const int i = __ldcg(m.best_idx + c2);
                                if (better(v, i, f.v, f.i)) { f.v = v; f.i = i; }
                            }
                            if (f.i == 0x7fffffff) f.i = 0;
                            *m.token = f.i;
                            if (a.out_ids) a.out_ids[a.step] = f.i;
                            if (a.done && f.i == a.eos) *a.done = 1;
                            atomicExch(m.am_ctr, 0u);
                        }
                    }
                    break;
                }
                default:  // PH_MATVEC
                    for (int j = ct; j < s.n; j += kConsumerThreads) a.mv_y[s.u0 + j] = yb[j];
                    break;
            }
        }
        if (a.trace && ct == 0) a.trace[(tr + 3) * grid + cta] = global_ns();
    }
}

}  // namespace

size_t decode_smem_bytes(const ModelDev& m) {
    return smem_offsets(m.nslots, m.slot_bytes, m.xs_floats, m.ybuf_floats, m.cfloats).total;
}

int launch_decode(const ModelDev& m, const StepArgs& a, int grid, cudaStream_t stream, std::string* err) {
    const size_t smem = decode_smem_bytes(m);
    void* args[] = {(void*)&m, (void*)&a};
    const void* fn = m.qtype == 8 ? (const void*)decode_kernel<8> : (const void*)decode_kernel<2>;
    static bool attr_done[2] = {false, false};
    const int ti = m.qtype == 8 ? 0 : 1;
    if (!attr_done[ti]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (e != cudaSuccess) {
            *err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
            return B2_ERR_CUDA;
        }
        attr_done[ti] = true;
    }
    cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, smem, stream);
    if (e != cudaSuccess) {
        *err = std::string("decode launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

}  // namespace b2
