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
//   warps 1..12      consumers: per phase, gather the phase input from the
//                    previous phase's LL words (the poll is the load), stage it
//                    in shared memory with RMSNorm / embedding decode /
//                    attention-split merge fused in, then dequantise their
//                    chunks in registers and accumulate in fp32, with the
//                    phase epilogue fused (bias + RoPE + KV append, residual
//                    add, SwiGLU, logits + argmax).
// Each CTA keeps the residual-stream rows it owns (the same rows in every Wo
// and down phase) in shared memory, so residual adds never touch global
// memory.  Every wait is bounded (globaltimer) and reports B2_ERR_TIMEOUT
// through the device error flag instead of hanging.
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
            g.units = m.nkv * a.splits;
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

// Gathers LL words src[0 .. n) (n even, src 16-byte aligned) once every word
// carries `tag`, calling put(i, value).  Each consumer thread polls its own
// words with 16-byte loads, up to 8 in flight; a word whose tag is stale is
// simply read again.  Bounded: gives up (returns false, error flag set) after
// kWaitLimitNs or when another CTA already reported an error.
template <class Put>
__device__ __forceinline__ bool ll_gather(const uint2* src, int n, unsigned tag, int ct, int* err, Put put) {
    const int n2 = n >> 1;
    uint64_t t0 = 0;
    for (int base = 0; base < n2; base += kConsumerThreads * 8) {
        uint4 v[8];
        for (;;) {
            bool ok = true;
#pragma unroll
            for (int k = 0; k < 8; k++) {
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
                return false;
            }
            if (*(volatile int*)err) return false;
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = base + ct + k * kConsumerThreads;
            if (i < n2) {
                put(2 * i, __uint_as_float(v[k].x));
                put(2 * i + 1, __uint_as_float(v[k].z));
            }
        }
    }
    return true;
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

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int QT>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const ModelDev m, const StepArgs a) {
    constexpr int US = QT == 8 ? 16 : 32;  // values per lane unit
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = m.nslots;
    const int SB = m.slot_bytes;
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)NS * SB + 128);
    float* xres = xs + m.xs_floats;                       // [kMaxOwnRows] residual rows owned
    float* qconst = xres + kMaxOwnRows;                   // [3][kMaxQkvRows] bias, cos, sin of the QKV rows
    uint64_t* full = reinterpret_cast<uint64_t*>(qconst + 3 * kMaxQkvRows);
    uint64_t* empty = full + NS;
    float* red = reinterpret_cast<float*>(empty + NS);    // 64 floats
    int* misc = reinterpret_cast<int*>(red + 64);         // 32 ints
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
    Best best{-INFINITY, 0x7fffffff};
    const int tok = a.mv_w ? 0 : *a.tok;
    const int own0 = (int)((long long)cta * m.H / grid);  // residual rows [own0, own1)
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
        const size_t tr = (size_t)(p - a.p_begin) * kTraceSlots;
        if (a.trace && ct == 0) a.trace[(tr + 0) * grid + cta] = global_ns();

        // 1+2. gather the phase input (the LL poll) and stage it in shared memory
        const unsigned tag_here = ll_tag(a.epoch, g.layer) + a.skew;
        const unsigned tag_prev = ll_tag(a.epoch, g.layer - 1) + a.skew;
        const int nu_h = m.H / US;
        if (g.kind == PH_QKV || g.kind == PH_GATEUP || g.kind == PH_LMHEAD) {
            // RMSNorm (transformer.go:922-932) fused into the stage; the norm
            // gains are fetched before the poll so their latency overlaps it.
            const float* nw = g.kind == PH_QKV ? m.layers[g.layer].attn_norm
                            : (g.kind == PH_GATEUP ? m.layers[g.layer].ffn_norm : m.out_norm);
            float wreg[8];
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int j = ct + k * kConsumerThreads;
                wreg[k] = (j < m.H) ? __ldg(nw + j) : 0.0f;
            }
            if (g.kind == PH_QKV) {
                // this CTA's QKV epilogue constants (bias, RoPE cos/sin at pos),
                // loaded while the poll below waits
                const int row0 = 2 * s.u0, nrow = 2 * s.n;
                const LayerDev& Ld = m.layers[g.layer];
                for (int i = ct; i < nrow; i += kConsumerThreads) {
                    const int row = row0 + i;
                    qconst[i] = Ld.bqkv ? __ldg(Ld.bqkv + row) : 0.0f;
                    float c = 1.0f, sn = 0.0f;
                    if (row < m.qd + m.kvd) {
                        const int pi = (row % m.hd) >> 1;
                        c = __ldg(m.rope_cos + (size_t)a.pos * (m.hd / 2) + pi);
                        sn = __ldg(m.rope_sin + (size_t)a.pos * (m.hd / 2) + pi);
                    }
                    qconst[kMaxQkvRows + i] = c;
                    qconst[2 * kMaxQkvRows + i] = sn;
                }
            }
            float ss = 0.0f;
            if (g.kind == PH_QKV && g.layer == 0) {
                for (int j = ct; j < m.H; j += kConsumerThreads) {
                    const float v = embed_elem(m, tok, j);
                    xs[xs_index<US>(j, nu_h)] = v;
                    if (j >= own0 && j - own0 < kMaxOwnRows) xres[j - own0] = v;
                    ss += v * v;
                }
            } else if (alive) {
                const uint2* src = g.kind == PH_GATEUP ? m.ll_x1 : m.ll_x2;
                const unsigned tg = g.kind == PH_GATEUP ? tag_here : tag_prev;
                alive = ll_gather(src, m.H, tg, ct, m.err, [&](int j, float v) {
                    xs[xs_index<US>(j, nu_h)] = v;
                    ss += v * v;
                });
            }
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
            ss = warp_sum(ss);
            if (lane == 0) red[cw] = ss;
            named_bar_sync(1, kConsumerThreads);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; w++) tot += red[w];
            const float r = (float)(1.0 / sqrt((double)(tot / (float)m.H) + (double)m.eps));
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int j = ct + k * kConsumerThreads;
                if (j < m.H) {
                    float* px = xs + xs_index<US>(j, nu_h);
                    *px = *px * r * wreg[k];
                }
            }
            for (int j = ct + 8 * kConsumerThreads; j < m.H; j += kConsumerThreads) {
                float* px = xs + xs_index<US>(j, nu_h);
                *px = *px * r * __ldg(nw + j);
            }
        } else if (g.kind == PH_WO) {
            // merge the attention splits: o = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M)
            const int S = a.splits, hd = m.hd, W2 = hd + 2;
            float* part = xs + m.qd;  // [nh][S][hd+2] after the qd outputs
            if (alive)
                alive = ll_gather(m.ll_part, m.nh * S * W2, tag_here, ct, m.err,
                                  [&](int i, float v) { part[i] = v; });
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
            named_bar_sync(1, kConsumerThreads);
            const int nu_q = m.qd / US;
            for (int i = ct; i < m.qd; i += kConsumerThreads) {
                const int h = i / hd, d = i % hd;
                const float* ph = part + (size_t)h * S * W2;
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
        } else if (g.kind == PH_DOWN) {
            const int nu_f = m.FF / US;
            if (alive)
                alive = ll_gather(m.ll_act, m.FF, tag_here, ct, m.err,
                                  [&](int j, float v) { xs[xs_index<US>(j, nu_f)] = v; });
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        } else if (g.kind == PH_ATTN) {
            if (a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        } else if (g.kind == PH_MATVEC) {
            const int nu = g.cols / US;
            for (int j = ct; j < g.cols; j += kConsumerThreads) xs[xs_index<US>(j, nu)] = a.mv_x[j];
        }
        sync_alive();
        if (a.trace && ct == 0) a.trace[(tr + 2) * grid + cta] = global_ns();

        // 3. the phase's work
        if (g.kind == PH_ATTN) {
            if (cta < g.units) {
                // transformer.go:658-685 for the query heads of one KV head over
                // one slice of the context (online softmax over 32-position
                // tiles); the slice partial (o, m, l) goes out as LL words and
                // every CTA merges the slices when it stages the Wo input.
                const int S = a.splits;
                const int kvh = cta / S, sidx = cta % S;
                const int grp = m.nh / m.nkv, hd = m.hd;
                const int ctx = a.pos + 1;
                const int t0 = (int)((long long)sidx * ctx / S), t1 = (int)((long long)(sidx + 1) * ctx / S);
                float* qsm = xs;                       // [grp*hd]
                float* osm = qsm + grp * hd;           // [grp*hd]
                float* sc = osm + grp * hd;            // [grp*kAttnTile]
                float* mrun = sc + grp * kAttnTile;    // [grp]
                float* lrun = mrun + grp;              // [grp]
                float* corr = lrun + grp;              // [grp]
                float* ks = xs + ((grp * hd * 2 + grp * kAttnTile + 3 * grp + 3) & ~3);  // [tile][hd+4]
                float* vs = ks + kAttnTile * (hd + 4);                                      // [tile][hd]
                const float scale = (float)(1.0 / sqrt((double)hd));
                const size_t lay = (size_t)g.layer * m.max_seq * m.kvd;
                const int hv = hd / 8;  // 8-element vectors per head row
                // K/V rows of a tile: cached positions come from the cache
                // (written by earlier launches); the new position's k and v
                // come from this launch's LL words.
                auto stage_kv = [&](int tb, int nt) {
                    for (int i = ct; i < nt * hv; i += kConsumerThreads) {
                        const int t = i / hv, c8 = i % hv;
                        if (tb + t == a.pos) continue;
                        const size_t off = lay + (size_t)(tb + t) * m.kvd + (size_t)kvh * hd + c8 * 8;
                        float kf[8], vf[8];
                        if (m.kv_fp32) {
                            const float4* kp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(m.kcache) + off);
                            const float4* vp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(m.vcache) + off);
                            float4 a0 = __ldcg(kp), a1 = __ldcg(kp + 1), b0 = __ldcg(vp), b1 = __ldcg(vp + 1);
                            kf[0] = a0.x; kf[1] = a0.y; kf[2] = a0.z; kf[3] = a0.w; kf[4] = a1.x; kf[5] = a1.y; kf[6] = a1.z; kf[7] = a1.w;
                            vf[0] = b0.x; vf[1] = b0.y; vf[2] = b0.z; vf[3] = b0.w; vf[4] = b1.x; vf[5] = b1.y; vf[6] = b1.z; vf[7] = b1.w;
                        } else {
                            const uint4 ku = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(m.kcache) + off));
                            const uint4 vu = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(m.vcache) + off));
                            const __half2* kh = reinterpret_cast<const __half2*>(&ku);
                            const __half2* vh = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const float2 f0 = __half22float2(kh[e]), f1 = __half22float2(vh[e]);
                                kf[2 * e] = f0.x; kf[2 * e + 1] = f0.y; vf[2 * e] = f1.x; vf[2 * e + 1] = f1.y;
                            }
                        }
                        float4* kd = reinterpret_cast<float4*>(ks + t * (hd + 4) + c8 * 8);
                        float4* vd = reinterpret_cast<float4*>(vs + t * hd + c8 * 8);
                        kd[0] = make_float4(kf[0], kf[1], kf[2], kf[3]);
                        kd[1] = make_float4(kf[4], kf[5], kf[6], kf[7]);
                        vd[0] = make_float4(vf[0], vf[1], vf[2], vf[3]);
                        vd[1] = make_float4(vf[4], vf[5], vf[6], vf[7]);
                    }
                };
                // the first tile's cached rows load before the q poll
                if (t1 > t0) stage_kv(t0, min(kAttnTile, t1 - t0));
                // q of this group's heads, after RoPE (transformer.go:649-650)
                if (alive)
                    alive = ll_gather(m.ll_qkv + (size_t)kvh * grp * hd, grp * hd, tag_here, ct, m.err,
                                      [&](int i, float v) { qsm[i] = v; });
                for (int i = ct; i < grp * hd; i += kConsumerThreads) osm[i] = 0.0f;
                if (ct < grp) { mrun[ct] = -INFINITY; lrun[ct] = 0.0f; }
                for (int tb = t0; tb < t1; tb += kAttnTile) {
                    const int nt = min(kAttnTile, t1 - tb);
                    if (tb != t0) {
                        named_bar_sync(1, kConsumerThreads);  // previous tile fully consumed
                        stage_kv(tb, nt);
                    }
                    if (alive && a.pos >= tb && a.pos < tb + nt) {
                        // the new position's k and v rows (transformer.go:654-656)
                        const int t = a.pos - tb;
                        const uint2* kl = m.ll_qkv + m.qd + (size_t)kvh * hd;
                        const uint2* vl = m.ll_qkv + m.qd + m.kvd + (size_t)kvh * hd;
                        alive = ll_gather(kl, hd, tag_here, ct, m.err, [&](int i, float v) { ks[t * (hd + 4) + i] = v; });
                        if (alive)
                            alive = ll_gather(vl, hd, tag_here, ct, m.err, [&](int i, float v) { vs[t * hd + i] = v; });
                    }
                    named_bar_sync(1, kConsumerThreads);
                    // scores: warp = query head, lane = position
                    for (int i = ct; i < grp * kAttnTile; i += kConsumerThreads) {
                        const int h = i / kAttnTile, t = i % kAttnTile;
                        if (t < nt) {
                            const float4* qv = reinterpret_cast<const float4*>(qsm + h * hd);
                            const float4* kv = reinterpret_cast<const float4*>(ks + t * (hd + 4));
                            float d0 = 0.0f, d1 = 0.0f;
                            for (int d4 = 0; d4 < hd / 4; d4 += 2) {
                                const float4 a0 = qv[d4], b0 = kv[d4], a1 = qv[d4 + 1], b1 = kv[d4 + 1];
                                d0 = fmaf(a0.x, b0.x, d0); d0 = fmaf(a0.y, b0.y, d0);
                                d0 = fmaf(a0.z, b0.z, d0); d0 = fmaf(a0.w, b0.w, d0);
                                d1 = fmaf(a1.x, b1.x, d1); d1 = fmaf(a1.y, b1.y, d1);
                                d1 = fmaf(a1.z, b1.z, d1); d1 = fmaf(a1.w, b1.w, d1);
                            }
                            sc[i] = (d0 + d1) * scale;
                        } else {
                            sc[i] = -INFINITY;
                        }
                    }
                    named_bar_sync(1, kConsumerThreads);
                    // per-head max / exp / sum, one warp per head
                    for (int h = cw; h < grp; h += kConsumerWarps) {
                        float mx = -INFINITY;
                        for (int t = lane; t < kAttnTile; t += 32) mx = fmaxf(mx, sc[h * kAttnTile + t]);
                        mx = warp_max(mx);
                        const float mnew = fmaxf(mrun[h], mx);
                        float sum = 0.0f;
                        for (int t = lane; t < kAttnTile; t += 32) {
                            float e = (t < nt) ? expf(sc[h * kAttnTile + t] - mnew) : 0.0f;
                            sc[h * kAttnTile + t] = e;
                            sum += e;
                        }
                        sum = warp_sum(sum);
                        if (lane == 0) {
                            const float c = (mrun[h] == -INFINITY) ? 0.0f : expf(mrun[h] - mnew);
                            corr[h] = c;
                            lrun[h] = lrun[h] * c + sum;
                            mrun[h] = mnew;
                        }
                    }
                    named_bar_sync(1, kConsumerThreads);
                    for (int i = ct; i < grp * hd; i += kConsumerThreads) {
                        const int h = i / hd, d = i % hd;
                        float o = osm[i] * corr[h];
                        const float* ph = sc + h * kAttnTile;
                        for (int t = 0; t < nt; t++) o = fmaf(ph[t], vs[t * hd + d], o);
                        osm[i] = o;
                    }
                }
                named_bar_sync(1, kConsumerThreads);
                // this slice's partial (o unnormalised, m, l) as LL words,
                // laid out [head][split][hd + 2]
                const unsigned tag = ll_tag(a.epoch, g.layer);
                for (int i = ct; i < grp * (hd + 2); i += kConsumerThreads) {
                    const int h = i / (hd + 2), d = i % (hd + 2);
                    const float v = d < hd ? osm[h * hd + d] : (d == hd ? mrun[h] : lrun[h]);
                    ll_store(m.ll_part + ((size_t)(kvh * grp + h) * S + sidx) * (hd + 2) + d, v, tag);
                }
            }
        } else {
            const unsigned tag = ll_tag(a.epoch, g.layer);
            for (int k = 0; k < s.nchunks; k++) {
                const unsigned gidx = gbase + k;
                if ((int)(gidx % kConsumerWarps) != cw) continue;
                const int slot = gidx % NS;
                const bool landed = __all_sync(0xffffffffu, chunk_wait(&full[slot], (gidx / NS) & 1, gidx, pstop, m.err));
                if (!landed) alive = false;
                if (alive) {
                    const uint8_t* dst = ring + (size_t)slot * SB;
                    const int uu0 = s.u0 + k * s.cu;
                    const int nu = min(s.cu, s.n - k * s.cu);
                    const size_t r0 = (size_t)uu0 * g.rpu;
                    const uint8_t* src = g.w + r0 * g.rb;
                    const uint8_t* base1 = dst + (reinterpret_cast<uintptr_t>(src) & 15);
                    const uint8_t* base2 = nullptr;
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
                        int rowa;
                        if (g.w2) {
                            ra = base1 + (size_t)pi * g.rb;
                            rb2 = base2 + (size_t)pi * g.rb;
                            two = true;
                            rowa = (int)r0 + pi;
                        } else {
                            ra = base1 + (size_t)(2 * pi) * g.rb;
                            two = (2 * pi + 1) < nrows;
                            rb2 = two ? ra + g.rb : ra;
                            rowa = (int)r0 + 2 * pi;
                        }
                        float a0, a1;
                        if (QT == 8) dot2_q8(ra, rb2, two, xs, g.cols, lane, a0, a1);
                        else dot2_q4(ra, rb2, two, xs, g.cols, lane, a0, a1);
                        a0 = warp_sum(a0);
                        a1 = warp_sum(a1);
                        if (lane == 0) {
                            switch (g.kind) {
                                case PH_QKV: {
                                    // bias (transformer.go:632-646), RoPE on interleaved
                                    // pairs (936-951), KV append (654-656)
                                    const int qi = rowa - 2 * s.u0;
                                    a0 += qconst[qi];
                                    a1 += qconst[qi + 1];
                                    if (rowa < m.qd + m.kvd) {
                                        const float rc = qconst[kMaxQkvRows + qi], rs = qconst[2 * kMaxQkvRows + qi];
                                        const float x0 = a0, x1 = a1;
                                        a0 = x0 * rc - x1 * rs;
                                        a1 = x0 * rs + x1 * rc;
                                    }
                                    ll_store2(m.ll_qkv + rowa, a0, a1, tag);
                                    if (rowa >= m.qd) {
                                        const bool isk = rowa < m.qd + m.kvd;
                                        const int col = rowa - m.qd - (isk ? 0 : m.kvd);
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
                                    break;
                                }
                                case PH_GATEUP:
                                    // SwiGLU (transformer.go:725-727, 954-956)
                                    ll_store(m.ll_act + rowa, a0 / (1.0f + expf(-a0)) * a1, tag);
                                    break;
                                case PH_WO:
                                case PH_DOWN: {
                                    // residual (transformer.go:576-578, 591-593)
                                    uint2* dstll = g.kind == PH_WO ? m.ll_x1 : m.ll_x2;
                                    float* xr = xres + (rowa - own0);
                                    xr[0] += a0;
                                    ll_store(dstll + rowa, xr[0], tag);
                                    if (two) {
                                        xr[1] += a1;
                                        ll_store(dstll + rowa + 1, xr[1], tag);
                                    }
                                    break;
                                }
                                case PH_LMHEAD:
                                    m.logits[rowa] = a0;
                                    if (better(a0, rowa, best.v, best.i)) { best.v = a0; best.i = rowa; }
                                    if (two) {
                                        m.logits[rowa + 1] = a1;
                                        if (better(a1, rowa + 1, best.v, best.i)) { best.v = a1; best.i = rowa + 1; }
                                    }
                                    break;
                                default:  // PH_MATVEC
                                    a.mv_y[rowa] = a0;
                                    if (two) a.mv_y[rowa + 1] = a1;
                                    break;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0 && landed) mbar_arrive(&empty[slot]);
            }
            gbase += s.nchunks;
        }

        // 4. this CTA's part of the phase is done
        sync_alive();
        if (a.trace && ct == 0) a.trace[(tr + 3) * grid + cta] = global_ns();
        if (g.kind == PH_LMHEAD) {
            // argmax, first maximum wins (transformer.go:1038-1046)
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
        }
    }
}

}  // namespace

size_t decode_smem_bytes(const ModelDev& m) {
    return (size_t)m.nslots * m.slot_bytes + 128 + (size_t)m.xs_floats * 4 + kMaxOwnRows * 4 + 3 * kMaxQkvRows * 4 +
           16 * (size_t)m.nslots + 64 * 4 + 32 * 4;
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
