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
//                    producer runs ahead across phase boundaries and grid
//                    barriers, limited only by the ring.
//   warps 1..8       consumers: for each phase, wait for the previous phase
//                    everywhere (grid barrier), stage the phase input vector
//                    in shared memory (RMSNorm / embedding / attention output
//                    fused here), then dequantise their chunks in registers
//                    and accumulate in fp32, with the phase epilogue fused
//                    (bias + RoPE + KV append, residual add, SwiGLU, logits +
//                    argmax).
// Every wait is bounded (globaltimer) and reports B2_ERR_TIMEOUT through the
// device error flag instead of hanging.
#include <cuda_runtime.h>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "model.h"

namespace b2 {

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s for any single wait
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kAttnTile = 64;

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

// Bounded wait on an mbarrier phase.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kWaitLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Bounded wait until a grid counter reaches target (wrap-safe).
__device__ bool grid_wait(const unsigned* ctr, unsigned target, int* err) {
    if ((int)(ld_acquire(ctr) - target) >= 0) return true;
    uint64_t t0 = global_ns();
    for (;;) {
        if ((int)(ld_acquire(ctr) - target) >= 0) return true;
        if (*(volatile int*)err) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------
// dequantising dot products, two rows against one staged input vector
// ---------------------------------------------------------------------------

// 16 consecutive int8 of a Q8_0 block starting at a 2-byte aligned shared
// address, dotted with xf[0..15].
__device__ __forceinline__ float q8_half_dot(const uint8_t* q, const float* xf) {
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(qa & 3) * 8;
    const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3], w4 = wp[4];
    uint32_t d[4] = {__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                     __funnelshift_r(w3, w4, sh)};
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float f[4];
        i8x4_to_f32(d[k], f);
        s = fmaf(f[0], xf[4 * k + 0], s);
        s = fmaf(f[1], xf[4 * k + 1], s);
        s = fmaf(f[2], xf[4 * k + 2], s);
        s = fmaf(f[3], xf[4 * k + 3], s);
    }
    return s;
}

// Q8_0: lane unit = half a block (16 values); block = [f16 d][32 x int8].
__device__ __forceinline__ void dot2_q8(const uint8_t* r0, const uint8_t* r1, bool two, const float* xs, int cols,
                                        int lane, float& a0, float& a1) {
    const int nhb = cols >> 4;
    for (int hb = lane; hb < nhb; hb += 32) {
        const int b = hb >> 1, h = hb & 1;
        float xf[16];
        const float4* xv = reinterpret_cast<const float4*>(xs + hb * 16);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float4 t = xv[k];
            xf[4 * k] = t.x; xf[4 * k + 1] = t.y; xf[4 * k + 2] = t.z; xf[4 * k + 3] = t.w;
        }
        const uint8_t* p0 = r0 + 34 * b;
        a0 = fmaf(f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p0)), q8_half_dot(p0 + 2 + 16 * h, xf), a0);
        if (two) {
            const uint8_t* p1 = r1 + 34 * b;
            a1 = fmaf(f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p1)), q8_half_dot(p1 + 2 + 16 * h, xf),
                      a1);
        }
    }
}

// 32 Q4_0 values (one block: [f16 d][16 bytes], low nibble = element j,
// high nibble = element j+16) dotted with xf[0..31].
__device__ __forceinline__ float q4_block_dot(const uint8_t* q, const float* xf) {
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(qa & 3) * 8;
    const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2], w3 = wp[3], w4 = wp[4];
    uint32_t d[4] = {__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                     __funnelshift_r(w3, w4, sh)};
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float lo[4], hi[4];
        u4x4_to_f32(d[k] & 0x0F0F0F0Fu, lo);
        u4x4_to_f32((d[k] >> 4) & 0x0F0F0F0Fu, hi);
#pragma unroll
        for (int e = 0; e < 4; e++) s = fmaf(lo[e], xf[4 * k + e], s);
#pragma unroll
        for (int e = 0; e < 4; e++) s = fmaf(hi[e], xf[16 + 4 * k + e], s);
    }
    return s;
}

__device__ __forceinline__ void dot2_q4(const uint8_t* r0, const uint8_t* r1, bool two, const float* xs, int cols,
                                        int lane, float& a0, float& a1) {
    const int nb = cols >> 5;
    for (int b = lane; b < nb; b += 32) {
        float xf[32];
        const float4* xv = reinterpret_cast<const float4*>(xs + b * 32);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            float4 t = xv[k];
            xf[4 * k] = t.x; xf[4 * k + 1] = t.y; xf[4 * k + 2] = t.z; xf[4 * k + 3] = t.w;
        }
        const uint8_t* p0 = r0 + 18 * b;
        a0 = fmaf(f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p0)), q4_block_dot(p0 + 2, xf), a0);
        if (two) {
            const uint8_t* p1 = r1 + 18 * b;
            a1 = fmaf(f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(p1)), q4_block_dot(p1 + 2, xf), a1);
        }
    }
}

template <int QT>
__device__ __forceinline__ void dot2(const uint8_t* r0, const uint8_t* r1, bool two, const float* xs, int cols,
                                     int lane, float& a0, float& a1) {
    if (QT == 8)
        dot2_q8(r0, r1, two, xs, cols, lane, a0, a1);
    else
        dot2_q4(r0, r1, two, xs, cols, lane, a0, a1);
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
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = m.nslots;
    const int SB = m.slot_bytes;
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)NS * SB + 128);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + m.xs_floats);
    uint64_t* empty = full + NS;
    float* red = reinterpret_cast<float*>(empty + NS);  // 64 floats
    int* misc = reinterpret_cast<int*>(red + 64);       // 16 ints

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, grid = gridDim.x;

    // A device-resident greedy loop that already produced EOS: arrive on every
    // counter this launch would have arrived on, so later launches' targets
    // stay consistent, and do nothing else.
    if (a.done && *(volatile const int*)a.done) {
        if (threadIdx.x == 0)
            for (int p = a.p_begin; p < a.p_end; p++)
                if (p != kPhasesPerLayer * m.L) red_release_add(m.bar + (size_t)p * kBarStride, 1u);
        return;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
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
                    const int slot = gidx % NS;
                    const uint32_t round = gidx / NS;
                    if (!mbar_wait(&empty[slot], (round & 1) ^ 1, m.err)) { ok = false; break; }
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
    const int cw = warp - 1;                 // consumer warp index
    const int ct = threadIdx.x - 32;         // consumer thread index
    unsigned gbase = 0;                      // chunk index of the phase's first chunk
    bool alive = true;
    Best best{-INFINITY, 0x7fffffff};
    int tok = 0;
    if (!a.mv_w) tok = *a.tok;

    for (int p = a.p_begin; p < a.p_end; p++) {
        const Geom g = phase_geom(m, a, p);
        const Split s = cta_split(g, cta, grid, SB);

        // 1. previous phase complete everywhere
        if (p > a.p_begin) {
            if (ct == 0) {
                bool ok = alive && grid_wait(m.bar + (size_t)(p - 1) * kBarStride, a.epoch * (unsigned)grid + a.skew, m.err);
                misc[0] = ok;
            }
            named_bar_sync(1, kConsumerThreads);
            alive = misc[0] != 0;
        }

        // 2. stage the phase input in shared memory
        if (alive) {
            const LayerDev* Ld = (g.kind != PH_MATVEC && g.kind != PH_LMHEAD) ? &m.layers[g.layer] : nullptr;
            if (g.kind == PH_QKV || g.kind == PH_GATEUP || g.kind == PH_LMHEAD) {
                // RMSNorm (transformer.go:922-932), fused into the stage.
                const float* nw = g.kind == PH_QKV ? Ld->attn_norm : (g.kind == PH_GATEUP ? Ld->ffn_norm : m.out_norm);
                const bool from_embed = (g.kind == PH_QKV && g.layer == 0);
                const int own0 = (int)((long long)cta * m.H / grid), own1 = (int)((long long)(cta + 1) * m.H / grid);
                float ss = 0.0f;
                for (int j = ct; j < m.H; j += kConsumerThreads) {
                    float v;
                    if (from_embed) {
                        v = embed_elem(m, tok, j);
                        if (j >= own0 && j < own1) m.x[j] = v;  // residual stream starts at the embedding
                    } else {
                        v = __ldcg(m.x + j);
                    }
                    xs[j] = v;
                    ss += v * v;
                }
                ss = warp_sum(ss);
                if (lane == 0) red[cw] = ss;
                named_bar_sync(1, kConsumerThreads);
                float tot = 0.0f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) tot += red[w];
                const float r = (float)(1.0 / sqrt((double)(tot / (float)m.H) + (double)m.eps));
                for (int j = ct; j < m.H; j += kConsumerThreads) xs[j] = xs[j] * r * nw[j];
            } else if (g.kind == PH_WO) {
                for (int j = ct; j < m.qd; j += kConsumerThreads) xs[j] = __ldcg(m.attn + j);
            } else if (g.kind == PH_DOWN) {
                for (int j = ct; j < m.FF; j += kConsumerThreads) xs[j] = __ldcg(m.act + j);
            } else if (g.kind == PH_MATVEC) {
                for (int j = ct; j < g.cols; j += kConsumerThreads) xs[j] = a.mv_x[j];
            }
        }
        named_bar_sync(1, kConsumerThreads);

        // 3. the phase's work
        if (g.kind == PH_ATTN) {
            if (alive && cta < g.units) {
                // transformer.go:658-685 for the query heads of one KV head over
                // one slice of the context, online softmax; partials merged by
                // the last slice to finish.
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
                const float scale = (float)(1.0 / sqrt((double)hd));
                for (int i = ct; i < grp * hd; i += kConsumerThreads) {
                    qsm[i] = __ldcg(m.q + kvh * grp * hd + i);
                    osm[i] = 0.0f;
                }
                if (ct < grp) { mrun[ct] = -INFINITY; lrun[ct] = 0.0f; }
                named_bar_sync(1, kConsumerThreads);
                const size_t lay = (size_t)g.layer * m.max_seq * m.kvd;
                for (int tb = t0; tb < t1; tb += kAttnTile) {
                    const int nt = min(kAttnTile, t1 - tb);
                    for (int i = ct; i < grp * kAttnTile; i += kConsumerThreads) {
                        const int h = i / kAttnTile, t = i % kAttnTile;
                        float dot = 0.0f;
                        if (t < nt) {
                            const size_t off = lay + (size_t)(tb + t) * m.kvd + (size_t)kvh * hd;
                            const float* qh = qsm + h * hd;
                            if (m.kv_fp32) {
                                const float* kp = reinterpret_cast<const float*>(m.kcache) + off;
                                for (int d = 0; d < hd; d++) dot = fmaf(qh[d], __ldcg(kp + d), dot);
                            } else {
                                const uint4* kp = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(m.kcache) + off);
                                for (int d8 = 0; d8 < hd / 8; d8++) {
                                    uint4 u = __ldcg(kp + d8);
                                    const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                                    for (int e = 0; e < 4; e++) {
                                        float2 f = __half22float2(hp[e]);
                                        dot = fmaf(qh[d8 * 8 + 2 * e], f.x, dot);
                                        dot = fmaf(qh[d8 * 8 + 2 * e + 1], f.y, dot);
                                    }
                                }
                            }
                            sc[i] = dot * scale;
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
                        const size_t off = lay + (size_t)tb * m.kvd + (size_t)kvh * hd + d;
                        for (int t = 0; t < nt; t++) {
                            float vv = m.kv_fp32 ? __ldcg(reinterpret_cast<const float*>(m.vcache) + off + (size_t)t * m.kvd)
                                                 : __half2float(__ldcg(reinterpret_cast<const __half*>(m.vcache) + off + (size_t)t * m.kvd));
                            o = fmaf(sc[h * kAttnTile + t], vv, o);
                        }
                        osm[i] = o;
                    }
                    named_bar_sync(1, kConsumerThreads);
                }
                // write this slice's partial (o unnormalised, m, l)
                for (int i = ct; i < grp * (hd + 2); i += kConsumerThreads) {
                    const int h = i / (hd + 2), d = i % (hd + 2);
                    const float v = d < hd ? osm[h * hd + d] : (d == hd ? mrun[h] : lrun[h]);
                    m.part[((size_t)(kvh * grp + h) * kMaxSplits + sidx) * (hd + 2) + d] = v;
                }
                named_bar_sync(1, kConsumerThreads);
                if (ct == 0) {
                    __threadfence();
                    unsigned old = atom_acq_rel_add(m.head_ctr + kvh * kBarStride, 1u);
                    misc[1] = (old == (unsigned)(S - 1));
                }
                named_bar_sync(1, kConsumerThreads);
                if (misc[1]) {
                    // last slice: log-sum-exp merge of all S partials
                    for (int i = ct; i < grp * hd; i += kConsumerThreads) {
                        const int h = i / hd, d = i % hd;
                        const float* ph = m.part + (size_t)(kvh * grp + h) * kMaxSplits * (hd + 2);
                        float M = -INFINITY;
                        for (int s2 = 0; s2 < S; s2++) M = fmaxf(M, __ldcg(ph + s2 * (hd + 2) + hd));
                        float Lsum = 0.0f, o = 0.0f;
                        for (int s2 = 0; s2 < S; s2++) {
                            const float ms = __ldcg(ph + s2 * (hd + 2) + hd);
                            const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
                            Lsum = fmaf(__ldcg(ph + s2 * (hd + 2) + hd + 1), w, Lsum);
                            o = fmaf(__ldcg(ph + s2 * (hd + 2) + d), w, o);
                        }
                        m.attn[(kvh * grp + h) * hd + d] = o / Lsum;
                    }
                    if (ct == 0) atomicExch(m.head_ctr + kvh * kBarStride, 0u);
                }
            }
        } else {
            for (int k = 0; k < s.nchunks; k++) {
                const unsigned gidx = gbase + k;
                if ((int)(gidx % kConsumerWarps) != cw) continue;
                const int slot = gidx % NS;
                if (!mbar_wait(&full[slot], (gidx / NS) & 1, m.err)) alive = false;
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
                        float a0 = 0.0f, a1 = 0.0f;
                        dot2<QT>(ra, rb2, two, xs, g.cols, lane, a0, a1);
                        a0 = warp_sum(a0);
                        a1 = warp_sum(a1);
                        if (lane == 0) {
                            switch (g.kind) {
                                case PH_QKV: {
                                    // bias (transformer.go:632-646), RoPE on interleaved
                                    // pairs (936-951), KV append (654-656)
                                    const LayerDev& Ld = m.layers[g.layer];
                                    if (Ld.bqkv) { a0 += Ld.bqkv[rowa]; a1 += Ld.bqkv[rowa + 1]; }
                                    const int pos = a.pos;
                                    if (rowa < m.qd + m.kvd) {
                                        const int i = (rowa % m.hd) >> 1;
                                        const float c = m.rope_cos[(size_t)pos * (m.hd / 2) + i];
                                        const float sn = m.rope_sin[(size_t)pos * (m.hd / 2) + i];
                                        const float x0 = a0, x1 = a1;
                                        a0 = x0 * c - x1 * sn;
                                        a1 = x0 * sn + x1 * c;
                                    }
                                    if (rowa < m.qd) {
                                        m.q[rowa] = a0;
                                        m.q[rowa + 1] = a1;
                                    } else {
                                        const bool isk = rowa < m.qd + m.kvd;
                                        const int col = rowa - m.qd - (isk ? 0 : m.kvd);
                                        const size_t off = ((size_t)g.layer * m.max_seq + pos) * m.kvd + col;
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
                                case PH_GATEUP: {
                                    // SwiGLU (transformer.go:725-727, 954-956)
                                    const float gt = a0, up = a1;
                                    m.act[rowa] = gt / (1.0f + expf(-gt)) * up;
                                    break;
                                }
                                case PH_WO:
                                case PH_DOWN:
                                    // residual (transformer.go:576-578, 591-593)
                                    m.x[rowa] = __ldcg(m.x + rowa) + a0;
                                    if (two) m.x[rowa + 1] = __ldcg(m.x + rowa + 1) + a1;
                                    break;
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
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
            gbase += s.nchunks;
        }

        // 4. this CTA's part of the phase is done
        named_bar_sync(1, kConsumerThreads);
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
                unsigned* ctr = m.bar + (size_t)(kPhasesPerLayer * m.L + 1) * kBarStride;
                unsigned old = atom_acq_rel_add(ctr, 1u);
                if (old == (unsigned)(grid - 1)) {
                    Best f{-INFINITY, 0x7fffffff};
                    for (int c2 = 0; c2 < grid; c2++) {
                        float v = __ldcg(m.best_val + c2);
                        int i = __ldcg(m.best_idx + c2);
                        if (better(v, i, f.v, f.i)) { f.v = v; f.i = i; }
                    }
                    if (f.i == 0x7fffffff) f.i = 0;
                    *m.token = f.i;
                    if (a.out_ids) a.out_ids[a.step] = f.i;
                    if (a.done && f.i == a.eos) *a.done = 1;
                    atomicExch(ctr, 0u);
                }
            }
        } else if (ct == 0 && a.p_end - a.p_begin > 1) {
            red_release_add(m.bar + (size_t)p * kBarStride, 1u);
        }
    }
}

}  // namespace

size_t decode_smem_bytes(const ModelDev& m) {
    return (size_t)m.nslots * m.slot_bytes + 128 + (size_t)m.xs_floats * 4 + 16 * (size_t)m.nslots + 64 * 4 +
           16 * 4;
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
