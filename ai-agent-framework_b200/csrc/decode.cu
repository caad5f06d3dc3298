// The decode step: one cooperative, persistent kernel per token.
//
// Replaces transformer.go:519-739 (forward / transformerLayer / selfAttention /
// feedForward) and the Q8_0 matvec of transformer.go:810-892 for B = 1.
//
// Per layer four phases: QA (q, k, v rows + attention), WO, GATEUP, DOWN;
// then the LM head.  Layout of one CTA (one per SM):
//   warp 0, lanes 0-3 producer: walks the static work plan of every phase of
//                    the launch (per-CTA plans in shared memory) and streams
//                    this CTA's chunks of the tiled weights with 1-D TMA bulk
//                    copies into a ring of shared-memory slots.  Weights never
//                    depend on activations, so it runs ahead across phases,
//                    limited by the ring.
//   warps 1..12      consumers, per phase:
//                    1. stage: gather the phase input from the previous
//                       phase's LL words (the poll is the load), multiplied by
//                       the RMSNorm gain, or decode the embedding row, or
//                       merge the attention splits, and split it as it
//                       arrives into three int8 planes per 32-element block
//                       (x ~ s * (p0 + p1/128 + p2/16384), ~21 significant
//                       bits); the QKV bias and RoPE row arrive by cp.async;
//                    2. rows: int8 tensor-core dot products (mma m16n8k32):
//                       the 16-row weight tile straight from the ring (A
//                       operand, no dequantisation) times the x planes (B
//                       operand); the int32 per-block sums are scaled by the
//                       weight and x block scales and accumulated in fp32;
//                    3. epilogue, one thread per output: RMSNorm scale, bias +
//                       RoPE + KV append, SwiGLU, residual add, logits +
//                       argmax, and the LL stores that hand the outputs on.
//                    In the QA phase the q CTAs (one per query head and
//                    context split) then attend over K/V tiles that cp.async
//                    copied into shared memory during the phase; the last
//                    split also takes the new position.
// Each CTA keeps the residual-stream rows it owns (the same rows in every Wo
// and down phase) in shared memory.  Every wait is bounded (globaltimer) and
// reports B2_ERR_TIMEOUT through the device error flag instead of hanging.
// The kernel-level matvec entry point (ggml block layout, caller memory) runs
// the same kernel in a one-phase mode with an fp32 dequantising dot.
#include <cuda_runtime.h>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "model.h"

namespace b2 {

namespace {

constexpr uint64_t kWaitLimitNs = 2000000000ull;      // 2 s for any consumer wait
constexpr uint64_t kProducerLimitNs = 8000000000ull;  // producer slot waits outlast consumer polls
// A wait reads the device error flag (another CTA gave up) only once it has
// lasted this long: the flag is a global load, an L2 round trip that would
// otherwise sit between two polls of every waiting thread and delay the
// moment it sees its data.  Normal hand-offs end well within it.
constexpr uint64_t kErrCheckNs = 20000ull;
// Attention split partials the Wo stage polls per round (merge_planes).
constexpr int kMergePerRound = 2;
constexpr int kConsumerThreads = 32 * kConsumerWarps;

// ---------------------------------------------------------------------------
// phase geometry
// ---------------------------------------------------------------------------

// A weight phase of the model: a tiled matrix, its rows and 32-blocks per
// row.  The gate/up matrix has 2*FF rows (gate and up interleaved 8 rows at
// a time: tile t = gate rows 8t .. 8t+7, then up rows 8t .. 8t+7).
struct TGeom {
    int kind;
    int layer;
    int sub;            // lm_head sub-phase
    const uint8_t* w;
    int rows;           // real matrix rows
    int tiles;          // ceil(rows / kTileRows)
    int nb;             // K / 32
};

__device__ __forceinline__ TGeom phase_geom(const ModelDev& m, const LayerDev* layers, int p) {
    TGeom g{};
    if (p >= kPhasesPerLayer * m.L) {
        g.kind = PH_LMHEAD;
        g.layer = m.L;
        g.sub = p - kPhasesPerLayer * m.L;
        g.w = m.lm_head;
        g.rows = m.V;
        g.nb = m.H / 32;
    } else {
        g.layer = p / kPhasesPerLayer;
        g.kind = p % kPhasesPerLayer;
        const LayerDev& L = layers[g.layer];
        switch (g.kind) {
            case PH_QA: g.w = L.wqkv; g.rows = m.qd + 2 * m.kvd; g.nb = m.H / 32; break;
            case PH_WO: g.w = L.wo; g.rows = m.H; g.nb = m.qd / 32; break;
            case PH_GATEUP: g.w = L.wgu; g.rows = 2 * m.FF; g.nb = m.H / 32; break;
            default: g.w = L.wd; g.rows = m.H; g.nb = m.FF / 32; break;  // PH_DOWN
        }
    }
    g.tiles = (g.rows + kTileRows - 1) / kTileRows;
    return g;
}

// This CTA's work plan in weight phase g (precomputed on the host).
__device__ __forceinline__ TPlan phase_plan(const TPlan* plans, const TGeom& g, int S) {
    return plans[plan_slot(g.kind, g.kind == PH_LMHEAD ? g.sub : S)];
}

// The matvec entry point's single phase: rows of a ggml-layout matrix.
struct Geom {
    const uint8_t* w;
    int rb;
    int cols;
    int units;
};

// Static split of the matvec rows over the grid and of a CTA's share into
// chunks that fit one ring slot.
struct Split {
    int u0, n, cu, nchunks;
};

__device__ __forceinline__ Split cta_split(const Geom& g, int cta, int grid, int slot_bytes) {
    Split s;
    s.u0 = (int)((long long)cta * g.units / grid);
    int u1 = (int)((long long)(cta + 1) * g.units / grid);
    s.n = u1 - s.u0;
    if (s.n <= 0) {
        s.cu = 1;
        s.nchunks = 0;
        return s;
    }
    int max_units = (slot_bytes - 32) / g.rb;
    int spread = (s.n + kConsumerWarps - 1) / kConsumerWarps;
    s.cu = max(1, min(max_units, spread));
    s.nchunks = (s.n + s.cu - 1) / s.cu;
    return s;
}

__device__ __forceinline__ void set_err(int* err, int code) { atomicCAS(err, 0, code); }

// Producer: bounded wait for a free ring slot.  The error flag (a global
// load, an L2 round trip) is only read while the slot is still taken, so an
// unblocked producer issues copies back to back; a blocked one gives up as
// soon as any CTA reported an error.
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        const uint64_t dt = global_ns() - t0;
        if (dt > kErrCheckNs && *(volatile int*)err) return false;
        if (dt > kProducerLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ unsigned ld_acquire_cta(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta(unsigned* p, unsigned v) {
    asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Consumer: bounded wait for chunk gidx to land.  The chunk must first have
// been issued (*issued > gidx): only then has its slot's previous round
// completed, so the parity wait cannot mistake that round for this one (a
// warp may otherwise reach a slot a full ring round before the producer
// does).  *pstop is the index of the first chunk the producer did not issue
// (it stops early only after an error); such chunks are skipped instead of
// waited for, and every chunk that was issued is waited for, so no bulk copy
// is left in flight at exit.
__device__ __forceinline__ bool chunk_wait(uint64_t* bar, uint32_t parity, unsigned gidx, const volatile unsigned* pstop,
                                           const unsigned* issued, int* err) {
    uint64_t t0 = 0;
    while (ld_acquire_cta(issued) <= gidx) {
        if (gidx >= *pstop) return false;
        const uint64_t now = global_ns();
        if (t0 == 0) t0 = now;
        if (now - t0 > kWaitLimitNs) {
            set_err(err, B2_ERR_TIMEOUT);
            return false;
        }
    }
    if (mbar_try_wait(bar, parity)) return true;
    if (t0 == 0) t0 = global_ns();
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
// decoded from its block of the tiled matrix (out-of-range ids embed to zero).
template <int QT>
__device__ __forceinline__ float embed_val(const uint8_t* embd, int V, int H, int Vp, int tok, int j) {
    if (tok < 0 || tok >= V) return 0.0f;
    const int nb = H / 32, b = j >> 5, e = j & 31;
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(embd + tiled_soff(tok, b, nb, Vp, QT)));
    if (QT == 8) return d * (float)(int8_t)embd[tiled_qoff(tok, b, e, nb, 8)];
    const uint8_t byte = embd[tiled_qoff(tok, b, e & 15, nb, 2)];
    const int nib = (e < 16) ? (byte & 15) : (byte >> 4);
    return d * (float)(nib - 8);
}
template <int QT>
__device__ __forceinline__ float embed_elem(const ModelDev& m, int tok, int j) {
    return embed_val<QT>(m.tok_embd, m.Vemb, m.H, m.Vp_emb, tok, j);
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
__device__ __forceinline__ int cb_bias(const ModelDev&) { return 0; }
__device__ __forceinline__ int cb_cos(const ModelDev&) { return kMaxQkvRows + 4; }
__device__ __forceinline__ int cb_sin(const ModelDev& m) { return kMaxQkvRows + 4 + m.hd / 2; }

// Attention scratch (at the shared byte offset the QA phase passes): q [hd]
// floats, the per-warp partials [kConsumerWarps][hd + 2] floats (o, m, l),
// their merge weights [16] floats, the new position's k and v LL words
// [2 * hd], then one K tile [TP][hd*ES + 16 bytes] and one V tile [TP][hd*ES].
struct AttnMap {
    float* aq;
    float* wpart;
    uint8_t* ktile;
    uint8_t* vtile;
};
template <int ES>
__device__ __forceinline__ AttnMap attn_map(float* base, int hd, int TP) {
    AttnMap r;
    r.aq = base;
    r.wpart = r.aq + hd;
    r.ktile = reinterpret_cast<uint8_t*>(r.wpart + kConsumerWarps * (hd + 2) + 16 + 4 * hd);
    r.vtile = r.ktile + (size_t)TP * (hd * ES + 16);
    return r;
}

// cp.async copies of the cached K and V rows of positions [tb, tb + nt) into
// the tile buffers (one committed group).
template <bool F32>
__device__ __noinline__ void attn_load_tile(const uint8_t* kg, const uint8_t* vg, uint32_t gs, int hd, int TP, int tb,
                                            int nt, uint32_t scratch_off) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int ES = F32 ? 4 : 2;
    const AttnMap am = attn_map<ES>(reinterpret_cast<float*>(smem + scratch_off), hd, TP);
    const int ct = threadIdx.x - 32;
    const int rowb = hd * ES, KS = rowb + 16, pieces = rowb / 16;
#pragma unroll 1
    for (int i = ct; i < nt * pieces; i += kConsumerThreads) {
        const int t = i / pieces, c = i - t * pieces;
        cp_async16(am.ktile + (size_t)t * KS + c * 16, kg + (size_t)(tb + t) * gs + c * 16);
        cp_async16(am.vtile + (size_t)t * rowb + c * 16, vg + (size_t)(tb + t) * gs + c * 16);
    }
    cp_async_commit();
}

// N (a multiple of 4) consecutive K or V elements of one cached row (fp16 or
// fp32) as floats.
template <bool F32, int N>
__device__ __forceinline__ void attn_row(const uint8_t* p, float* f) {
    if (F32) {
#pragma unroll
        for (int e = 0; e < N; e += 4) {
            const float4 x = *reinterpret_cast<const float4*>(p + 4 * e);
            f[e] = x.x;
            f[e + 1] = x.y;
            f[e + 2] = x.z;
            f[e + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < N; e += 4) {
            const uint2 u = *reinterpret_cast<const uint2*>(p + 2 * e);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            f[e] = a.x;
            f[e + 1] = a.y;
            f[e + 2] = b.x;
            f[e + 3] = b.y;
        }
    }
}

// The attention of one query head over the cached positions [t0, t1) (one
// context split), transformer.go:658-685, for head dimension HD.  q (after
// RoPE) is already in the scratch; the first tile's copies were issued before
// the phase's input poll, so they overlapped the hand-off and the q
// projection.  A group of LP = HD / DL lanes takes one position at a time
// and keeps its own online softmax: each lane holds DL elements of q, of the
// position's k and v rows and of the running output, so a step needs only
// the LP-lane reduction of q . k (a warp advances 32 / LP positions per
// step; DL = 8 measured best for HD 64 and 128: fewer groups to merge at the
// end than with 16 lanes of 4, shorter steps than with 4 lanes of 16).  The streams are merged at the end, first across the groups of a
// warp (shuffles), then across warps (shared memory, one barrier).  The last
// split (`last`) also takes the new position, whose k (after RoPE) and v are
// the LL words knew[0 .. HD) and knew[kvd .. kvd + HD) that the k / v CTAs
// publish in this phase (exact fp32, as the reference attends to them); they
// are copied into the scratch before the tile loop.  Writes the split partial
// (o unnormalised, m, l) as LL words for the Wo phase's merge.  Returns 0 if
// the new position's words never came (error flag set).  Not inlined, so its
// registers do not add to the kernel's peak.
template <bool F32, int HD, int DL>
__device__ __noinline__ int attn_phase(const uint8_t* kg, const uint8_t* vg, uint32_t gs, int TP, int t0, int t1,
                                       unsigned tag_out, uint2* out, uint32_t scratch_off, const uint2* knew, int kvd,
                                       int last, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int ES = F32 ? 4 : 2;
    constexpr int LP = HD / DL, G = 32 / LP;  // lanes per position, positions per step
    static_assert(LP >= 1 && LP <= 32, "lanes per position");
    const int ct = threadIdx.x - 32, lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 1;
    const AttnMap am = attn_map<ES>(reinterpret_cast<float*>(smem + scratch_off), HD, TP);
    constexpr int rowb = HD * ES, KS = rowb + 16;
    const float scale = 1.0f / sqrtf((float)HD);
    const int grp = lane / LP, d0 = (lane % LP) * DL;
    float q[DL], o[DL];
#pragma unroll
    for (int k = 0; k < DL; k++) {
        q[k] = am.aq[d0 + k] * scale;
        o[k] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    // the new position's words (last split): copied now (cp.async, through
    // L2) into the scratch and checked after the tiles
    const bool nw = last && cw == 0;
    uint2* kn_s = reinterpret_cast<uint2*>(am.wpart + kConsumerWarps * (HD + 2) + 16);  // [2 * HD] words
    if (nw) {
#pragma unroll 1
        for (int i = lane; i < HD; i += 32)
            cp_async16(kn_s + 2 * i, knew + 2 * (i % (HD / 2)) + (i < HD / 2 ? 0 : kvd));
    }
    cp_async_commit();
    cp_async_wait_1();  // the first K/V tile (issued at phase start), not these words
    named_bar_sync(1, kConsumerThreads);
#pragma unroll 1
    for (int tb = t0; tb < t1; tb += TP) {
        const int nt = min(TP, t1 - tb);
        if (tb != t0) {
            named_bar_sync(1, kConsumerThreads);  // the previous tile is no longer read
            attn_load_tile<F32>(kg, vg, gs, HD, TP, tb, nt, scratch_off);
            cp_async_wait();
            named_bar_sync(1, kConsumerThreads);
        }
#pragma unroll 1
        for (int tw = cw * G; tw < nt; tw += kConsumerWarps * G) {  // warp-uniform trip count
            const int tp = tw + grp;
            const bool on = tp < nt;
            const int tr = on ? tp : tw;
            float kf[DL], vf[DL];
            attn_row<F32, DL>(am.ktile + (size_t)tr * KS + d0 * ES, kf);
            attn_row<F32, DL>(am.vtile + (size_t)tr * rowb + d0 * ES, vf);
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int k = 0; k < DL; k += 2) {
                s0 = fmaf(q[k], kf[k], s0);
                s1 = fmaf(q[k + 1], kf[k + 1], s1);
            }
            float sc = s0 + s1;
#pragma unroll
            for (int off = 1; off < LP; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
            if (on) {
                // one exponential per position: the larger of (m, sc) keeps weight 1
                const float e = __expf(-fabsf(sc - m));  // m = -inf: e = 0
                const bool up = sc > m;
                const float c = up ? e : 1.0f, pr = up ? 1.0f : e;
                l = fmaf(l, c, pr);
#pragma unroll
                for (int k = 0; k < DL; k++) o[k] = fmaf(pr, vf[k], o[k] * c);
                m = up ? sc : m;
            }
        }
    }
    int ok = 1;
    if (nw) {
        // the new position, in warp 0's first lane group; stale words are read
        // again from global memory
        cp_async_wait();
        __syncwarp();
        uint64_t w0 = 0;
        for (;;) {
            bool got = true;
#pragma unroll 1
            for (int i = lane; i < 2 * HD; i += 32) got &= kn_s[i].y == tag_out;
            if (__all_sync(0xffffffffu, got)) break;
            const uint64_t now = global_ns();
            if (w0 == 0) w0 = now;
            if (now - w0 > kWaitLimitNs) {
                set_err(err, B2_ERR_TIMEOUT);
                ok = 0;
                break;
            }
            if (now - w0 > kErrCheckNs && *(volatile int*)err) {
                ok = 0;
                break;
            }
            __syncwarp();
            for (int i = lane; i < HD; i += 32) {
                const uint4 kw = ll_load2(knew + 2 * (i % (HD / 2)) + (i < HD / 2 ? 0 : kvd));
                kn_s[2 * i] = make_uint2(kw.x, kw.y);
                kn_s[2 * i + 1] = make_uint2(kw.z, kw.w);
            }
            __syncwarp();
        }
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int k = 0; k < DL; k += 2) {
            s0 = fmaf(q[k], __uint_as_float(kn_s[d0 + k].x), s0);
            s1 = fmaf(q[k + 1], __uint_as_float(kn_s[d0 + k + 1].x), s1);
        }
        float sc = s0 + s1;
#pragma unroll
        for (int off = 1; off < LP; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
        if (grp == 0) {
            const float e = __expf(-fabsf(sc - m));
            const bool up = sc > m;
            const float c = up ? e : 1.0f, pr = up ? 1.0f : e;
            l = fmaf(l, c, pr);
#pragma unroll
            for (int k = 0; k < DL; k++) o[k] = fmaf(pr, __uint_as_float(kn_s[HD + d0 + k].x), o[k] * c);
            m = up ? sc : m;
        }
    }
    // merge the lane groups of this warp, then publish the warp's stream
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, off), lo = __shfl_xor_sync(0xffffffffu, l, off);
        const float mx = fmaxf(m, mo);
        const float c1 = m == -INFINITY ? 0.0f : __expf(m - mx), c2 = mo == -INFINITY ? 0.0f : __expf(mo - mx);
        l = l * c1 + lo * c2;
#pragma unroll
        for (int k = 0; k < DL; k++) o[k] = o[k] * c1 + __shfl_xor_sync(0xffffffffu, o[k], off) * c2;
        m = mx;
    }
    float* wp = am.wpart + cw * (HD + 2);
    if (grp == 0) {
#pragma unroll
        for (int k = 0; k < DL; k++) wp[d0 + k] = o[k];
        if (lane == 0) {
            wp[HD] = m;
            wp[HD + 1] = l;
        }
    }
    named_bar_sync(1, kConsumerThreads);
    float* wc = am.wpart + kConsumerWarps * (HD + 2);  // [kConsumerWarps] weights, then M
    if (ct < kConsumerWarps) {
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) mx = fmaxf(mx, am.wpart[w * (HD + 2) + HD]);
        const float mw = am.wpart[ct * (HD + 2) + HD];
        wc[ct] = mw == -INFINITY ? 0.0f : __expf(mw - mx);
        if (ct == 0) wc[kConsumerWarps] = mx;
    }
    named_bar_sync(1, kConsumerThreads);
    if (ct < HD + 2) {
        const int col = ct == HD ? HD + 1 : ct;  // (the m slot carries M instead)
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) acc = fmaf(am.wpart[w * (HD + 2) + col], wc[w], acc);
        ll_store(out + ct, ct == HD ? wc[kConsumerWarps] : acc, tag_out);
    }
    return ok;
}

// mma.m16n8k32 with int32 accumulate: A = 16 weight rows x 32 (s8 for Q8_0,
// u8 nibbles for Q4_0), B = x planes in columns 0-2; c01 / c23 start the
// accumulators of output columns 2t, 2t+1.
template <bool AU8>
__device__ __forceinline__ void mma_k32(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                        uint32_t c0, uint32_t c1, uint32_t& d0, uint32_t& d1, uint32_t& d2,
                                        uint32_t& d3) {
    if (AU8)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// 1.5 * 2^23 as float bits: an int32 accumulator started here holds the bit
// pattern of the float 1.5 * 2^23 + P for |P| < 2^22, so P comes back exactly
// with one subtraction (no int -> float conversion instruction).
constexpr uint32_t kAccMagic = 0x4B400000u;
constexpr float kAccMagicF = 12582912.0f;

// Dot products of one 16-row tile over nbc blocks against the x planes of
// blocks xb0 .. xb0 + nbc.  q: shared address of the tile's quants
// ([nbc][16 rows][QB]), sc_off: smem offset of its scales ([nbc][16] f16 in
// (g, g + 8) pairs).  Lane (g, t) accumulates planes 2t, 2t+1 of rows g and
// g + 8; the planes are weighted (1, 2^-7, 2^-14) and summed over t at the
// end.  Returns rows g and g + 8 in the lanes with t == 0.  Not inlined: the
// kernel's other phases then do not share its registers.
template <int QT>
__device__ __noinline__ float2 tile_dot(uint32_t q, uint32_t sc_off, int nbc, uint32_t xq_off, uint32_t xsc_off,
                                        uint32_t xsm_off, int xb0) {
    constexpr int QB = QT == 8 ? 32 : 16;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint8_t* sc = smem + sc_off;
    const uint2* xq = reinterpret_cast<const uint2*>(smem + xq_off);
    const float* xsc = reinterpret_cast<const float*>(smem + xsc_off);
    const int* xsm = reinterpret_cast<const int*>(smem + xsm_off);
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // ldmatrix row address of this lane
    uint32_t lo;
    if (QT == 8) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8, half = (lane >> 4) & 1;
        lo = (uint32_t)(row * 32 + ((half ^ ((row >> 2) & 1)) << 4));  // rows with bit 2 set: halves swapped
    } else {
        lo = (uint32_t)((lane & 15) * 16);
    }
    const unsigned long long m2 = f2_pack(-kAccMagicF, -kAccMagicF);
    unsigned long long acc0 = f2_pack(0.0f, 0.0f), acc1 = acc0;
#pragma unroll 2
    for (int b = 0; b < nbc; b++) {
        uint32_t a0, a1, a2, a3;
        uint32_t c0 = kAccMagic, c1 = kAccMagic;
        if (QT == 8) {
            ldsm_x4(q + (uint32_t)(b * 16 * QB) + lo, a0, a1, a2, a3);
        } else {
            uint32_t w0, w1;
            ldsm_x2(q + (uint32_t)(b * 16 * QB) + lo, w0, w1);
            a0 = w0 & 0x0F0F0F0Fu;         // row g, elements 4t .. 4t+3 (low nibbles)
            a1 = w1 & 0x0F0F0F0Fu;         // row g + 8
            a2 = (w0 >> 4) & 0x0F0F0F0Fu;  // row g, elements 16+4t .. (high nibbles)
            a3 = (w1 >> 4) & 0x0F0F0F0Fu;
            // (q - 8) . p = q . p - 8 sum(p): the accumulator starts of planes
            // 2t, 2t + 1 were stored with the planes
            if (t < 2) {
                const uint2 cs = *reinterpret_cast<const uint2*>(xsm + (xb0 + b) * 4 + 2 * t);
                c0 = cs.x;
                c1 = cs.y;
            }
        }
        const uint2 bv = lane < 12 ? xq[(xb0 + b) * 12 + lane] : make_uint2(0u, 0u);
        uint32_t d0, d1, d2, d3;
        mma_k32<QT != 8>(a0, a1, a2, a3, bv.x, bv.y, c0, c1, d0, d1, d2, d3);
        const float2 ds = __half22float2(*reinterpret_cast<const __half2*>(sc + b * 32 + 4 * g));  // rows g, g + 8
        const float xs = xsc[xb0 + b];
        const float s0 = ds.x * xs, s1 = ds.y * xs;
        acc0 = f2_fma(f2_pack(s0, s0), f2_add(f2_pack(__uint_as_float(d0), __uint_as_float(d1)), m2), acc0);
        acc1 = f2_fma(f2_pack(s1, s1), f2_add(f2_pack(__uint_as_float(d2), __uint_as_float(d3)), m2), acc1);
    }
    // lane t holds planes 2t, 2t+1: weights 1, 2^-7 (t = 0), 2^-14, 0 (t = 1)
    const float p0 = t == 0 ? 1.0f : (t == 1 ? 6.103515625e-05f : 0.0f);
    const float p1 = t == 0 ? 0.0078125f : 0.0f;
    const float2 u = f2_unpack(acc0), v = f2_unpack(acc1);
    float y0 = u.x * p0 + u.y * p1, y1 = v.x * p0 + v.y * p1;
    y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
    return make_float2(y0, y1);
}

// Quarter-block of 8 values -> int8 planes (see quantize_planes); the four
// threads of a block (consecutive lanes) agree on its max with two shuffles.
// Every lane of the warp must call it.
__device__ __forceinline__ void planes8(const float* v, bool on, int b, int sub, uint8_t* xqb, float* xsc, int* xsm,
                                        bool sums) {
    const float M = kAccMagicF;
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; e++) amax = fmaxf(amax, on ? fabsf(v[e]) : 0.0f);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float inv = amax > 0.0f ? __fdividef(127.0f, amax) : 0.0f;
    uint32_t by[3][8];
    int sg[3] = {0, 0, 0};
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const float q = on ? v[e] * inv : 0.0f;
        const float f0 = q + M, r0 = f0 - M;
        const float q1 = (q - r0) * 128.0f;
        const float f1 = q1 + M, r1 = f1 - M;
        const float f2 = (q1 - r1) * 128.0f + M;
        by[0][e] = __float_as_uint(f0);
        by[1][e] = __float_as_uint(f1);
        by[2][e] = __float_as_uint(f2);
        if (sums) {
            sg[0] += (int)r0;
            sg[1] += (int)r1;
            sg[2] += (int)(f2 - M);
        }
    }
    if (sums) {
#pragma unroll
        for (int gq = 0; gq < 3; gq++) {
            sg[gq] += __shfl_xor_sync(0xffffffffu, sg[gq], 1);
            sg[gq] += __shfl_xor_sync(0xffffffffu, sg[gq], 2);
        }
    }
    if (on) {
        // elements sub*8 + 0..7: word w = sub / 2 (a0 or a2), lane groups
        // t0 = (sub & 1) * 2 and t0 + 1, bytes e & 3
        const int w = sub >> 1, t0 = (sub & 1) * 2;
        uint32_t* xw = reinterpret_cast<uint32_t*>(xqb + b * 96);
#pragma unroll
        for (int gq = 0; gq < 3; gq++) {
            const uint32_t lo = __byte_perm(__byte_perm(by[gq][0], by[gq][1], 0x0040),
                                            __byte_perm(by[gq][2], by[gq][3], 0x0040), 0x5410);
            const uint32_t hi = __byte_perm(__byte_perm(by[gq][4], by[gq][5], 0x0040),
                                            __byte_perm(by[gq][6], by[gq][7], 0x0040), 0x5410);
            xw[(gq * 4 + t0) * 2 + w] = lo;
            xw[(gq * 4 + t0 + 1) * 2 + w] = hi;
        }
        if (sub == 0) {
            xsc[b] = amax * (1.0f / 127.0f);
            if (sums) {
                // Q4_0 accumulator starts: (q - 8) . p = q . p - 8 sum(p)
                *reinterpret_cast<uint4*>(xsm + b * 4) =
                    make_uint4(kAccMagic - 8u * (uint32_t)sg[0], kAccMagic - 8u * (uint32_t)sg[1],
                               kAccMagic - 8u * (uint32_t)sg[2], kAccMagic);
            }
        }
    }
}

// The phase input straight into int8 planes, without staging it as floats:
// each thread polls the LL words of whole quarter-blocks (8 values = four
// 16-byte loads), multiplies them by the norm gains (global `gain`; none when
// null) and splits them (planes8).  The RMSNorm scale is one scalar per
// token, so it is applied to the dot products instead (the dot is linear); the
// sum of squares of the raw values is returned for it.  With NADD > 0 each
// value is src + add[0] + ... + add[NADD - 1] (arrays add_stride words apart,
// the same tag, all polled in the same round): the residual stream after a
// down phase split over K.  With `embed` set the
// values are the embedding of token tok (layer 0; an id outside the
// vocabulary embeds to zero) instead of LL words.  A
// failed or timed-out poll sets ok = 0 but the loop runs to the end, so every
// lane reaches every shuffle.  Not inlined (register peak, code size).
template <int QT, int NADD>
__device__ __noinline__ GatherRes gather_planes(const uint2* src, int nbk, unsigned tag, int* err, int embed, int tok,
                                                const uint8_t* embd, int V, int H, int Vp, uint32_t xq_off,
                                                uint32_t xsc_off, uint32_t xsm_off, const float* gain, int sums,
                                                const uint2* add, int add_stride) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* xqb = smem + xq_off;
    float* xsc = reinterpret_cast<float*>(smem + xsc_off);
    int* xsm = reinterpret_cast<int*>(smem + xsm_off);
    const int ct = threadIdx.x - 32;
    bool ok = true;
    uint64_t t0 = 0;
    float ss = 0.0f;
#pragma unroll 1
    for (int base = 0; base < 4 * nbk; base += kConsumerThreads) {
        const int i = base + ct;
        const bool on = i < 4 * nbk;
        if (!__any_sync(0xffffffffu, on)) continue;  // (warp-uniform: planes8 shuffles)
        const int b = i >> 2, sub = i & 3, j0 = b * 32 + sub * 8;
        float v[8];
        float4 g0 = make_float4(1.0f, 1.0f, 1.0f, 1.0f), g1 = g0;
        if (on && gain) {  // issued before the poll, so their latency overlaps it
            g0 = __ldg(reinterpret_cast<const float4*>(gain + j0));
            g1 = __ldg(reinterpret_cast<const float4*>(gain + j0 + 4));
        }
        if (on && embed) {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = embed_val<QT>(embd, V, H, Vp, tok, j0 + e);
        } else if (on) {
            const uint2* sp = src + j0;
            uint4 w[4], wa[NADD > 0 ? NADD : 1][4];
            for (;;) {
                bool got = true;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    w[k] = ll_load2(sp + 2 * k);
                    got &= (w[k].y == tag) & (w[k].w == tag);
                }
#pragma unroll
                for (int a = 0; a < NADD; a++)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        wa[a][k] = ll_load2(add + (size_t)a * add_stride + j0 + 2 * k);
                        got &= (wa[a][k].y == tag) & (wa[a][k].w == tag);
                    }
                if (got || !ok) break;
                const uint64_t now = global_ns();
                if (t0 == 0) t0 = now;
                if (now - t0 > kWaitLimitNs) {
                    set_err(err, B2_ERR_TIMEOUT);
                    ok = false;
                } else if (now - t0 > kErrCheckNs && *(volatile int*)err) {
                    ok = false;
                }
            }
#pragma unroll
            for (int k = 0; k < 4; k++) {
                v[2 * k] = __uint_as_float(w[k].x);
                v[2 * k + 1] = __uint_as_float(w[k].z);
            }
            // the down-phase partials, added in slice order (every reader of
            // the residual stream adds them in this order)
#pragma unroll
            for (int a = 0; a < NADD; a++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    v[2 * k] += __uint_as_float(wa[a][k].x);
                    v[2 * k + 1] += __uint_as_float(wa[a][k].z);
                }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.0f;
        }
        if (on) {
            const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                ss += v[e] * v[e];
                v[e] *= gg[e];
            }
        }
        planes8(v, on, b, sub, xqb, xsc, xsm, sums != 0);
    }
    return GatherRes{ss, ok ? 1 : 0};
}

// The Wo phase input straight into int8 planes: the attention output of
// every head, merged from its S context-split partials (o unnormalised, m, l;
// LL words [nh][S][hd + 2]) as transformer.go:664-685 over all positions:
// o = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M), M = max_s m_s (the new
// position is part of the last split, so the sum is positive).  Each thread
// merges the 8 outputs of one quarter-block (one head, hd >= 16) up to
// kMergePerRound splits per poll, rescaling as the maximum grows, and splits them (planes8).  Polls
// and fails like gather_planes (every lane reaches every shuffle).  Not
// inlined (register peak, code size).
__device__ __noinline__ int merge_planes(const uint2* part, int nbk, int S, int hsh, unsigned tag, int* err,
                                         uint32_t xq_off, uint32_t xsc_off, uint32_t xsm_off, int sums) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* xqb = smem + xq_off;
    float* xsc = reinterpret_cast<float*>(smem + xsc_off);
    int* xsm = reinterpret_cast<int*>(smem + xsm_off);
    const int ct = threadIdx.x - 32, hd = 1 << hsh, W2 = hd + 2;
    bool ok = true;
    uint64_t t0 = 0;
#pragma unroll 1
    for (int base = 0; base < 4 * nbk; base += kConsumerThreads) {
        const int i = base + ct;
        const bool on = i < 4 * nbk;
        if (!__any_sync(0xffffffffu, on)) continue;  // (warp-uniform: planes8 shuffles)
        const int b = i >> 2, sub = i & 3, j0 = b * 32 + sub * 8;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = 0.0f;
        if (on) {
            const uint2* ph = part + (size_t)(j0 >> hsh) * S * W2 + (j0 & (hd - 1));
            float M = -INFINITY, L = 0.0f;
#pragma unroll 1
            for (int s0 = 0; s0 < S; s0 += kMergePerRound) {
                // up to kMergePerRound splits per poll round (loads of all of
                // them in flight at once); a slot past the last split re-reads
                // the last one and is not merged
                uint4 w[kMergePerRound][5];
                for (;;) {
                    bool got = true;
#pragma unroll
                    for (int u = 0; u < kMergePerRound; u++) {
                        const uint2* pp = ph + (size_t)min(s0 + u, S - 1) * W2;
#pragma unroll
                        for (int k = 0; k < 4; k++) w[u][k] = ll_load2(pp + 2 * k);
                        w[u][4] = ll_load2(pp - (j0 & (hd - 1)) + hd);  // (m, l)
                    }
#pragma unroll
                    for (int u = 0; u < kMergePerRound; u++)
#pragma unroll
                        for (int k = 0; k < 5; k++) got &= (w[u][k].y == tag) & (w[u][k].w == tag);
                    if (got || !ok) break;
                    const uint64_t now = global_ns();
                    if (t0 == 0) t0 = now;
                    if (now - t0 > kWaitLimitNs) {
                        set_err(err, B2_ERR_TIMEOUT);
                        ok = false;
                    } else if (now - t0 > kErrCheckNs && *(volatile int*)err) {
                        ok = false;
                    }
                }
#pragma unroll
                for (int u = 0; u < kMergePerRound; u++) {
                    if (s0 + u >= S) break;
                    const float ms = __uint_as_float(w[u][4].x), ls = __uint_as_float(w[u][4].z);
                    const float Mn = fmaxf(M, ms);
                    const float co = M == -INFINITY ? 0.0f : expf(M - Mn);
                    const float cn = ms == -INFINITY ? 0.0f : expf(ms - Mn);
                    L = fmaf(L, co, ls * cn);
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        v[2 * k] = fmaf(v[2 * k], co, __uint_as_float(w[u][k].x) * cn);
                        v[2 * k + 1] = fmaf(v[2 * k + 1], co, __uint_as_float(w[u][k].z) * cn);
                    }
                    M = Mn;
                }
            }
            const float rl = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] *= rl;
        }
        planes8(v, on, b, sub, xqb, xsc, xsm, sums != 0);
    }
    return ok ? 1 : 0;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

// Tensor parallel, after the Wo or the down dots: this rank's partial sums of
// residual rows row0 .. row0 + n (K-slices summed from the phase buffer at
// shared offset yb_off, rc = n outputs per slice) go to slot [tp_rank] of
// every rank's exchange region xo (peer stores over NVLink); then the N
// ranks' partials of these rows are read back from this rank's own buffer and
// added to the residual (shared offset xres_off) in rank order, so every rank
// holds the same residual stream; the sums are published as LL words.
// yb_off and xres_off are byte offsets from the dynamic shared array (not
// shared-window addresses: the array does not start at address 0).
// Returns 0 if a partial never came (error flag set).  Not inlined (the
// one-GPU path does not carry its code and registers).
__device__ __noinline__ int tp_reduce_rows(const ModelDev& m, size_t xo, int row0, int n, int nks, uint32_t yb_off,
                                           uint32_t xres_off, uint2* dstll, unsigned tag) {
    extern __shared__ __align__(128) uint8_t smem[];
    const float* yb = reinterpret_cast<const float*>(smem + yb_off);
    float* xres = reinterpret_cast<float*>(smem + xres_off);
    const int ct = threadIdx.x - 32;
    const size_t mine = xo + ((size_t)m.tp_rank * m.H + row0) * 8;
    int ok = 1;
#pragma unroll 1
    for (int j = ct; j < n; j += kConsumerThreads) {
        float d = yb[j];
#pragma unroll 1
        for (int ks = 1; ks < nks; ks++) d += yb[ks * n + j];
#pragma unroll 1
        for (int q = 0; q < m.tp; q++) ll_store_sys(reinterpret_cast<uint2*>(m.xpeer[q] + mine) + j, d, tag);
    }
#pragma unroll 1
    for (int j = ct; j < n; j += kConsumerThreads) {
        float xr = xres[j];
#pragma unroll 1
        for (int q = 0; q < m.tp && ok; q++) {
            const uint2* src = reinterpret_cast<const uint2*>(m.xpeer[m.tp_rank] + xo + ((size_t)q * m.H + row0) * 8) + j;
            uint64_t w0 = 0;
            for (;;) {
                const uint2 w = ll_load_sys(src);
                if (w.y == tag) {
                    xr += __uint_as_float(w.x);
                    break;
                }
                const uint64_t now = global_ns();
                if (w0 == 0) w0 = now;
                if (now - w0 > kWaitLimitNs) {
                    set_err(m.err, B2_ERR_TIMEOUT);
                    ok = 0;
                    break;
                }
                if (now - w0 > kErrCheckNs && *(volatile int*)m.err) {
                    ok = 0;
                    break;
                }
            }
        }
        xres[j] = xr;
        ll_store(dstll + row0 + j, xr, tag);
    }
    return ok;
}

// Tensor parallel, the lm_head's last CTA: this rank's argmax key goes to
// every rank's exchange buffer; returns the largest of all ranks' keys (the
// same on every rank).
__device__ __noinline__ unsigned long long tp_argmax_key(const ModelDev& m, unsigned long long key, unsigned tag) {
    const size_t xa = xch_am(m.H, m.tp);
    const uint4 kw = make_uint4((uint32_t)(key >> 32), tag, (uint32_t)key, tag);
    for (int q = 0; q < m.tp; q++) st4_sys(reinterpret_cast<uint4*>(m.xpeer[q] + xa) + m.tp_rank, kw);
    const uint4* mine = reinterpret_cast<const uint4*>(m.xpeer[m.tp_rank] + xa);
    for (int q = 0; q < m.tp; q++) {
        uint64_t w0 = 0;
        for (;;) {
            const uint4 w = ld4_sys(mine + q);
            if (w.y == tag && w.w == tag) {
                const unsigned long long kq = ((unsigned long long)w.x << 32) | w.z;
                if (kq > key) key = kq;
                break;
            }
            const uint64_t now = global_ns();
            if (w0 == 0) w0 = now;
            if (now - w0 > kWaitLimitNs || (now - w0 > kErrCheckNs && *(volatile int*)m.err)) {
                set_err(m.err, B2_ERR_TIMEOUT);
                break;
            }
        }
    }
    return key;
}

template <int QT, bool MV, bool TR, bool KV32>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ ModelDev m, const StepArgs a) {
    constexpr int US = QT == 8 ? 16 : 32;  // matvec: values per lane unit
    constexpr int QB = QT == 8 ? 32 : 16;  // tiled: quant bytes per row and block
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = m.nslots;
    const int SB = m.slot_bytes;
    const SmemOffsets so = smem_offsets(NS, SB, m.xs_floats, m.ybuf_floats + m.ybuf_odd, m.cfloats, m.nbx, MV ? 0 : m.L);
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + so.xs);
    uint8_t* xqb = smem + so.xq;
    float* xsc = reinterpret_cast<float*>(smem + so.xsc);
    int* xsm = reinterpret_cast<int*>(smem + so.xsm);
    float* xres = reinterpret_cast<float*>(smem + so.xres);
    float* ybuf = reinterpret_cast<float*>(smem + so.ybuf);
    float* cb = reinterpret_cast<float*>(smem + so.cbuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + so.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + so.empty);
    float* red = reinterpret_cast<float*>(smem + so.red);
    int* misc = reinterpret_cast<int*>(smem + so.misc);
    const TPlan* plans = reinterpret_cast<const TPlan*>(smem + so.plan);       // this CTA's work plans
    const LayerDev* layers = reinterpret_cast<const LayerDev*>(smem + so.lay);  // the layer table
    volatile unsigned* pstop = reinterpret_cast<volatile unsigned*>(misc + 31);  // first chunk not issued
    volatile int* dead = misc + 30;  // set by any consumer thread whose wait failed
    unsigned* issued = reinterpret_cast<unsigned*>(misc + 29);  // chunks the producer has issued

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, grid = gridDim.x;

    // A device-resident greedy loop that already produced EOS does no work.
    if (!MV && a.done && *(volatile const int*)a.done) return;

    if (!MV) {
        // this CTA's plans and the layer table, for the whole launch
        const uint2* ps = reinterpret_cast<const uint2*>(m.plans + (size_t)cta * kPlanSlots);
        uint2* pd = reinterpret_cast<uint2*>(smem + so.plan);
        #pragma unroll 1
        for (int i = threadIdx.x; i < (int)(kPlanSlots * sizeof(TPlan) / 8); i += blockDim.x) pd[i] = ps[i];
        const uint2* ls = reinterpret_cast<const uint2*>(m.layers);
        uint2* ld = reinterpret_cast<uint2*>(smem + so.lay);
        #pragma unroll 1
        for (int i = threadIdx.x; i < (int)(m.L * sizeof(LayerDev) / 8); i += blockDim.x) ld[i] = ls[i];
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        *pstop = 0xffffffffu;
        *dead = 0;
        *issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    // Lanes 0..np-1 of warp 0 each issue one chunk of every batch of np
    // consecutive chunks: the lanes share one instruction stream, so the warp
    // issues several chunks for the cost of one (the producer shares its SM
    // sub-partition with three busy consumer warps).  np <= the ring size, so
    // no batch holds two chunks of one slot.  Slots, ring rounds, tile groups
    // and K-slices advance incrementally.
    if (warp == 0) {
        constexpr int kProdLanes = 4;
        const int np = NS < kProdLanes ? NS : kProdLanes;
        if (lane < kProdLanes) {
            unsigned gbase_p = 0;  // global index of the phase's first chunk
            bool ok = true;
            for (int p = a.p_begin; p < a.p_end; p++) {
                const size_t trp = (size_t)(p - a.p_begin) * kTraceSlots;
                int nchunks;
                TGeom g{};
                TPlan pl{};
                Geom mg{};
                Split ms{};
                if (MV) {
                    mg = Geom{a.mv_w, a.mv_rb, a.mv_cols, a.mv_rows};
                    ms = cta_split(mg, cta, grid, SB);
                    nchunks = ms.nchunks;
                    pl.nks = 1;
                } else {
                    g = phase_geom(m, layers, p);
                    pl = phase_plan(plans, g, a.splits);
                    nchunks = pl.nchunks;
                }
                if (TR && a.trace && lane == 0 && nchunks) a.trace[(trp + 4) * grid + cta] = global_ns();
                uint64_t waited = 0;
                const size_t sreg = MV ? 0 : (size_t)g.tiles * kTileRows * g.nb * QB;  // scale region offset
                // this lane's first chunk k = lane, and its position
                int slot = (int)((gbase_p + lane) % NS);
                uint32_t par = (((gbase_p + lane) / NS) & 1u) ^ 1u;  // free-slot wait parity
                int kt = lane / pl.nks, ks = lane - kt * pl.nks;
                const int dq = np / pl.nks, dr = np - dq * pl.nks;
                for (int k0 = 0; k0 < nchunks; k0 += np) {
                    const int k = k0 + lane;
                    const bool mine = lane < np && k < nchunks;
                    // 1. every lane waits for its slot; 2. only lanes before the
                    // first failed wait issue, so no copy goes out past *pstop
                    bool got = false;
                    if (mine) {
                        const uint64_t t0w = (TR && a.trace) ? global_ns() : 0;
                        got = slot_wait(&empty[slot], par, m.err);
                        if (TR && a.trace) waited += global_ns() - t0w;
                    }
                    const unsigned bad = __ballot_sync(0xfu, mine && !got);
                    const int first_bad = bad ? __ffs(bad) - 1 : kProdLanes;
                    if (mine && lane < first_bad) {
                        uint8_t* dst = ring + (size_t)slot * SB;
                        if (MV) {
                            const int uu0 = ms.u0 + k * ms.cu;
                            const int nu = min(ms.cu, ms.n - k * ms.cu);
                            const size_t nbytes = (size_t)nu * mg.rb;
                            const uint8_t* src = mg.w + (size_t)uu0 * mg.rb;
                            const uint8_t* sal =
                                reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
                            const uint32_t len = (uint32_t)(((src - sal) + nbytes + 15) & ~size_t(15));
                            mbar_arrive_expect_tx(&full[slot], len);
                            bulk_g2s(dst, sal, len, &full[slot]);
                        } else {
                            // chunk k = (tile group kt, K-slice ks)
                            const int t0 = pl.u0 + kt * pl.nt, ntc = min(pl.nt, pl.u0 + pl.n - t0);
                            const int bb0 = ks * pl.bpk, nbc = min(pl.bpk, pl.kbn - bb0);
                            const size_t unit0 = (size_t)t0 * g.nb + pl.kb0 + bb0;
                            const uint32_t qlen = (uint32_t)(ntc * nbc * kTileRows * QB);
                            const uint32_t slen = (uint32_t)(ntc * nbc * 2 * kTileRows);
                            mbar_arrive_expect_tx(&full[slot], qlen + slen);
                            bulk_g2s(dst, g.w + unit0 * kTileRows * QB, qlen, &full[slot]);
                            bulk_g2s(dst + qlen, g.w + sreg + unit0 * 2 * kTileRows, slen, &full[slot]);
                        }
                    }
                    __syncwarp(0xfu);
                    // publish the chunks issued (in order); after a failed wait,
                    // consumers skip every chunk from the first one not issued
                    const int nis = bad ? first_bad : min(np, nchunks - k0);
                    if (bad && lane == 0) *pstop = gbase_p + (unsigned)(k0 + first_bad);
                    if (lane == 0) st_release_cta(issued, gbase_p + (unsigned)(k0 + nis));
                    if (bad) {
                        ok = false;
                        break;
                    }
                    slot += np;
                    while (slot >= NS) {
                        slot -= NS;
                        par ^= 1u;
                    }
                    ks += dr;
                    kt += dq;
                    if (ks >= pl.nks) {
                        ks -= pl.nks;
                        kt++;
                    }
                }
                if (TR && a.trace && lane == 0 && nchunks) {
                    a.trace[(trp + 5) * grid + cta] = global_ns();
                    a.trace[(trp + 8) * grid + cta] = waited;
                    a.trace[(trp + 9) * grid + cta] = (unsigned)nchunks;
                }
                gbase_p += (unsigned)nchunks;
                if (!ok) break;
            }
        }
        return;
    }

    // ----------------------------------------------------------- consumers
    const int cw = warp - 1;              // consumer warp index
    const int ct = threadIdx.x - 32;      // consumer thread index
    unsigned gbase = 0;                   // chunk index of the phase's first chunk
    bool alive = true;
    const int tok = MV ? 0 : *a.tok;
    // residual rows this CTA owns: its tiles of the H-row phases (Wo, down)
    int own_u0 = 0, own_n = 0;
    own_tiles(m.H / kTileRows, cta, grid, &own_u0, &own_n);
    const int own0 = kTileRows * own_u0, own1 = own0 + kTileRows * own_n;
    // Consumer barrier that also makes `alive` uniform across the CTA: a
    // failed wait in any thread stops the work of all (warp collectives in
    // the row loop must never run with part of a warp).
    auto sync_alive = [&]() {
        if (!alive) *dead = 1;
        named_bar_sync(1, kConsumerThreads);
        alive = (*dead == 0);
    };

    if (MV) {
        // ---- kernel-level matvec: y = W x, ggml rows, fp32 dequantising dot
        const Geom mg{a.mv_w, a.mv_rb, a.mv_cols, a.mv_rows};
        const Split s = cta_split(mg, cta, grid, SB);
        const int nu = mg.cols / US;
        #pragma unroll 1
        for (int j = ct; j < mg.cols; j += kConsumerThreads) xs[xs_index<US>(j, nu)] = a.mv_x[j];
        sync_alive();
        #pragma unroll 1
        for (int k = 0; k < s.nchunks; k++) {
            const unsigned gidx = k;
            if ((int)(gidx % kConsumerWarps) != cw) continue;
            const int slot = gidx % NS;
            const bool landed = __all_sync(0xffffffffu, chunk_wait(&full[slot], (gidx / NS) & 1, gidx, pstop, issued, m.err));
            if (!landed) alive = false;
            if (alive) {
                const int uu0 = s.u0 + k * s.cu;
                const int nrows = min(s.cu, s.n - k * s.cu);
                const uint8_t* src = mg.w + (size_t)uu0 * mg.rb;
                const uint8_t* base1 = ring + (size_t)slot * SB + (reinterpret_cast<uintptr_t>(src) & 15);
                #pragma unroll 1
                for (int pi = 0; pi < (nrows + 1) / 2; pi++) {
                    const uint8_t* ra = base1 + (size_t)(2 * pi) * mg.rb;
                    const bool two = (2 * pi + 1) < nrows;
                    const uint8_t* rb2 = two ? ra + mg.rb : ra;
                    float a0, a1;
                    if (QT == 8) dot2_q8(ra, rb2, two, xs, mg.cols, lane, a0, a1);
                    else dot2_q4(ra, rb2, two, xs, mg.cols, lane, a0, a1);
                    const float v = warp_sum2(a0, a1, lane);
                    if (lane == 0) a.mv_y[uu0 + 2 * pi] = v;
                    if (lane == 16 && two) a.mv_y[uu0 + 2 * pi + 1] = v;
                }
            }
            __syncwarp();
            if (lane == 0 && landed) mbar_arrive(&empty[slot]);
        }
        return;
    }

    #pragma unroll 1
    for (int p = a.p_begin; p < a.p_end; p++) {
        const TGeom g = phase_geom(m, layers, p);
        const TPlan pl = phase_plan(plans, g, a.splits);
        const bool has_rows = pl.nchunks > 0;
        const bool qa = g.kind == PH_QA;
        const int S = a.splits;
        const bool qcta = qa && cta < m.nh * S;  // q + attention role in the QA phase
        const size_t tr = (size_t)(p - a.p_begin) * kTraceSlots;
        if (TR && a.trace && ct == 0) {
            a.trace[(tr + 0) * grid + cta] = global_ns();
            misc[20] = 0;
            misc[21] = 0;
            misc[22] = 0;
            misc[23] = 0;
            misc[24] = 0;
        }
        const unsigned tag_here = ll_tag(a.epoch, g.layer) + a.skew;
        const unsigned tag_prev = ll_tag(a.epoch, g.layer - 1) + a.skew;
        // attention work of a q CTA: head h, split sidx over the cached positions [0, pos)
        const int hd = m.hd, TP = m.attn_tile;
        const int h = qcta ? cta / S : 0, sidx = qcta ? cta - h * S : 0, kvh = h / (m.nh / m.nkv);
        const int at0 = (int)((long long)sidx * a.pos / S), at1 = (int)((long long)(sidx + 1) * a.pos / S);
        const int es = KV32 ? 4 : 2;
        const size_t lay = ((size_t)g.layer * m.max_seq * m.kvd + (size_t)kvh * hd) * es;
        const uint8_t* kg = reinterpret_cast<const uint8_t*>(m.kcache) + lay;
        const uint8_t* vg = reinterpret_cast<const uint8_t*>(m.vcache) + lay;
        const uint32_t attn_off = so.xs;  // the attention scratch

        // 1. stage the phase input: gather (+ norm / merge) into xs, then planes
        if (qa && !has_rows && qcta && at1 > at0) {
            // a q CTA with no q / k / v rows of its own (the distributed form
            // with fewer tiles than CTAs) still attends: its first cached K/V
            // tile goes out now, as in the stage below
            cp_async_commit();
            attn_load_tile<KV32>(kg, vg, (uint32_t)(m.kvd * es), hd, TP, at0, min(TP, at1 - at0), attn_off);
        }
        if (qa && g.layer == 0) {
            // transformer.go:524-531: the residual stream starts at the embedding
            #pragma unroll 1
            for (int j = own0 + ct; j < own1; j += kConsumerThreads) xres[j - own0] = embed_elem<QT>(m, tok, j);
        }
        if ((qa || g.kind == PH_GATEUP || g.kind == PH_LMHEAD) && has_rows) {
            // QKV constants first (they land while the poll below waits)
            if (qa) {
                const float* bq = layers[g.layer].bqkv;
                const int r0b = (kTileRows * pl.u0) & ~3, r1 = kTileRows * (pl.u0 + pl.n);
                if (bq)
                    #pragma unroll 1
                    for (int i = ct; i < (r1 - r0b + 3) / 4; i += kConsumerThreads)
                        cp_async16(cb + cb_bias(m) + 4 * i, bq + r0b + 4 * i);
                const int hh = hd / 2;
                #pragma unroll 1
                for (int i = ct; i < hh / 4; i += kConsumerThreads) {
                    cp_async16(cb + cb_cos(m) + 4 * i, m.rope_cos + (size_t)a.pos * hh + 4 * i);
                    cp_async16(cb + cb_sin(m) + 4 * i, m.rope_sin + (size_t)a.pos * hh + 4 * i);
                }
            }
            cp_async_commit();
            // a q CTA's first cached K/V tile goes out now too (its own group,
            // waited for in the attention): it overlaps the poll and the dot
            if (qcta && at1 > at0)
                attn_load_tile<KV32>(kg, vg, (uint32_t)(m.kvd * es), hd, TP, at0, min(TP, at1 - at0), attn_off);
            // RMSNorm (transformer.go:922-932): x * gain goes into the planes here,
            // the scale 1/rms multiplies the dot products in the epilogue
            const float* nw = qa ? layers[g.layer].attn_norm
                                 : (g.kind == PH_GATEUP ? layers[g.layer].ffn_norm : m.out_norm);
            float ss = 0.0f;
            if (alive) {
                // QA (after layer 0) and the LM head read the residual stream after
                // the previous down phase: x2, or with the down phase split over K
                // x1 plus the down partials of the previous layer
                GatherRes gr;
                if (m.dn_split > 1 && g.kind != PH_GATEUP && !(qa && g.layer == 0))
                    gr = gather_planes<QT, kDownSplit>(m.ll_x1, m.H / 32, tag_prev, m.err, 0, tok, m.tok_embd, m.Vemb,
                                                       m.H, m.Vp_emb, so.xq, so.xsc, so.xsm, nw, QT != 8,
                                                       m.ll_dnp + (size_t)((g.layer - 1) & 1) * kDownSplit * m.H, m.H);
                else
                    gr = gather_planes<QT, 0>(g.kind == PH_GATEUP ? m.ll_x1 : m.ll_x2, m.H / 32,
                                              g.kind == PH_GATEUP ? tag_here : tag_prev, m.err, qa && g.layer == 0, tok,
                                              m.tok_embd, m.Vemb, m.H, m.Vp_emb, so.xq, so.xsc, so.xsm, nw, QT != 8,
                                              nullptr, 0);
                alive = gr.ok;
                ss = gr.ss;
            }
            if (TR && a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
            if (qcta && at1 > at0) cp_async_wait_1();  // the constants (not the K/V tile)
            else cp_async_wait();
            ss = warp_sum(ss);
            if (lane == 0) red[32 + cw] = ss;  // summed after the rows barrier
        } else if (g.kind == PH_WO && has_rows) {
            // with the down phase split over K, the residual rows this CTA owns
            // still lack the previous layer's down partials: their words go to
            // shared memory now (two 16-row slices of LL words, checked in the
            // epilogue) and land while the merge below polls
            if (m.dn_split > 1 && g.layer > 0 && ct < 2 * kTileRows / 2)
                cp_async16(smem + so.dnp + 16 * ct,
                           m.ll_dnp + ((size_t)(((g.layer - 1) & 1) * kDownSplit + ct / 8)) * m.H + own0 + 2 * (ct % 8));
            cp_async_commit();
            // the attention of every head, merged from its split partials
            if (alive)
                alive = merge_planes(m.ll_part, m.qd / 32, S, __ffs(hd) - 1, tag_here, m.err, so.xq, so.xsc, so.xsm,
                                     QT != 8) != 0;
            cp_async_wait();
            if (TR && a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        } else if (g.kind == PH_DOWN && has_rows) {
            // this CTA's blocks of the SwiGLU output (all of them, or its half of
            // the row when the phase is split over K)
            if (alive)
                alive = gather_planes<QT, 0>(m.ll_act + 32 * pl.kb0, pl.kbn, tag_here, m.err, 0, 0, m.tok_embd, m.Vemb,
                                             m.H, m.Vp_emb, so.xq, so.xsc, so.xsm, nullptr, QT != 8, nullptr, 0).ok;
            if (TR && a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        } else {
            if (TR && a.trace && ct == 0) a.trace[(tr + 1) * grid + cta] = global_ns();
        }
        sync_alive();
        if (TR && a.trace && ct == 0) a.trace[(tr + 2) * grid + cta] = global_ns();

        // parity buffers (even phases' one first, sized for the lm_head); every
        // lm_head sub-phase uses the even one, whatever its parity (the stage
        // barrier of each phase orders its dots after the previous epilogue)
        float* yb = ybuf + (((p & 1) && g.kind != PH_LMHEAD) ? m.ybuf_floats : 0);
        const int rc = kTileRows * pl.n;  // outputs of one K-slice in yb
        {
            // 2. rows: tensor-core dot products of this CTA's tiles into yb
            const uint64_t tl0 = (TR && a.trace) ? global_ns() : 0;
            // this warp's chunks are k = first, first + kConsumerWarps, ... (global
            // index = cw mod kConsumerWarps); slot, ring round, tile group and
            // K-slice advance incrementally (no divisions in the loop)
            const int first = (int)((unsigned)(cw + kConsumerWarps) - gbase % kConsumerWarps) % kConsumerWarps;
            int slot = (int)((gbase + first) % NS);
            uint32_t par = ((gbase + first) / NS) & 1u;
            int kt = first / pl.nks, ks = first - kt * pl.nks;
            const int dq = kConsumerWarps / pl.nks, dr = kConsumerWarps - dq * pl.nks;
            #pragma unroll 1
            for (int k = first; k < pl.nchunks; k += kConsumerWarps) {
                const unsigned gidx = gbase + k;
                const uint64_t tw = (TR && a.trace) ? global_ns() : 0;
                const bool landed = __all_sync(0xffffffffu, chunk_wait(&full[slot], par, gidx, pstop, issued, m.err));
                if (TR && a.trace && lane == 0) {
                    const unsigned dt = (unsigned)(global_ns() - tw);
                    atomicAdd(reinterpret_cast<unsigned*>(misc + 20), dt);
                    if (dt > 256) atomicAdd(reinterpret_cast<unsigned*>(misc + 21), 1u);
                }
                if (!landed) alive = false;
                if (alive) {
                    const int lt0 = kt * pl.nt, ntc = min(pl.nt, pl.n - lt0);
                    const int bb0 = ks * pl.bpk, nbc = min(pl.bpk, pl.kbn - bb0);
                    const int qlen = ntc * nbc * kTileRows * QB;
                    float* yk = yb + ks * rc;
                    #pragma unroll 1
                    for (int tl = 0; tl < ntc; tl++) {
                        const uint32_t qa = (uint32_t)(slot * SB + tl * nbc * kTileRows * QB);
                        const uint32_t sa = (uint32_t)(slot * SB + qlen + tl * nbc * 2 * kTileRows);
                        const uint64_t td0 = (TR && a.trace) ? global_ns() : 0;
                        const float2 y = tile_dot<QT>(smem_u32(smem) + qa, sa, nbc, so.xq, so.xsc, so.xsm, bb0);
                        if (TR && a.trace && lane == 0) atomicAdd(reinterpret_cast<unsigned*>(misc + 22), (unsigned)(global_ns() - td0));
                        const int lr = (lt0 + tl) * kTileRows + (lane >> 2);  // local row of y.x; y.y is lr + 8
                        if ((lane & 3) == 0) {
                            yk[lr] = y.x;
                            yk[lr + 8] = y.y;
                        }
                    }
                }
                __syncwarp();
                if (lane == 0 && landed) mbar_arrive(&empty[slot]);
                slot += kConsumerWarps;
                while (slot >= NS) {
                    slot -= NS;
                    par ^= 1u;
                }
                ks += dr;
                kt += dq;
                if (ks >= pl.nks) {
                    ks -= pl.nks;
                    kt++;
                }
            }
            gbase += pl.nchunks;
            if (TR && a.trace && lane == 0) {
                const unsigned dl = (unsigned)(global_ns() - tl0);
                atomicAdd(reinterpret_cast<unsigned*>(misc + 23), dl);
                atomicMax(reinterpret_cast<unsigned*>(misc + 24), dl);
            }
        }
        sync_alive();
        if (TR && a.trace && ct == 0) {
            a.trace[(tr + 10) * grid + cta] = global_ns();
            a.trace[(tr + 11) * grid + cta] = (unsigned)misc[22] | ((unsigned long long)(unsigned)misc[23] << 32);
            a.trace[(tr + 9) * grid + cta] |= (unsigned long long)(unsigned)misc[24] << 32;
        }

        // 3. epilogue, one thread per output; K-slice partials summed in order
        const unsigned tag = ll_tag(a.epoch, g.layer);
        float rms = 1.0f;  // RMSNorm scale of the norm phases (transformer.go:922-932)
        if (qa || g.kind == PH_GATEUP || g.kind == PH_LMHEAD) {
            float tot = 0.0f;
            #pragma unroll
            for (int w = 0; w < kConsumerWarps; w++) tot += red[32 + w];
            // in fp32 with the fast divide and reciprocal square root (Go
            // rounds a float64 result to float32; these are within 2 ulp of
            // it, and the IEEE forms cost a long dependent chain here)
            rms = rsqrtf(__fdividef(tot, (float)m.H) + m.eps);
        }
        if (TR && a.trace && ct == 0) a.trace[(tr + 12) * grid + cta] = global_ns();
        const int row0 = kTileRows * pl.u0;
        auto ysum = [&](int i) {
            float v = yb[i];
            #pragma unroll 4
            for (int ks = 1; ks < pl.nks; ks++) v += yb[ks * rc + i];
            return v;
        };
        if ((alive && has_rows) || g.kind == PH_LMHEAD) {
            // (every CTA takes part in the argmax, so its arrival counter
            // always completes and resets)
            switch (g.kind) {
                case PH_QA: {
                    // bias (transformer.go:632-646), RoPE on interleaved pairs
                    // (936-951); q rows stay in this CTA for its attention (published
                    // in the distributed form), k / v rows are published (the q CTAs'
                    // new position) and appended to the KV cache (654-656)
                    const bool bias = layers[g.layer].bqkv != nullptr;
                    const int bias0 = row0 & ~3;
                    float* aq = reinterpret_cast<float*>(smem + attn_off);
                    #pragma unroll 1
                    for (int j = ct; j < kTileRows / 2 * pl.n; j += kConsumerThreads) {
                        const int row = row0 + 2 * j;
                        float a0 = ysum(2 * j) * rms, a1 = ysum(2 * j + 1) * rms;
                        if (bias) {
                            a0 += cb[cb_bias(m) + row - bias0];
                            a1 += cb[cb_bias(m) + row + 1 - bias0];
                        }
                        if (row < m.qd + m.kvd) {
                            const int pi2 = (row % hd) >> 1;
                            const float rc2 = cb[cb_cos(m) + pi2], rs = cb[cb_sin(m) + pi2];
                            const float x0 = a0, x1 = a1;
                            a0 = x0 * rc2 - x1 * rs;
                            a1 = x0 * rs + x1 * rc2;
                        }
                        if (row < m.qd && !m.qa_dist) {
                            aq[row - h * hd] = a0;
                            aq[row - h * hd + 1] = a1;
                            continue;
                        }
                        ll_store2(m.ll_qkv + row, a0, a1, tag);
                        if (row < m.qd) continue;
                        const bool isk = row < m.qd + m.kvd;
                        const int col = row - m.qd - (isk ? 0 : m.kvd);
                        const size_t off = ((size_t)g.layer * m.max_seq + a.pos) * m.kvd + col;
                        void* cache = isk ? m.kcache : m.vcache;
                        if (KV32) {
                            reinterpret_cast<float*>(cache)[off] = a0;
                            reinterpret_cast<float*>(cache)[off + 1] = a1;
                        } else {
                            *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(cache) + off) = __floats2half2_rn(a0, a1);
                        }
                    }
                    break;
                }
                case PH_GATEUP:
                    // SwiGLU (transformer.go:725-727, 954-956): output j of tile
                    // t has its gate at row 16t + j % 8 and its up 8 rows below
                    #pragma unroll 1
                    for (int j = ct; j < kTileRows / 2 * pl.n; j += kConsumerThreads) {
                        const int r = (j >> 3) * kTileRows + (j & 7);
                        const float gv = ysum(r) * rms, uv = ysum(r + 8) * rms;
                        ll_store(m.ll_act + row0 / 2 + j, __fdividef(gv, 1.0f + __expf(-gv)) * uv, tag);
                    }
                    break;
                case PH_WO:
                case PH_DOWN: {
                    if (g.kind == PH_DOWN && m.dn_split > 1) {
                        // split over K: this half-row's partial sums of the tile's
                        // residual rows, for the readers of the residual stream
                        uint2* dp = m.ll_dnp +
                                    ((size_t)((g.layer & 1) * kDownSplit + dn_slice_of(cta, grid, m.H / kTileRows))) * m.H +
                                    row0;
                        #pragma unroll 1
                        for (int j = ct; j < kTileRows * pl.n; j += kConsumerThreads) ll_store(dp + j, ysum(j), tag);
                        break;
                    }
                    if (g.kind == PH_WO && m.dn_split > 1 && g.layer > 0) {
                        // the owned rows become x2 of the previous layer: x1 plus its
                        // down partials in slice order (as every gather adds them);
                        // words the prefetch found stale are polled again
                        const uint2* dw = reinterpret_cast<const uint2*>(smem + so.dnp);
                        #pragma unroll 1
                        for (int j = ct; j < kTileRows * pl.n; j += kConsumerThreads) {
                            float xr = xres[j];
                            #pragma unroll
                            for (int sl = 0; sl < kDownSplit; sl++) {
                                uint2 w = dw[sl * kTileRows + j];
                                const uint2* gw = m.ll_dnp +
                                                  ((size_t)(((g.layer - 1) & 1) * kDownSplit + sl)) * m.H + row0 + j;
                                uint64_t w0 = 0;
                                while (w.y != tag_prev && alive) {
                                    w = ll_load1(gw);
                                    const uint64_t now = global_ns();
                                    if (w0 == 0) w0 = now;
                                    if (now - w0 > kWaitLimitNs) {
                                        set_err(m.err, B2_ERR_TIMEOUT);
                                        alive = false;
                                    }
                                }
                                xr += __uint_as_float(w.x);
                            }
                            xres[j] = xr;
                        }
                    }
                    // residual (transformer.go:576-578, 591-593); the rows are
                    // exactly the residual rows this CTA owns
                    uint2* dstll = g.kind == PH_WO ? m.ll_x1 : m.ll_x2;
                    if (m.tp > 1) {
                        // (byte offsets from the dynamic shared array, like every helper's)
                        if (!tp_reduce_rows(m, g.kind == PH_WO ? 0 : xch_dn(m.H, m.tp), row0, kTileRows * pl.n, pl.nks,
                                            (uint32_t)(reinterpret_cast<uint8_t*>(yb) - smem),
                                            (uint32_t)(reinterpret_cast<uint8_t*>(xres) - smem), dstll, tag))
                            alive = false;
                        break;
                    }
                    #pragma unroll 1
                    for (int j = ct; j < kTileRows * pl.n; j += kConsumerThreads) {
                        const float xr = xres[j] + ysum(j);
                        xres[j] = xr;
                        ll_store(dstll + row0 + j, xr, tag);
                    }
                    break;
                }
                default: {  // PH_LMHEAD
                    // logits + argmax, first maximum wins (transformer.go:1038-1046)
                    // (indices are vocab ids: this rank's share starts at v_off)
                    Best best{-INFINITY, 0x7fffffff};
                    #pragma unroll 1
                    for (int j = ct; alive && j < kTileRows * pl.n; j += kConsumerThreads) {
                        const int row = row0 + j;
                        if (row >= g.rows) break;
                        const float v = ysum(j) * rms;
                        m.logits[row] = v;
                        if (better(v, row + m.v_off, best.v, best.i)) { best.v = v; best.i = row + m.v_off; }
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
                        #pragma unroll 1
                        for (int w = 1; w < kConsumerWarps; w++)
                            if (better(red[w], misc[4 + w], b.v, b.i)) { b.v = red[w]; b.i = misc[4 + w]; }
                        // one atomic max per CTA on (order-preserving value bits, ~index):
                        // the largest value wins, and among equal values the lowest index
                        if (b.i != 0x7fffffff) {
                            const uint32_t u = __float_as_uint(b.v);
                            const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
                            atomicMax(m.am_key, ((unsigned long long)ord << 32) | (uint32_t)~(uint32_t)b.i);
                        }
                        // (the arrivals, and the key's read and reset, in the last sub-phase)
                        if (g.sub == m.n_lm - 1) {
                        __threadfence();
                        const unsigned old = atom_acq_rel_add(m.am_ctr, 1u);
                        if (old == (unsigned)(grid - 1)) {
                            // last CTA: every other CTA's max is in am_key
                            unsigned long long key = atomicExch(m.am_key, 0ull);
                            if (m.tp > 1) key = tp_argmax_key(m, key, tag);
                            const int f = key ? (int)~(uint32_t)key : 0;
                            *m.token = f;
                            if (a.out_ids) a.out_ids[a.step] = f;
                            if (a.done && f == a.eos) *a.done = 1;
                            atomicExch(m.am_ctr, 0u);
                        }
                        }
                    }
                    break;
                }
            }
        }
        if (qcta) {
            // 2'. the head's attention over its split of the positions (q is in the
            // scratch; the distributed form reads it back from the LL words)
            if (m.qa_dist && alive && ct < hd / 2) {
                float* aq = reinterpret_cast<float*>(smem + attn_off);
                const uint2* src = m.ll_qkv + (size_t)h * hd + 2 * ct;
                uint64_t w0 = 0;
                for (;;) {
                    const uint4 w = ll_load2(src);
                    if ((w.y == tag) & (w.w == tag)) {
                        aq[2 * ct] = __uint_as_float(w.x);
                        aq[2 * ct + 1] = __uint_as_float(w.z);
                        break;
                    }
                    const uint64_t now = global_ns();
                    if (w0 == 0) w0 = now;
                    if (now - w0 > kWaitLimitNs) {
                        set_err(m.err, B2_ERR_TIMEOUT);
                        alive = false;
                        break;
                    }
                    if (now - w0 > kErrCheckNs && *(volatile int*)m.err) {
                        alive = false;
                        break;
                    }
                }
            }
            sync_alive();
            if (alive) {
                uint2* po = m.ll_part + ((size_t)h * S + sidx) * (hd + 2);
                const uint2* kn = m.ll_qkv + m.qd + (size_t)kvh * hd;
                const uint32_t gsb = (uint32_t)(m.kvd * es);
                const int lst = sidx == S - 1;
                int r;
                switch (hd) {
                    case 16: r = attn_phase<KV32, 16, 8>(kg, vg, gsb, TP, at0, at1, tag, po, attn_off, kn, m.kvd, lst, m.err); break;
                    case 32: r = attn_phase<KV32, 32, 8>(kg, vg, gsb, TP, at0, at1, tag, po, attn_off, kn, m.kvd, lst, m.err); break;
                    case 64: r = attn_phase<KV32, 64, 8>(kg, vg, gsb, TP, at0, at1, tag, po, attn_off, kn, m.kvd, lst, m.err); break;
                    case 128: r = attn_phase<KV32, 128, 8>(kg, vg, gsb, TP, at0, at1, tag, po, attn_off, kn, m.kvd, lst, m.err); break;
                    default: r = attn_phase<KV32, 256, 8>(kg, vg, gsb, TP, at0, at1, tag, po, attn_off, kn, m.kvd, lst, m.err); break;
                }
                alive = r != 0;
            }
            else
                cp_async_wait();  // the prefetched tile, before the scratch is reused
        }
        if (TR && a.trace && ct == 0) {
            a.trace[(tr + 3) * grid + cta] = global_ns();
            a.trace[(tr + 6) * grid + cta] = (unsigned)misc[20];
            a.trace[(tr + 7) * grid + cta] = (unsigned)misc[21];
        }
    }
    cp_async_wait();
}

}  // namespace

size_t decode_smem_bytes(const ModelDev& m) {
    return smem_offsets(m.nslots, m.slot_bytes, m.xs_floats, m.ybuf_floats + m.ybuf_odd, m.cfloats, m.nbx,
                        m.plans ? m.L : 0).total;
}

int launch_decode(const ModelDev& m, const StepArgs& a, int grid, cudaStream_t stream, std::string* err) {
    for (int p = 0; p < m.tp && m.tp > 1; p++)
        if (!m.xpeer[p]) {
            *err = "tensor-parallel model not connected (b2_tp_connect)";
            return B2_ERR_BAD_ARG;
        }
    const size_t smem = decode_smem_bytes(m);
    void* args[] = {(void*)&m, (void*)&a};
    // instantiations: (Q8_0, Q4_0) x (model, matvec) x (plain, traced); the
    // plain kernels carry no trace code at all (smaller instruction footprint)
    // model kernels: (Q8_0, Q4_0) x (plain, traced) x (fp16, fp32 KV cache);
    // matvec kernels: (Q8_0, Q4_0).  Each kernel carries only its own paths
    // (the instruction cache is the limit at B = 1).
    static const void* const fns[10] = {
        (const void*)decode_kernel<8, false, false, false>, (const void*)decode_kernel<2, false, false, false>,
        (const void*)decode_kernel<8, false, true, false>,  (const void*)decode_kernel<2, false, true, false>,
        (const void*)decode_kernel<8, false, false, true>,  (const void*)decode_kernel<2, false, false, true>,
        (const void*)decode_kernel<8, false, true, true>,   (const void*)decode_kernel<2, false, true, true>,
        (const void*)decode_kernel<8, true, false, false>,  (const void*)decode_kernel<2, true, false, false>};
    const int q = m.qtype == 8 ? 0 : 1;
    const int ti = a.mv_w ? 8 + q : q + (a.trace ? 2 : 0) + (m.kv_fp32 ? 4 : 0);
    const void* fn = fns[ti];
    static bool attr_done[10] = {false, false, false, false, false, false, false, false, false, false};
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
