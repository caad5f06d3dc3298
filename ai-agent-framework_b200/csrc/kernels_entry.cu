// Kernel-level entry points: the dequantising matvec on its own and the
// long-context GQA decode attention.
#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "model.h"

namespace b2 {
namespace {

struct DeviceScratch {
    int* err = nullptr;
    int sms = 0;
};

std::mutex g_mu;
std::vector<DeviceScratch> g_scratch;

DeviceScratch* scratch_for_current(std::string* err) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { *err = "no CUDA device"; return nullptr; }
    std::lock_guard<std::mutex> g(g_mu);
    if ((int)g_scratch.size() <= dev) g_scratch.resize(dev + 1);
    DeviceScratch& s = g_scratch[dev];
    if (!s.err) {
        if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) { *err = "cudaMalloc failed"; return nullptr; }
        cudaMemset(s.err, 0, sizeof(int));
        cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return &s;
}

// ---------------------------------------------------------------------------
// attention: transformer.go:658-685 for one new query token per sequence,
// split over the context (flash-decoding) with a log-sum-exp merge.
// ---------------------------------------------------------------------------

template <int N>
__device__ __forceinline__ void cp_async_wait_stages() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kAttThreads = 256;
constexpr int kAttWarps = kAttThreads / 32;
constexpr int kMaxGrp = 8;      // query heads per KV head handled in registers
constexpr int kMaxDimsLane = 8; // head_dim up to 256

// One CTA = one (sequence, KV head, context slice), GRP query heads of head
// dimension HD.  A group of LP = HD / 8 lanes takes one position at a time
// (8 elements of k and v per lane, 16-byte loads) and keeps its own online
// softmax per query head, so a step needs only the LP-lane reduction of
// q . k; a warp advances 32 / LP positions per step and issues the loads of
// U steps before using them, so enough bytes are in flight to stream the
// cache.  Groups merge by shuffles, warps through shared memory; the CTA
// writes one partial (o unnormalised, m, l) per query head.
// VAR: sequences of their own lengths (lens[b] + add positions) in caches
// `stride` positions apart (a batch of decode sequences); otherwise every
// sequence has ctx positions, stored back to back.
struct AttnSeqs {
    const int* lens;
    int add, stride;
};

template <int HD, int GRP, bool VAR>
__global__ void __launch_bounds__(kAttThreads, (GRP <= 4 ? 2 : 1))
    attn_split_kernel(const float* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                      float* __restrict__ part, int nh, int nkv, int ctx, int S, const AttnSeqs seqs) {
    constexpr int DL = 8, LP = HD / DL, G = 32 / LP, U = GRP <= 3 ? 4 : (GRP == 4 ? 3 : 2);
    extern __shared__ float sm[];
    pdl_trigger();
    pdl_wait();
    const int cta = blockIdx.x;
    const int s = cta % S, g = (cta / S) % nkv, b = cta / (S * nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / LP, d0 = (lane % LP) * DL;
    const int len = VAR ? __ldg(seqs.lens + b) + seqs.add : ctx;
    const int t0 = (int)((long long)s * len / S), t1 = (int)((long long)(s + 1) * len / S);
    const size_t kvd = (size_t)nkv * HD;
    const size_t bstride = VAR ? (size_t)seqs.stride : (size_t)ctx;
    const __half* kb = k + (size_t)b * bstride * kvd + (size_t)g * HD + d0;
    const __half* vb = v + (size_t)b * bstride * kvd + (size_t)g * HD + d0;
    const float scale = (float)(1.0 / sqrt((double)HD));
    float qr[GRP][DL], o[GRP][DL], mr[GRP], lr[GRP];
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        const float* qh = q + ((size_t)b * nh + (size_t)g * GRP + h) * HD + d0;
        const float4 x0 = *reinterpret_cast<const float4*>(qh), x1 = *reinterpret_cast<const float4*>(qh + 4);
        qr[h][0] = x0.x * scale; qr[h][1] = x0.y * scale; qr[h][2] = x0.z * scale; qr[h][3] = x0.w * scale;
        qr[h][4] = x1.x * scale; qr[h][5] = x1.y * scale; qr[h][6] = x1.z * scale; qr[h][7] = x1.w * scale;
        mr[h] = -INFINITY;
        lr[h] = 0.0f;
#pragma unroll
        for (int e = 0; e < DL; e++) o[h][e] = 0.0f;
    }
    constexpr int step = kAttWarps * G;  // positions per CTA step
    for (int base = t0 + warp * G; base < t1; base += step * U) {
        uint4 kr[U], vr[U];
        bool on[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = base + u * step + grp;
            on[u] = t < t1;
            const size_t tt = (size_t)(on[u] ? t : t0);
            kr[u] = __ldg(reinterpret_cast<const uint4*>(kb + tt * kvd));
            vr[u] = __ldg(reinterpret_cast<const uint4*>(vb + tt * kvd));
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (!__any_sync(0xffffffffu, on[u])) break;  // warp-uniform
            float kf[DL], vf[DL];
            const __half2* kh = reinterpret_cast<const __half2*>(&kr[u]);
            const __half2* vh = reinterpret_cast<const __half2*>(&vr[u]);
#pragma unroll
            for (int e = 0; e < DL / 2; e++) {
                const float2 a = __half22float2(kh[e]), c = __half22float2(vh[e]);
                kf[2 * e] = a.x; kf[2 * e + 1] = a.y; vf[2 * e] = c.x; vf[2 * e + 1] = c.y;
            }
#pragma unroll
            for (int h = 0; h < GRP; h++) {
                float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                for (int e = 0; e < DL; e += 2) {
                    s0 = fmaf(qr[h][e], kf[e], s0);
                    s1 = fmaf(qr[h][e + 1], kf[e + 1], s1);
                }
                float sc = s0 + s1;
#pragma unroll
                for (int off = 1; off < LP; off <<= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
                if (on[u]) {
                    // one exponential per position: the larger of (m, sc) keeps weight 1
                    const float ex = __expf(-fabsf(sc - mr[h]));  // m = -inf: 0
                    const bool up = sc > mr[h];
                    const float cf = up ? ex : 1.0f, pr = up ? 1.0f : ex;
                    lr[h] = fmaf(lr[h], cf, pr);
#pragma unroll
                    for (int e = 0; e < DL; e++) o[h][e] = fmaf(pr, vf[e], o[h][e] * cf);
                    mr[h] = up ? sc : mr[h];
                }
            }
        }
    }
    // merge the lane groups of this warp
#pragma unroll
    for (int off = LP; off < 32; off <<= 1) {
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            const float mo = __shfl_xor_sync(0xffffffffu, mr[h], off), lo = __shfl_xor_sync(0xffffffffu, lr[h], off);
            const float mx = fmaxf(mr[h], mo);
            const float c1 = mr[h] == -INFINITY ? 0.0f : __expf(mr[h] - mx);
            const float c2 = mo == -INFINITY ? 0.0f : __expf(mo - mx);
            lr[h] = lr[h] * c1 + lo * c2;
#pragma unroll
            for (int e = 0; e < DL; e++) o[h][e] = o[h][e] * c1 + __shfl_xor_sync(0xffffffffu, o[h][e], off) * c2;
            mr[h] = mx;
        }
    }
    // merge the warps of this CTA: [warp][GRP][HD + 2] (o, m, l)
    float* wp = sm + (size_t)warp * GRP * (HD + 2);
    if (grp == 0) {
#pragma unroll
        for (int h = 0; h < GRP; h++) {
#pragma unroll
            for (int e = 0; e < DL; e++) wp[h * (HD + 2) + d0 + e] = o[h][e];
            if (lane == 0) {
                wp[h * (HD + 2) + HD] = mr[h];
                wp[h * (HD + 2) + HD + 1] = lr[h];
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < GRP * (HD + 2); i += kAttThreads) {
        const int h = i / (HD + 2), d = i - h * (HD + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttWarps; w++) M = fmaxf(M, sm[((size_t)w * GRP + h) * (HD + 2) + HD]);
        float val = M;
        if (d != HD) {
            val = 0.0f;
#pragma unroll
            for (int w = 0; w < kAttWarps; w++) {
                const float* pw = sm + ((size_t)w * GRP + h) * (HD + 2);
                const float f = pw[HD] == -INFINITY ? 0.0f : __expf(pw[HD] - M);
                val = fmaf(pw[d], f, val);
            }
        }
        part[(((size_t)b * nh + (size_t)g * GRP + h) * S + s) * (HD + 2) + d] = val;
    }
}

// ---------------------------------------------------------------------------
// The same split attention on the tensor cores (head dimension 64 or 128, up
// to 16 query heads per KV head).  One CTA = one (sequence, KV head, context
// slice), 4 warps; the cached K and V rows of the slice stream through a
// cp.async ring of kMmaStages tiles of kMmaTile positions in 128-byte-swizzled
// shared memory.  Per 16 positions a warp computes S = Q K^T with
// mma.m16n8k16 (the group's query heads are the 16 rows of A; rows past the
// group are zero), keeps an online softmax per row on the accumulator
// fragments, and adds P V with P taken straight from the S fragments (two
// n8 accumulator tiles form one k16 A fragment).  Q and P are split into two
// fp16 terms each (hi + lo, the lo term the rounding remainder), so the
// products carry about 22 bits: the result matches the fp32 loop of
// transformer.go:663-685 to ~1e-6, with K and V used exactly.  The four
// warps' (o, m, l) merge in shared memory into the same partial record as
// attn_split_kernel writes.
// ---------------------------------------------------------------------------
constexpr int kMmaThreads = 128;
constexpr int kMmaTile = 64;   // positions per ring tile (16 per warp)
constexpr int kMmaStages = 3;
constexpr int kMmaMaxGrp = 16;

template <int HD>
struct MmaSmem {
    static constexpr int kRow = HD * 2;                    // bytes of one cached row
    static constexpr int kTile = kMmaTile * kRow;          // one K (or V) tile
    static constexpr int kQ = 16 * kRow;                   // Q hi (then Q lo) [16 rows][HD] fp16
    static constexpr int kStages = kMmaStages;
    static constexpr int kMerge = 4 * 16 * (HD + 2) * 4;   // warps' (o, m, l) for the merge
    static constexpr int kRing = kStages * 2 * kTile;
    static constexpr int kTotal = kRing + 2 * kQ + (kMerge > 0 ? 0 : 0);
};

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile
template <int HD>
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)(r * (HD * 2) + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
                 "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void mma_f16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm4_t(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// (a, b) -> half2 hi and the half2 of the remainders
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int HD, bool VAR>
__global__ void __launch_bounds__(kMmaThreads, 1)
    attn_mma_kernel(const float* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
                    float* __restrict__ part, int nh, int nkv, int grp, int ctx, int S, const AttnSeqs seqs) {
    using SM = MmaSmem<HD>;
    constexpr int KS = HD / 16;        // k16 steps of S = Q K^T
    constexpr int NT = HD / 8;         // n8 tiles of O
    constexpr int CH = HD * 2 / 16;    // 16-byte chunks per row
    extern __shared__ __align__(1024) uint8_t asm_raw[];
    uint8_t* ring = asm_raw;                         // [stage][K tile | V tile]
    uint8_t* qh = ring + SM::kRing;                  // [16][HD] fp16, swizzled
    uint8_t* ql = qh + SM::kQ;
    pdl_trigger();
    pdl_wait();
    const int cta = blockIdx.x;
    const int s = cta % S, g = (cta / S) % nkv, b = cta / (S * nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, ti = lane & 3;
    const int len = VAR ? __ldg(seqs.lens + b) + seqs.add : ctx;
    const int t0 = (int)((long long)s * len / S), t1 = (int)((long long)(s + 1) * len / S);
    const size_t kvd = (size_t)nkv * HD;
    const size_t bstride = VAR ? (size_t)seqs.stride : (size_t)ctx;
    const __half* kb = k + (size_t)b * bstride * kvd + (size_t)g * HD;
    const __half* vb = v + (size_t)b * bstride * kvd + (size_t)g * HD;
    const int ntile = (t1 - t0 + kMmaTile - 1) / kMmaTile;

    auto issue = [&](int tile) {
        if (tile < ntile) {
            uint8_t* kt = ring + (size_t)(tile % kMmaStages) * 2 * SM::kTile;
            uint8_t* vt = kt + SM::kTile;
            for (int i = threadIdx.x; i < kMmaTile * CH; i += kMmaThreads) {
                const int r = i / CH, c = i - r * CH;
                const int t = t0 + tile * kMmaTile + r;
                const bool ok = t < t1;
                const size_t row = (size_t)(ok ? t : t0) * kvd;
                cp_async16_zfill(kt + sw_off<HD>(r, c), kb + row + c * 8, ok);
                cp_async16_zfill(vt + sw_off<HD>(r, c), vb + row + c * 8, ok);
            }
        }
        cp_async_commit();
    };
#pragma unroll 1
    for (int i = 0; i < kMmaStages - 1; i++) issue(i);

    // Q (scaled by 1 / sqrt(HD)) as hi + lo fp16 rows; rows past the group zero
    const float scale = (float)(1.0 / sqrt((double)HD));
    for (int i = threadIdx.x; i < 16 * (HD / 2); i += kMmaThreads) {
        const int r = i / (HD / 2), c2 = i - r * (HD / 2);  // row, pair of columns
        float a = 0.0f, bb = 0.0f;
        if (r < grp) {
            const float* qr = q + ((size_t)b * nh + (size_t)g * grp + r) * HD + 2 * c2;
            a = qr[0] * scale;
            bb = qr[1] * scale;
        }
        uint32_t hi, lo;
        split2(a, bb, hi, lo);
        const uint32_t off = sw_off<HD>(r, (2 * c2) / 8) + ((2 * c2) % 8) * 2;
        *reinterpret_cast<uint32_t*>(qh + off) = hi;
        *reinterpret_cast<uint32_t*>(ql + off) = lo;
    }

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows gi, gi + 8
    const uint32_t qh_s = smem_u32(qh), ql_s = smem_u32(ql);
    // ldmatrix row / chunk of this lane for an A (Q) fragment: matrices
    // (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
    const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_kc = (lane >> 4) & 1;
    // B (K) fragments, non-transposed: (pos 0-7, k 0-7), (pos 0-7, k 8-15), (pos 8-15, k 0-7), (pos 8-15, k 8-15)
    const int bk_row = (lane & 7) + ((lane >> 4) & 1) * 8, bk_kc = (lane >> 3) & 1;
    // B (V) fragments, transposed: (pos 0-7, d 0-7), (pos 8-15, d 0-7), (pos 0-7, d 8-15), (pos 8-15, d 8-15)
    const int bv_row = (lane & 7) + ((lane >> 3) & 1) * 8, bv_dc = (lane >> 4) & 1;

#pragma unroll 1
    for (int tile = 0; tile < ntile; tile++) {
        issue(tile + kMmaStages - 1);
        cp_async_wait_stages<kMmaStages - 1>();
        __syncthreads();
        const uint8_t* kt = ring + (size_t)(tile % kMmaStages) * 2 * SM::kTile;
        const uint32_t kt_s = smem_u32(kt), vt_s = kt_s + SM::kTile;
        const int p0 = warp * 16;  // this warp's 16 positions of the tile
        const int tb = t0 + tile * kMmaTile + p0;
        if (tb < t1) {
            float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int kk = 0; kk < KS; kk++) {
                uint32_t ah[4], al[4], bkr[4];
                ldsm4(qh_s + sw_off<HD>(a_row, 2 * kk + a_kc), ah);
                ldsm4(ql_s + sw_off<HD>(a_row, 2 * kk + a_kc), al);
                ldsm4(kt_s + sw_off<HD>(p0 + bk_row, 2 * kk + bk_kc), bkr);
                mma_f16_16816(s0, ah, bkr[0], bkr[1]);
                mma_f16_16816(s0, al, bkr[0], bkr[1]);
                mma_f16_16816(s1, ah, bkr[2], bkr[3]);
                mma_f16_16816(s1, al, bkr[2], bkr[3]);
            }
            // positions past the slice: score -inf
            const int c0 = tb + 2 * ti, c1 = tb + 8 + 2 * ti;
            if (c0 >= t1) { s0[0] = -INFINITY; s0[2] = -INFINITY; }
            if (c0 + 1 >= t1) { s0[1] = -INFINITY; s0[3] = -INFINITY; }
            if (c1 >= t1) { s1[0] = -INFINITY; s1[2] = -INFINITY; }
            if (c1 + 1 >= t1) { s1[1] = -INFINITY; s1[3] = -INFINITY; }
            // online softmax per row (row gi: s*[0..1], row gi + 8: s*[2..3])
            float r0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
            float r1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
            r0 = fmaxf(r0, __shfl_xor_sync(0xffffffffu, r0, 1));
            r1 = fmaxf(r1, __shfl_xor_sync(0xffffffffu, r1, 1));
            r0 = fmaxf(r0, __shfl_xor_sync(0xffffffffu, r0, 2));
            r1 = fmaxf(r1, __shfl_xor_sync(0xffffffffu, r1, 2));
            const float n0 = fmaxf(m0, r0), n1 = fmaxf(m1, r1);  // (finite: position tb is valid)
            const float f0 = m0 == -INFINITY ? 0.0f : __expf(m0 - n0), f1 = m1 == -INFINITY ? 0.0f : __expf(m1 - n1);
            m0 = n0;
            m1 = n1;
            float p[8] = {__expf(s0[0] - n0), __expf(s0[1] - n0), __expf(s0[2] - n1), __expf(s0[3] - n1),
                          __expf(s1[0] - n0), __expf(s1[1] - n0), __expf(s1[2] - n1), __expf(s1[3] - n1)};
            l0 = fmaf(l0, f0, p[0] + p[1] + p[4] + p[5]);
            l1 = fmaf(l1, f1, p[2] + p[3] + p[6] + p[7]);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                o[n][0] *= f0; o[n][1] *= f0; o[n][2] *= f1; o[n][3] *= f1;
            }
            // P as the A fragment of P V: (row gi, k 2ti..), (row gi + 8, ..), (row gi, k 8 + 2ti..), (row gi + 8, ..)
            uint32_t ph[4], pl[4];
            split2(p[0], p[1], ph[0], pl[0]);
            split2(p[2], p[3], ph[1], pl[1]);
            split2(p[4], p[5], ph[2], pl[2]);
            split2(p[6], p[7], ph[3], pl[3]);
#pragma unroll
            for (int n2 = 0; n2 < NT / 2; n2++) {  // two n8 tiles (16 dims) per transposed load
                uint32_t bvr[4];
                ldsm4_t(vt_s + sw_off<HD>(p0 + bv_row, 2 * n2 + bv_dc), bvr);
                mma_f16_16816(o[2 * n2], ph, bvr[0], bvr[1]);
                mma_f16_16816(o[2 * n2], pl, bvr[0], bvr[1]);
                mma_f16_16816(o[2 * n2 + 1], ph, bvr[2], bvr[3]);
                mma_f16_16816(o[2 * n2 + 1], pl, bvr[2], bvr[3]);
            }
        }
        __syncthreads();  // the slot is refilled by the next iteration's issue
    }
    cp_async_wait();
    // row sums over the four lanes of a row
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    // merge the warps: [warp][16 rows][HD + 2] floats over the ring
    __syncthreads();
    float* mw = reinterpret_cast<float*>(ring);
    float* wr = mw + (size_t)warp * 16 * (HD + 2);
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int d = n * 8 + 2 * ti;
        wr[gi * (HD + 2) + d] = o[n][0];
        wr[gi * (HD + 2) + d + 1] = o[n][1];
        wr[(gi + 8) * (HD + 2) + d] = o[n][2];
        wr[(gi + 8) * (HD + 2) + d + 1] = o[n][3];
    }
    if (ti == 0) {
        wr[gi * (HD + 2) + HD] = m0;
        wr[gi * (HD + 2) + HD + 1] = l0;
        wr[(gi + 8) * (HD + 2) + HD] = m1;
        wr[(gi + 8) * (HD + 2) + HD + 1] = l1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < grp * (HD + 2); i += kMmaThreads) {
        const int h = i / (HD + 2), d = i - h * (HD + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; w++) M = fmaxf(M, mw[((size_t)w * 16 + h) * (HD + 2) + HD]);
        float val = M;
        if (d != HD) {
            val = 0.0f;
#pragma unroll
            for (int w = 0; w < 4; w++) {
                const float* pw = mw + ((size_t)w * 16 + h) * (HD + 2);
                const float f = pw[HD] == -INFINITY ? 0.0f : __expf(pw[HD] - M);
                val = fmaf(pw[d], f, val);
            }
        }
        part[(((size_t)b * nh + (size_t)g * grp + h) * S + s) * (HD + 2) + d] = val;
    }
}

constexpr int kMaxAttnDevices = 64;

template <int HD, bool VAR>
bool launch_mma_hd(int grp, int grid, cudaStream_t st, const float* q, const __half* k, const __half* v, float* part,
                   int nh, int nkv, int ctx, int S, const AttnSeqs& seqs) {
    // the attribute belongs to a device: set on each device's first launch
    static std::atomic<bool> attr[kMaxAttnDevices] = {};
    constexpr int smem = MmaSmem<HD>::kTotal;
    static_assert(4 * 16 * (HD + 2) * 4 <= MmaSmem<HD>::kRing, "the warp merge fits over the ring");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxAttnDevices) return false;
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(attn_mma_kernel<HD, VAR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return false;
        attr[dev] = true;
    }
    launch_pdl(attn_mma_kernel<HD, VAR>, dim3(grid), dim3(kMmaThreads), smem, st, q, k, v, part, nh, nkv, grp, ctx, S,
               seqs);
    return true;
}

// Launches attn_split_kernel for head dimension hd (64, 128, 256) and group
// size grp (1 .. 8); returns false for other geometries.
template <int HD, bool VAR>
bool launch_split_hd(int grp, int grid, cudaStream_t st, const float* q, const __half* k, const __half* v, float* part,
                     int nh, int nkv, int ctx, int S, const AttnSeqs& seqs) {
    auto go = [&](auto kern, int g) {
        const size_t smem = sizeof(float) * (size_t)kAttWarps * g * (HD + 2);
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        launch_pdl(kern, dim3(grid), dim3(kAttThreads), smem, st, q, k, v, part, nh, nkv, ctx, S, seqs);
        return true;
    };
    switch (grp) {
        case 1: return go(attn_split_kernel<HD, 1, VAR>, 1);
        case 2: return go(attn_split_kernel<HD, 2, VAR>, 2);
        case 3: return go(attn_split_kernel<HD, 3, VAR>, 3);
        case 4: return go(attn_split_kernel<HD, 4, VAR>, 4);
        case 5: return go(attn_split_kernel<HD, 5, VAR>, 5);
        case 6: return go(attn_split_kernel<HD, 6, VAR>, 6);
        case 7: return go(attn_split_kernel<HD, 7, VAR>, 7);
        case 8: return go(attn_split_kernel<HD, 8, VAR>, 8);
        default: return false;
    }
}

// seqs null: every sequence has ctx positions stored back to back.
bool launch_split(int hd, int grp, int grid, cudaStream_t st, const float* q, const __half* k, const __half* v,
                  float* part, int nh, int nkv, int ctx, int S, const AttnSeqs* seqs = nullptr) {
    const AttnSeqs none{nullptr, 0, 0};
    if (grp <= kMmaMaxGrp && (hd == 64 || hd == 128)) {  // the tensor-core form
        if (hd == 64)
            return seqs ? launch_mma_hd<64, true>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, *seqs)
                        : launch_mma_hd<64, false>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, none);
        return seqs ? launch_mma_hd<128, true>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, *seqs)
                    : launch_mma_hd<128, false>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, none);
    }
    switch (hd) {
        case 64:
            return seqs ? launch_split_hd<64, true>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, *seqs)
                        : launch_split_hd<64, false>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, none);
        case 128:
            return seqs ? launch_split_hd<128, true>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, *seqs)
                        : launch_split_hd<128, false>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, none);
        case 256:
            return seqs ? launch_split_hd<256, true>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, *seqs)
                        : launch_split_hd<256, false>(grp, grid, st, q, k, v, part, nh, nkv, ctx, S, none);
        default: return false;
    }
}

__global__ void attn_merge_kernel(const float* __restrict__ part, float* __restrict__ out, int nh, int hd, int S) {
    pdl_trigger();
    pdl_wait();
    const int bh = blockIdx.x;  // sequence * nh + head
    const float* ph = part + (size_t)bh * S * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, ph[s * (hd + 2) + hd]);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float L = 0.0f, o = 0.0f;
        for (int s = 0; s < S; s++) {
            const float ms = ph[s * (hd + 2) + hd];
            const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            L = fmaf(ph[s * (hd + 2) + hd + 1], w, L);
            o = fmaf(ph[s * (hd + 2) + d], w, o);
        }
        out[(size_t)bh * hd + d] = o / L;
    }
}

}  // namespace

// Context splits per (sequence, KV head): up to two CTAs per SM worth, or
// more while every split keeps at least 256 positions (four K / V tiles:
// the per-CTA setup stays small against them) up to four times that, never
// under 64 positions a split; among those the count whose CTAs fill their
// last wave best (two CTAs per SM: the tensor-core form's shared memory and
// registers), the smallest on a tie, so no wave runs a few CTAs alone.
int attention_splits(int batch, int nkv, int ctx, int sms) {
    const int units = std::max(1, batch * nkv);
    const int slots = 2 * sms;
    const int want = (slots + units - 1) / units;
    const int by_len = std::max(1, (ctx + 63) / 64);
    const int cap = std::max(1, std::min(by_len, std::max(want, std::min(4 * want, ctx / 256))));
    auto fill = [&](int s) {
        const long long ctas = (long long)units * s, waves = (ctas + slots - 1) / slots;
        return (double)ctas / (double)(waves * slots);
    };
    int best = 1;
    for (int s = 2; s <= cap; s++)
        if (fill(s) > fill(best) + 1e-9) best = s;
    return best;
}

int matvec_lean(int qtype, const void* w, const float* x, float* y, int rows, int cols, int sms, cudaStream_t s,
                std::string* err);

}  // namespace b2

using namespace b2;

int b2_matvec_impl(int qtype, const void* w, const float* x, float* y, int rows, int cols, cudaStream_t s,
                   std::string* err) {
    DeviceScratch* sc = scratch_for_current(err);
    if (!sc) return B2_ERR_CUDA;
    // rows of a multiple of 256 columns: the matvec kernel of its own; other
    // widths: the decode kernel's single-phase mode
    {
        const int lean = matvec_lean(qtype, w, x, y, rows, cols, sc->sms, s, err);
        if (lean <= 0) return lean;
    }
    if (reinterpret_cast<uintptr_t>(w) & 15) {
        *err = "weight pointer must be 16-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    ModelDev m{};
    m.qtype = qtype;
    const int bpb = qtype == 8 ? 34 : 18;
    const int rb = cols / 32 * bpb;
    m.xs_floats = (cols + 31) & ~31;
    m.ybuf_floats = ((rows + sc->sms - 1) / sc->sms + 31) & ~31;
    m.ybuf_odd = m.ybuf_floats;
    m.cfloats = 32;
    m.nbx = 0;
    const int need = rb + 32;
    const int slot = std::max(8192, (need + 1023) & ~1023);
    int ns = 0;
    while (ns < 32 && smem_offsets(ns + 1, slot, m.xs_floats, m.ybuf_floats + m.ybuf_odd, m.cfloats, 0, 0).total <= 232448u) ns++;
    if (ns < 2) {
        *err = "matrix rows too wide for the shared-memory ring";
        return B2_ERR_BAD_ARG;
    }
    m.slot_bytes = slot;
    m.nslots = ns;
    m.err = sc->err;
    StepArgs a{};
    a.mv_w = static_cast<const uint8_t*>(w);
    a.mv_x = x;
    a.mv_y = y;
    a.mv_rows = rows;
    a.mv_cols = cols;
    a.mv_rb = rb;
    a.p_begin = 0;
    a.p_end = 1;
    return launch_decode(m, a, sc->sms, s, err);
}

// The allocating entry point's split partials, one buffer per (device,
// stream): calls on one stream are ordered and share it; calls on different
// streams never race on each other's.
struct AttnScratch {
    float* part = nullptr;
    size_t part_floats = 0;
};
std::map<std::pair<int, cudaStream_t>, AttnScratch> g_attn_scratch;  // under g_mu

int b2_attention_impl(const float* q, const uint16_t* k, const uint16_t* v, float* out, int batch, int nh, int nkv,
                      int hd, int ctx, cudaStream_t s, std::string* err) {
    const int grp = nh / nkv;
    if (grp > kMaxGrp || hd % 32 || hd / 32 > kMaxDimsLane) {
        *err = "attention geometry unsupported (need nh/nkv <= 8 and head_dim in {64, 128, 256})";
        return B2_ERR_BAD_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) {
        *err = "q, k and v must be 16-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    DeviceScratch* sc = scratch_for_current(err);
    if (!sc) return B2_ERR_CUDA;
    int dev = 0;
    cudaGetDevice(&dev);
    const int S = attention_splits(batch, nkv, ctx, sc->sms);
    const size_t need = (size_t)batch * nh * S * (hd + 2);
    float* part;
    {
        std::lock_guard<std::mutex> g(g_mu);
        AttnScratch& a = g_attn_scratch[{dev, s}];
        if (a.part_floats < need) {
            if (a.part) cudaFree(a.part);
            a.part = nullptr;
            a.part_floats = 0;
            if (cudaMalloc(&a.part, need * sizeof(float)) != cudaSuccess) {
                *err = "scratch allocation failed";
                return B2_ERR_OOM;
            }
            a.part_floats = need;
        }
        part = a.part;
    }
    const int grid = batch * nkv * S;
    const __half* kh = reinterpret_cast<const __half*>(k);
    const __half* vh = reinterpret_cast<const __half*>(v);
    if (!launch_split(hd, grp, grid, s, q, kh, vh, part, nh, nkv, ctx, S)) {
        *err = "head_dim must be 64, 128 or 256";
        return B2_ERR_BAD_ARG;
    }
    launch_pdl(attn_merge_kernel, dim3(batch * nh), dim3(std::min(hd, 256)), 0, s, part, out, nh, hd, S);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("attention launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

// Attention of a batch of decode sequences with lengths of their own: q
// [batch][nh*hd]; sequence b has lens[b] + add cached positions at k, v +
// b * stride * nkv * hd (fp16).  part holds part_floats floats for the split
// partials (the split count is capped to fit).  Used by the batched decode.
int b2_attention_seqs_launch(const float* q, const __half* k, const __half* v, float* part, size_t part_floats,
                             float* out, int batch, int nh, int nkv, int hd, const int* lens, int add, int stride,
                             int max_len, int sms, cudaStream_t s) {
    const int grp = nh / nkv;
    if (grp > kMaxGrp || (hd != 64 && hd != 128 && hd != 256)) return B2_ERR_UNSUPPORTED_TYPE;
    int S = attention_splits(batch, nkv, max_len, sms);
    const size_t per_split = (size_t)batch * nh * (hd + 2);
    S = (int)std::max<size_t>(1, std::min<size_t>((size_t)S, part_floats / per_split));
    const AttnSeqs seqs{lens, add, stride};
    if (!launch_split(hd, grp, batch * nkv * S, s, q, k, v, part, nh, nkv, 0, S, &seqs)) return B2_ERR_UNSUPPORTED_TYPE;
    launch_pdl(attn_merge_kernel, dim3(batch * nh), dim3(std::min(hd, 256)), 0, s, part, out, nh, hd, S);
    return cudaGetLastError() == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the attention entry point.
//
// The split partials live in one file-scope device array instead of memory
// obtained with cudaMalloc, so a call allocates nothing.  Every GPU that loads
// this library holds the array (kNoAllocScratchFloats floats, 2 MiB) until
// the process exits.  Its address comes from cudaGetSymbolAddress, once per
// device, on that device's first call; the host-side name of the array is
// only a stand-in and is never passed to a kernel.  All calls share the
// array and it keeps the last call's contents: nothing in it needs to start
// at zero, because the partial kernel writes every entry (o, m, l of each
// head and split) that the merge kernel then reads.  Calls whose kernels
// overlap on the GPU (different streams, or different host threads without
// ordering) race on the array.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchFloats = 512 * 1024;
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_part[kNoAllocMaxDevices] = {};
int g_noalloc_sms[kNoAllocMaxDevices] = {};
}  // namespace

static __device__ __align__(256) float b2_attn_noalloc_scratch[kNoAllocScratchFloats];

int b2_attention_noalloc_impl(const float* q, const uint16_t* k, const uint16_t* v, float* out, int batch, int nh,
                              int nkv, int hd, int ctx, cudaStream_t s, std::string* err) {
    const int grp = nh / nkv;
    if (grp > kMaxGrp || hd % 32 || hd / 32 > kMaxDimsLane || (hd != 64 && hd != 128 && hd != 256)) {
        *err = "attention geometry unsupported (need nh/nkv <= 8 and head_dim in {64, 128, 256})";
        return B2_ERR_BAD_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) {
        *err = "q, k and v must be 16-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    const size_t per_split = (size_t)batch * nh * (hd + 2);
    if (per_split > kNoAllocScratchFloats) {
        *err = "batch * num_heads * (head_dim + 2) = " + std::to_string(per_split) +
               " floats exceeds the allocation-free scratch of " + std::to_string(kNoAllocScratchFloats) +
               " floats; use b2_attention_decode for this size";
        return B2_ERR_BAD_ARG;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        *err = "device ordinal beyond the allocation-free entry point's table";
        return B2_ERR_BAD_ARG;
    }
    float* part = nullptr;
    int sms = 0;
    {
        // once per device, with that device current
        std::lock_guard<std::mutex> g(g_noalloc_mu);
        if (!g_noalloc_part[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, b2_attn_noalloc_scratch);
            if (e != cudaSuccess) {
                *err = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
                return B2_ERR_CUDA;
            }
            int n = 0;
            e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) {
                *err = std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e);
                return B2_ERR_CUDA;
            }
            g_noalloc_sms[dev] = n;
            g_noalloc_part[dev] = static_cast<float*>(p);
        }
        part = g_noalloc_part[dev];
        sms = g_noalloc_sms[dev];
    }
    int S = attention_splits(batch, nkv, ctx, sms);
    S = std::min<int>(S, (int)(kNoAllocScratchFloats / per_split));
    const int grid = batch * nkv * S;
    const __half* kh = reinterpret_cast<const __half*>(k);
    const __half* vh = reinterpret_cast<const __half*>(v);
    if (!launch_split(hd, grp, grid, s, q, kh, vh, part, nh, nkv, ctx, S)) {
        *err = "head_dim must be 64, 128 or 256";
        return B2_ERR_BAD_ARG;
    }
    attn_merge_kernel<<<batch * nh, std::min(hd, 256), 0, s>>>(part, out, nh, hd, S);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("attention launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}
