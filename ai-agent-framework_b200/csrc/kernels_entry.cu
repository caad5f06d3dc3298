// Kernel-level entry points: the dequantising matvec on its own and the
// long-context GQA decode attention.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "model.h"

namespace b2 {
namespace {

struct DeviceScratch {
    int* err = nullptr;
    float* part = nullptr;
    size_t part_floats = 0;
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

constexpr int kAttThreads = 256;
constexpr int kAttWarps = kAttThreads / 32;
constexpr int kMaxGrp = 8;      // query heads per KV head handled in registers
constexpr int kMaxDimsLane = 8; // head_dim up to 256

// One CTA = one (sequence, KV head, context slice).  Warps take positions
// round-robin; within a warp the lanes split the head dimension.  Each warp
// keeps an online softmax (m, l, o) per query head; the CTA merges its warps
// and writes one partial (o unnormalised, m, l) per query head.
template <int DPL>  // dims per lane = hd / 32
__global__ void __launch_bounds__(kAttThreads) attn_partial_kernel(const float* __restrict__ q, const __half* __restrict__ k,
                                                                   const __half* __restrict__ v, float* __restrict__ part,
                                                                   int nh, int nkv, int hd, int ctx, int S) {
    extern __shared__ float sm[];
    const int grp = nh / nkv;
    const int cta = blockIdx.x;
    const int s = cta % S, g = (cta / S) % nkv, b = cta / (S * nkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = (int)((long long)s * ctx / S), t1 = (int)((long long)(s + 1) * ctx / S);
    const size_t kvd = (size_t)nkv * hd;
    const __half* kb = k + (size_t)b * ctx * kvd + (size_t)g * hd + lane * DPL;
    const __half* vb = v + (size_t)b * ctx * kvd + (size_t)g * hd + lane * DPL;
    const float scale = (float)(1.0 / sqrt((double)hd));

    float qr[kMaxGrp][DPL];
#pragma unroll
    for (int h = 0; h < kMaxGrp; h++)
#pragma unroll
        for (int d = 0; d < DPL; d++)
            qr[h][d] = (h < grp) ? q[((size_t)b * nh + g * grp + h) * hd + lane * DPL + d] : 0.0f;

    float mrun[kMaxGrp], lrun[kMaxGrp], o[kMaxGrp][DPL];
#pragma unroll
    for (int h = 0; h < kMaxGrp; h++) {
        mrun[h] = -INFINITY;
        lrun[h] = 0.0f;
#pragma unroll
        for (int d = 0; d < DPL; d++) o[h][d] = 0.0f;
    }

    for (int t = t0 + warp; t < t1; t += kAttWarps) {
        float kf[DPL], vf[DPL];
        if (DPL == 4) {
            const uint2 ku = __ldg(reinterpret_cast<const uint2*>(kb + (size_t)t * kvd));
            const uint2 vu = __ldg(reinterpret_cast<const uint2*>(vb + (size_t)t * kvd));
            const __half2* kh = reinterpret_cast<const __half2*>(&ku);
            const __half2* vh = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
            for (int e = 0; e < DPL / 2; e++) {
                float2 a = __half22float2(kh[e]), c = __half22float2(vh[e]);
                kf[2 * e] = a.x; kf[2 * e + 1] = a.y; vf[2 * e] = c.x; vf[2 * e + 1] = c.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < DPL; e += 2) {
                float2 a = __half22float2(*reinterpret_cast<const __half2*>(kb + (size_t)t * kvd + e));
                float2 c = __half22float2(*reinterpret_cast<const __half2*>(vb + (size_t)t * kvd + e));
                kf[e] = a.x; kf[e + 1] = a.y; vf[e] = c.x; vf[e + 1] = c.y;
            }
        }
#pragma unroll
        for (int h = 0; h < kMaxGrp; h++) {
            if (h >= grp) break;
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < DPL; d++) dot = fmaf(qr[h][d], kf[d], dot);
            dot = warp_sum(dot) * scale;
            const float mn = fmaxf(mrun[h], dot);
            const float c = expf(mrun[h] - mn);  // exp(-inf) = 0 on the first position
            const float p = expf(dot - mn);
            lrun[h] = lrun[h] * c + p;
            mrun[h] = mn;
#pragma unroll
            for (int d = 0; d < DPL; d++) o[h][d] = fmaf(p, vf[d], o[h][d] * c);
        }
    }

    // merge the warps of this CTA
    float* wm = sm;                                  // [warps][grp]
    float* wl = wm + kAttWarps * kMaxGrp;            // [warps][grp]
    float* wo = wl + kAttWarps * kMaxGrp;            // [warps][grp][hd]
    for (int h = 0; h < grp; h++) {
        if (lane == 0) { wm[warp * kMaxGrp + h] = mrun[h]; wl[warp * kMaxGrp + h] = lrun[h]; }
#pragma unroll
        for (int d = 0; d < DPL; d++) wo[((size_t)warp * kMaxGrp + h) * hd + lane * DPL + d] = o[h][d];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < grp * (hd + 2); i += kAttThreads) {
        const int h = i / (hd + 2), d = i % (hd + 2);
        float M = -INFINITY;
        for (int w = 0; w < kAttWarps; w++) M = fmaxf(M, wm[w * kMaxGrp + h]);
        float val = 0.0f;
        if (d == hd) {
            val = M;
        } else {
            for (int w = 0; w < kAttWarps; w++) {
                const float mw = wm[w * kMaxGrp + h];
                const float f = (mw == -INFINITY) ? 0.0f : expf(mw - M);
                val = fmaf(d < hd ? wo[((size_t)w * kMaxGrp + h) * hd + d] : wl[w * kMaxGrp + h], f, val);
            }
        }
        part[(((size_t)b * nh + g * grp + h) * S + s) * (hd + 2) + d] = val;
    }
}

__global__ void attn_merge_kernel(const float* __restrict__ part, float* __restrict__ out, int nh, int hd, int S) {
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

int attention_splits(int batch, int nkv, int ctx, int sms) {
    const int want = (2 * sms + batch * nkv - 1) / (batch * nkv);
    const int by_len = (ctx + 63) / 64;
    return std::max(1, std::min(want, by_len));
}

}  // namespace b2

using namespace b2;

int b2_matvec_impl(int qtype, const void* w, const float* x, float* y, int rows, int cols, cudaStream_t s,
                   std::string* err) {
    DeviceScratch* sc = scratch_for_current(err);
    if (!sc) return B2_ERR_CUDA;
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

int b2_attention_impl(const float* q, const uint16_t* k, const uint16_t* v, float* out, int batch, int nh, int nkv,
                      int hd, int ctx, cudaStream_t s, std::string* err) {
    const int grp = nh / nkv;
    if (grp > kMaxGrp || hd % 32 || hd / 32 > kMaxDimsLane) {
        *err = "attention geometry unsupported (need nh/nkv <= 8 and head_dim in {64, 128, 256})";
        return B2_ERR_BAD_ARG;
    }
    DeviceScratch* sc = scratch_for_current(err);
    if (!sc) return B2_ERR_CUDA;
    const int S = attention_splits(batch, nkv, ctx, sc->sms);
    const size_t need = (size_t)batch * nh * S * (hd + 2);
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (sc->part_floats < need) {
            if (sc->part) cudaFree(sc->part);
            sc->part = nullptr;
            sc->part_floats = 0;
            if (cudaMalloc(&sc->part, need * sizeof(float)) != cudaSuccess) {
                *err = "scratch allocation failed";
                return B2_ERR_OOM;
            }
            sc->part_floats = need;
        }
    }
    const size_t smem = sizeof(float) * (2 * kAttWarps * kMaxGrp + (size_t)kAttWarps * kMaxGrp * hd);
    const int grid = batch * nkv * S;
    const __half* kh = reinterpret_cast<const __half*>(k);
    const __half* vh = reinterpret_cast<const __half*>(v);
    switch (hd / 32) {
        case 2:
            cudaFuncSetAttribute(attn_partial_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attn_partial_kernel<2><<<grid, kAttThreads, smem, s>>>(q, kh, vh, sc->part, nh, nkv, hd, ctx, S);
            break;
        case 4:
            cudaFuncSetAttribute(attn_partial_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attn_partial_kernel<4><<<grid, kAttThreads, smem, s>>>(q, kh, vh, sc->part, nh, nkv, hd, ctx, S);
            break;
        case 8:
            cudaFuncSetAttribute(attn_partial_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            attn_partial_kernel<8><<<grid, kAttThreads, smem, s>>>(q, kh, vh, sc->part, nh, nkv, hd, ctx, S);
            break;
        default:
            *err = "head_dim must be 64, 128 or 256";
            return B2_ERR_BAD_ARG;
    }
    attn_merge_kernel<<<batch * nh, std::min(hd, 256), 0, s>>>(sc->part, out, nh, hd, S);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("attention launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
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
    const size_t smem = sizeof(float) * (2 * kAttWarps * kMaxGrp + (size_t)kAttWarps * kMaxGrp * hd);
    const int grid = batch * nkv * S;
    const __half* kh = reinterpret_cast<const __half*>(k);
    const __half* vh = reinterpret_cast<const __half*>(v);
    if (hd == 64) {
        attn_partial_kernel<2><<<grid, kAttThreads, smem, s>>>(q, kh, vh, part, nh, nkv, hd, ctx, S);
    } else if (hd == 128) {
        attn_partial_kernel<4><<<grid, kAttThreads, smem, s>>>(q, kh, vh, part, nh, nkv, hd, ctx, S);
    } else {
        cudaFuncSetAttribute(attn_partial_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attn_partial_kernel<8><<<grid, kAttThreads, smem, s>>>(q, kh, vh, part, nh, nkv, hd, ctx, S);
    }
    attn_merge_kernel<<<batch * nh, std::min(hd, 256), 0, s>>>(part, out, nh, hd, S);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("attention launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}
