// b2_matvec over the caller's ggml block rows (transformer.go:810-865
// matVecMulQ8Chunk): y[r] = sum_b d_rb * sum_j q_rbj * x[32b + j], Q8_0 or
// Q4_0, one vector.  A kernel of its own (no persistent-kernel start-up):
//
//   * the vector is split once per CTA, in shared memory, into three int8
//     planes per 32-block, x ~= s_b (p0 + p1 / 2^7 + p2 / 2^14) with
//     s_b = max|x_b| / 127 (|x - x'| <= 2^-15 s_b per element);
//   * each warp owns pairs of rows (pair p, p + all warps, ...) and streams
//     them in chunks of 64 blocks through a warp-private cp.async ring in
//     shared memory (16-byte copies: rows of a multiple of 256 columns start
//     on a 16-byte boundary); the two rows share each block's plane loads;
//   * a lane takes whole blocks of the chunk: the 34- (18-) byte block is
//     realigned from aligned 32-bit shared loads with byte permutes, and
//     its dot with the three planes is 24 dp4a (exact int32); the block
//     adds d * s_b * (A0 + A1 / 2^7 + A2 / 2^14) to the lane's fp32 sum
//     (Q4_0: q - 8 as q against the planes less 8 times their sums);
//   * the warp's lanes are summed by shuffles.
//
// Bound: HBM (the weight bytes once); about 1.8 instructions per weight.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "../../include/b2decode.h"
#include "dev.cuh"

namespace b2 {
namespace {

constexpr int kLvChunk = 64;  // blocks per chunk: 2 per lane
constexpr int kLvStages = 3;  // ring depth per warp
// Per type: rows a warp takes at once (they share the vector's plane loads)
// and warps per CTA (the shared-memory latency wants many of them).
template <int QT>
struct LvCfg {
    static constexpr int kRows = 2;
    static constexpr int kWarps = QT == 8 ? 8 : 16;
    static constexpr int kBpb = QT == 8 ? 34 : 18;
    static constexpr int kRowChunk = kLvChunk * kBpb;   // bytes of one row's chunk
    static constexpr int kStage = kRows * kRowChunk;    // one stage: kRows row chunks
};

template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Shared memory: [nb][3][32] int8 planes, [nb] scales, [nb][4] plane sums,
// then the warps' rings (16-byte aligned).
__host__ __device__ inline size_t lean_planes_bytes(int nb) { return ((size_t)nb * 116 + 15) & ~size_t(15); }
template <int QT>
size_t lean_smem_bytes(int nb) {
    using C = LvCfg<QT>;
    return lean_planes_bytes(nb) + (size_t)C::kWarps * kLvStages * C::kStage;
}

template <int QT>
__global__ void __launch_bounds__(32 * LvCfg<QT>::kWarps, 1)
    matvec_lean_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x, float* __restrict__ y, int rows,
                       int cols) {
    using C = LvCfg<QT>;
    constexpr int BPB = C::kBpb, RW = C::kRows, NW = C::kWarps;
    extern __shared__ __align__(16) uint8_t lsm[];
    const int nb = cols / 32;
    int8_t* xp = reinterpret_cast<int8_t*>(lsm);
    float* xs = reinterpret_cast<float*>(lsm + (size_t)nb * 96);
    int* xsum = reinterpret_cast<int*>(xs + nb);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = lsm + lean_planes_bytes(nb) + (size_t)warp * kLvStages * C::kStage;

    // the vector's planes, one block per thread at a time
    for (int b = threadIdx.x; b < nb; b += 32 * NW) {
        const float4* xb = reinterpret_cast<const float4*>(x + (size_t)b * 32);
        float v[32];
        float mx = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 t = __ldg(xb + i);
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
#pragma unroll
        for (int i = 0; i < 32; i++) mx = fmaxf(mx, fabsf(v[i]));
        const float s = mx > 0.0f ? mx / 127.0f : 1.0f;
        int s0 = 0, s1 = 0, s2 = 0;
        int8_t* pb = xp + (size_t)b * 96;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const float u = v[i] / s;
            const float p0 = rintf(u), r1 = (u - p0) * 128.0f;
            const float p1 = rintf(r1), r2 = (r1 - p1) * 128.0f;
            const float p2 = rintf(r2);
            pb[i] = (int8_t)(int)p0;
            pb[32 + i] = (int8_t)(int)p1;
            pb[64 + i] = (int8_t)(int)p2;
            s0 += (int)p0;
            s1 += (int)p1;
            s2 += (int)p2;
        }
        xs[b] = s;
        xsum[4 * b] = s0;
        xsum[4 * b + 1] = s1;
        xsum[4 * b + 2] = s2;
    }
    __syncthreads();

    // this warp's row groups: rows g RW .. g RW + RW - 1 for g = gw, gw + all warps, ...
    const size_t rb = (size_t)nb * BPB;
    const int nch = (nb + kLvChunk - 1) / kLvChunk;
    const int ngroups = (rows + RW - 1) / RW;
    const int g0 = blockIdx.x * NW + warp, gstep = gridDim.x * NW;
    const int mine = g0 < ngroups ? (ngroups - g0 + gstep - 1) / gstep : 0;
    const int total = mine * nch;
    auto issue = [&](int t) {
        if (t < total) {
            const int grp = g0 + (t / nch) * gstep, c = t % nch;
            const int nbk = min(kLvChunk, nb - c * kLvChunk);
            const int n16 = nbk * BPB / 16;
            uint8_t* dst = ring + (size_t)(t % kLvStages) * C::kStage;
#pragma unroll
            for (int q = 0; q < RW; q++) {
                const int row = grp * RW + q;
                if (row < rows) {
                    const uint8_t* src = w + (size_t)row * rb + (size_t)c * kLvChunk * BPB;
                    for (int i = lane; i < n16; i += 32) cp_async16(dst + q * C::kRowChunk + 16 * i, src + 16 * i);
                }
            }
        }
        cp_async_commit();  // (empty groups keep the count uniform)
    };
#pragma unroll
    for (int t = 0; t < kLvStages - 1; t++) issue(t);
    float acc[RW];
#pragma unroll
    for (int q = 0; q < RW; q++) acc[q] = 0.0f;
    for (int t = 0; t < total; t++) {
        issue(t + kLvStages - 1);
        cp_async_wait_n<kLvStages - 1>();
        __syncwarp();
        const int grp = g0 + (t / nch) * gstep, c = t % nch;
        const int nbk = min(kLvChunk, nb - c * kLvChunk);
        const uint8_t* stage = ring + (size_t)(t % kLvStages) * C::kStage;
#pragma unroll
        for (int i = 0; i < kLvChunk / 32; i++) {
            const int j = lane + 32 * i;
            if (j < nbk) {
                const int gb = c * kLvChunk + j;
                const int off = j * BPB;
                // byte offset 0 or 2 within the first word: the quants start 2 bytes later
                const bool odd = (off & 3) != 0;
                const uint32_t sel = odd ? 0x7654u : 0x5432u;
                const int4* xq = reinterpret_cast<const int4*>(xp + (size_t)gb * 96);
                const int4 x00 = xq[0], x01 = xq[1], x10 = xq[2], x11 = xq[3], x20 = xq[4], x21 = xq[5];
                const float sx = xs[gb];
                int c0 = 0, c1 = 0, c2 = 0;
                if (QT != 8) {
                    c0 = 8 * xsum[4 * gb];
                    c1 = 8 * xsum[4 * gb + 1];
                    c2 = 8 * xsum[4 * gb + 2];
                }
#pragma unroll
                for (int q = 0; q < RW; q++) {
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(stage + q * C::kRowChunk + (off & ~3));
                    const uint32_t w0 = wp[0];
                    const uint16_t dbits = odd ? (uint16_t)(w0 >> 16) : (uint16_t)(w0 & 0xFFFFu);
                    const float d = __half2float(__ushort_as_half(dbits));
                    int a0 = 0, a1 = 0, a2 = 0;
                    if (QT == 8) {
                        uint32_t qv[8];
                        uint32_t prev = w0;
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            const uint32_t nxt = wp[k + 1];
                            qv[k] = __byte_perm(prev, nxt, sel);
                            prev = nxt;
                        }
                        a0 = dp4a_ss((int)qv[0], x00.x, a0); a0 = dp4a_ss((int)qv[1], x00.y, a0);
                        a0 = dp4a_ss((int)qv[2], x00.z, a0); a0 = dp4a_ss((int)qv[3], x00.w, a0);
                        a0 = dp4a_ss((int)qv[4], x01.x, a0); a0 = dp4a_ss((int)qv[5], x01.y, a0);
                        a0 = dp4a_ss((int)qv[6], x01.z, a0); a0 = dp4a_ss((int)qv[7], x01.w, a0);
                        a1 = dp4a_ss((int)qv[0], x10.x, a1); a1 = dp4a_ss((int)qv[1], x10.y, a1);
                        a1 = dp4a_ss((int)qv[2], x10.z, a1); a1 = dp4a_ss((int)qv[3], x10.w, a1);
                        a1 = dp4a_ss((int)qv[4], x11.x, a1); a1 = dp4a_ss((int)qv[5], x11.y, a1);
                        a1 = dp4a_ss((int)qv[6], x11.z, a1); a1 = dp4a_ss((int)qv[7], x11.w, a1);
                        a2 = dp4a_ss((int)qv[0], x20.x, a2); a2 = dp4a_ss((int)qv[1], x20.y, a2);
                        a2 = dp4a_ss((int)qv[2], x20.z, a2); a2 = dp4a_ss((int)qv[3], x20.w, a2);
                        a2 = dp4a_ss((int)qv[4], x21.x, a2); a2 = dp4a_ss((int)qv[5], x21.y, a2);
                        a2 = dp4a_ss((int)qv[6], x21.z, a2); a2 = dp4a_ss((int)qv[7], x21.w, a2);
                    } else {
                        // byte i: low nibble = element i, high nibble = element i + 16
                        uint32_t qv[4];
                        uint32_t prev = w0;
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const uint32_t nxt = wp[k + 1];
                            qv[k] = __byte_perm(prev, nxt, sel);
                            prev = nxt;
                        }
                        uint32_t lo[4], hi[4];
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            lo[k] = qv[k] & 0x0F0F0F0Fu;
                            hi[k] = (qv[k] >> 4) & 0x0F0F0F0Fu;
                        }
                        a0 = dp4a_us(lo[0], x00.x, a0); a0 = dp4a_us(lo[1], x00.y, a0);
                        a0 = dp4a_us(lo[2], x00.z, a0); a0 = dp4a_us(lo[3], x00.w, a0);
                        a0 = dp4a_us(hi[0], x01.x, a0); a0 = dp4a_us(hi[1], x01.y, a0);
                        a0 = dp4a_us(hi[2], x01.z, a0); a0 = dp4a_us(hi[3], x01.w, a0);
                        a1 = dp4a_us(lo[0], x10.x, a1); a1 = dp4a_us(lo[1], x10.y, a1);
                        a1 = dp4a_us(lo[2], x10.z, a1); a1 = dp4a_us(lo[3], x10.w, a1);
                        a1 = dp4a_us(hi[0], x11.x, a1); a1 = dp4a_us(hi[1], x11.y, a1);
                        a1 = dp4a_us(hi[2], x11.z, a1); a1 = dp4a_us(hi[3], x11.w, a1);
                        a2 = dp4a_us(lo[0], x20.x, a2); a2 = dp4a_us(lo[1], x20.y, a2);
                        a2 = dp4a_us(lo[2], x20.z, a2); a2 = dp4a_us(lo[3], x20.w, a2);
                        a2 = dp4a_us(hi[0], x21.x, a2); a2 = dp4a_us(hi[1], x21.y, a2);
                        a2 = dp4a_us(hi[2], x21.z, a2); a2 = dp4a_us(hi[3], x21.w, a2);
                        a0 -= c0;
                        a1 -= c1;
                        a2 -= c2;
                    }
                    const float dot = fmaf((float)a2, 1.0f / 16384.0f, fmaf((float)a1, 1.0f / 128.0f, (float)a0));
                    acc[q] = fmaf(d * sx, dot, acc[q]);
                }
            }
        }
        if (c == nch - 1) {  // the rows' last chunk: the warp's sums
#pragma unroll
            for (int q = 0; q < RW; q++) {
                float v = acc[q];
                for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int row = grp * RW + q;
                if (lane == 0 && row < rows) y[row] = v;
                acc[q] = 0.0f;
            }
        }
        __syncwarp();  // the buffer is refilled by a later issue
    }
    cp_async_wait_n<0>();
}

}  // namespace

// 0: launched; 1: the shape does not fit this kernel (the caller takes
// another path); < 0: a B2_* error.
int matvec_lean(int qtype, const void* w, const float* x, float* y, int rows, int cols, int sms, cudaStream_t s,
                std::string* err) {
    if ((qtype != 8 && qtype != 2) || cols % 256 || rows < 1 || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(x) & 15))
        return 1;
    const size_t smem = qtype == 8 ? lean_smem_bytes<8>(cols / 32) : lean_smem_bytes<2>(cols / 32);
    if (smem > 232448) return 1;
    auto kern = qtype == 8 ? matvec_lean_kernel<8> : matvec_lean_kernel<2>;
    const int warps = qtype == 8 ? LvCfg<8>::kWarps : LvCfg<2>::kWarps;
    const int rw = qtype == 8 ? LvCfg<8>::kRows : LvCfg<2>::kRows;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        *err = "matvec: shared-memory attribute refused";
        return B2_ERR_CUDA;
    }
    const int groups = (rows + rw - 1) / rw;  // a warp per group of rows at a time
    const int grid = std::max(1, std::min(sms, (groups + warps - 1) / warps));
    kern<<<grid, 32 * warps, smem, s>>>(static_cast<const uint8_t*>(w), x, y, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("matvec launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return 0;
}

}  // namespace b2
