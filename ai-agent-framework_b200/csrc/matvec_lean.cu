// b2_matvec over the caller's ggml block rows (transformer.go:810-865
// matVecMulQ8Chunk): y[r] = sum_b d_rb * sum_j q_rbj * x[32b + j], Q8_0 or
// Q4_0, one vector.  A kernel of its own (no persistent-kernel start-up):
//
//   * the vector is split once per CTA, in shared memory, into three int8
//     planes per 32-block, x ~= s_b (p0 + p1 / 2^7 + p2 / 2^14) with
//     s_b = max|x_b| / 127 (|x - x'| <= 2^-15 s_b per element);
//   * each warp owns rows (row r, r + all warps, ...) and streams them in
//     chunks of 64 blocks through a warp-private cp.async ring in shared
//     memory (16-byte copies: rows of a multiple of 256 columns start on a
//     16-byte boundary);
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

constexpr int kLvWarps = 16;                 // (the shared-memory loads' latency wants many warps)
constexpr int kLvThreads = 32 * kLvWarps;
constexpr int kLvChunk = 64;                  // blocks per chunk: 2 per lane
constexpr int kLvStages = 3;                  // ring depth per warp
constexpr int kLvChunkBytes = kLvChunk * 34;  // a Q8_0 chunk (a Q4_0 one is 2304 bytes)

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
size_t lean_smem_bytes(int nb) {
    const size_t planes = (size_t)nb * 96 + (size_t)nb * 4 + (size_t)nb * 16;
    return ((planes + 15) & ~size_t(15)) + (size_t)kLvWarps * kLvStages * kLvChunkBytes;
}

template <int QT>
__global__ void __launch_bounds__(kLvThreads, 1)
    matvec_lean_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x, float* __restrict__ y, int rows,
                       int cols) {
    constexpr int BPB = QT == 8 ? 34 : 18;  // bytes per block
    extern __shared__ __align__(16) uint8_t lsm[];
    const int nb = cols / 32;
    int8_t* xp = reinterpret_cast<int8_t*>(lsm);
    float* xs = reinterpret_cast<float*>(lsm + (size_t)nb * 96);
    int* xsum = reinterpret_cast<int*>(xs + nb);
    const size_t planes_bytes = ((size_t)nb * 96 + (size_t)nb * 4 + (size_t)nb * 16 + 15) & ~size_t(15);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* ring = lsm + planes_bytes + (size_t)warp * kLvStages * kLvChunkBytes;

    // the vector's planes, one block per thread at a time
    for (int b = threadIdx.x; b < nb; b += kLvThreads) {
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

    const size_t rb = (size_t)nb * BPB;
    const int nch = (nb + kLvChunk - 1) / kLvChunk;
    const int r0 = blockIdx.x * kLvWarps + warp, rstep = gridDim.x * kLvWarps;
    const int nrows = r0 < rows ? (rows - r0 + rstep - 1) / rstep : 0;
    const int total = nrows * nch;
    auto issue = [&](int t) {
        if (t < total) {
            const int row = r0 + (t / nch) * rstep, c = t % nch;
            const int nbk = min(kLvChunk, nb - c * kLvChunk);
            const uint8_t* src = w + (size_t)row * rb + (size_t)c * kLvChunk * BPB;
            uint8_t* dst = ring + (size_t)(t % kLvStages) * kLvChunkBytes;
            const int n16 = nbk * BPB / 16;
            for (int i = lane; i < n16; i += 32) cp_async16(dst + 16 * i, src + 16 * i);
        }
        cp_async_commit();  // (empty groups keep the count uniform)
    };
#pragma unroll
    for (int t = 0; t < kLvStages - 1; t++) issue(t);
    float acc = 0.0f;
    for (int t = 0; t < total; t++) {
        issue(t + kLvStages - 1);
        cp_async_wait_n<kLvStages - 1>();
        __syncwarp();
        const int c = t % nch;
        const int nbk = min(kLvChunk, nb - c * kLvChunk);
        const uint8_t* chunk = ring + (size_t)(t % kLvStages) * kLvChunkBytes;
#pragma unroll
        for (int i = 0; i < kLvChunk / 32; i++) {
            const int j = lane + 32 * i;
            if (j < nbk) {
                const int gb = c * kLvChunk + j;
                const int off = j * BPB;
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(chunk + (off & ~3));
                // byte offset 0 or 2 within the first word: the quants start 2 bytes later
                const bool odd = (off & 3) != 0;
                const uint32_t sel = odd ? 0x7654u : 0x5432u;
                const uint32_t w0 = wp[0];
                const uint16_t dbits = odd ? (uint16_t)(w0 >> 16) : (uint16_t)(w0 & 0xFFFFu);
                const float d = __half2float(__ushort_as_half(dbits));
                const int4* xq = reinterpret_cast<const int4*>(xp + (size_t)gb * 96);
                int a0 = 0, a1 = 0, a2 = 0;
                if (QT == 8) {
                    uint32_t q[8];
                    uint32_t prev = w0;
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const uint32_t nxt = wp[k + 1];
                        q[k] = __byte_perm(prev, nxt, sel);
                        prev = nxt;
                    }
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int4 x0 = xq[h], x1 = xq[2 + h], x2 = xq[4 + h];
                        a0 = dp4a_ss((int)q[4 * h], x0.x, a0); a0 = dp4a_ss((int)q[4 * h + 1], x0.y, a0);
                        a0 = dp4a_ss((int)q[4 * h + 2], x0.z, a0); a0 = dp4a_ss((int)q[4 * h + 3], x0.w, a0);
                        a1 = dp4a_ss((int)q[4 * h], x1.x, a1); a1 = dp4a_ss((int)q[4 * h + 1], x1.y, a1);
                        a1 = dp4a_ss((int)q[4 * h + 2], x1.z, a1); a1 = dp4a_ss((int)q[4 * h + 3], x1.w, a1);
                        a2 = dp4a_ss((int)q[4 * h], x2.x, a2); a2 = dp4a_ss((int)q[4 * h + 1], x2.y, a2);
                        a2 = dp4a_ss((int)q[4 * h + 2], x2.z, a2); a2 = dp4a_ss((int)q[4 * h + 3], x2.w, a2);
                    }
                } else {
                    // byte i: low nibble = element i, high nibble = element i + 16
                    uint32_t q[4];
                    uint32_t prev = w0;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t nxt = wp[k + 1];
                        q[k] = __byte_perm(prev, nxt, sel);
                        prev = nxt;
                    }
#pragma unroll
                    for (int h = 0; h < 2; h++) {  // h 0: elements 0..15 (low nibbles), 1: 16..31
                        const int4 x0 = xq[h], x1 = xq[2 + h], x2 = xq[4 + h];
                        uint32_t u[4];
#pragma unroll
                        for (int k = 0; k < 4; k++) u[k] = (h ? (q[k] >> 4) : q[k]) & 0x0F0F0F0Fu;
                        a0 = dp4a_us(u[0], x0.x, a0); a0 = dp4a_us(u[1], x0.y, a0);
                        a0 = dp4a_us(u[2], x0.z, a0); a0 = dp4a_us(u[3], x0.w, a0);
                        a1 = dp4a_us(u[0], x1.x, a1); a1 = dp4a_us(u[1], x1.y, a1);
                        a1 = dp4a_us(u[2], x1.z, a1); a1 = dp4a_us(u[3], x1.w, a1);
                        a2 = dp4a_us(u[0], x2.x, a2); a2 = dp4a_us(u[1], x2.y, a2);
                        a2 = dp4a_us(u[2], x2.z, a2); a2 = dp4a_us(u[3], x2.w, a2);
                    }
                    a0 -= 8 * xsum[4 * gb];
                    a1 -= 8 * xsum[4 * gb + 1];
                    a2 -= 8 * xsum[4 * gb + 2];
                }
                const float dot = fmaf((float)a2, 1.0f / 16384.0f, fmaf((float)a1, 1.0f / 128.0f, (float)a0));
                acc = fmaf(d * xs[gb], dot, acc);
            }
        }
        if (c == nch - 1) {  // the row's last chunk: the warp's sum
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) y[r0 + (t / nch) * rstep] = acc;
            acc = 0.0f;
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
    const size_t smem = lean_smem_bytes(cols / 32);
    if (smem > 232448) return 1;
    auto kern = qtype == 8 ? matvec_lean_kernel<8> : matvec_lean_kernel<2>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        *err = "matvec: shared-memory attribute refused";
        return B2_ERR_CUDA;
    }
    const int grid = std::max(1, std::min(sms, (rows + kLvWarps - 1) / kLvWarps));  // a warp per row at a time
    kern<<<grid, kLvThreads, smem, s>>>(static_cast<const uint8_t*>(w), x, y, rows, cols);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("matvec launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return 0;
}

}  // namespace b2
