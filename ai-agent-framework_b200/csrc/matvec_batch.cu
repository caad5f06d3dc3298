// Batched dequantising matvec: Y = W X for up to sixteen fp32 vectors in one
// pass over a Q8_0 / Q4_0 matrix, in the GGUF row layout (b2_matvec_batch)
// or in the decode kernel's tiled layout of a loaded model (b2_model_matvec
// and the batched decode).
//
// The reference evaluates one vector at a time (transformer.go:810-865
// matVecMulQ8Chunk, driven over row ranges by matVecMulQ8Pooled at
// transformer.go:868-892: per 32-block, q * d against x in fp32; Q4_0
// blocks take the same dot with (q - 8) * d, the ggml block layout).  Here
// the weights stream from HBM once for all vectors and the products run on
// the int8 tensor-core path:
//
//   * Each vector is split per 32-block into three int8 planes,
//     x ~= s * (p0 + p1 / 2^7 + p2 / 2^14) with s = max|x| / 127 (about 22
//     bits of precision relative to the block maximum, i.e. fp32-grade
//     dots).  The planes sit in global memory in the B-fragment order of
//     mma.m16n8k32, one column per vector, one mma per plane and group of
//     eight vectors (NT = 1 or 2 column tiles share each A fragment).
//   * A warp owns a unit = (16-row tile, slice of the 32-blocks).  Its weight
//     bytes stream through warp-private shared-memory stages filled with
//     cp.async (16 B, L1-bypassing), 8 blocks of the tile per stage.  Raw
//     rows: the fragments come from the 34- / 18-byte blocks with aligned
//     32-bit loads and byte permutes.  Tiled: a stage is the chunk's
//     (tile, block) units and their scales, and the fragments come by
//     ldmatrix.
//   * Each 32-block gives, per plane, the exact int32 dot in an accumulator
//     started at the float bits of 1.5 * 2^23 (Q4_0: minus 8 * the plane
//     sum, so (q - 8) . p comes out), read back with one subtraction, then
//     scaled by d_w * s_x and accumulated in fp32.
//   * With fewer tiles than warps the blocks are split into KS slices; every
//     unit writes its partial sums and the last unit of a tile to arrive
//     (an atomic counter, reset by that unit) adds the slices in slice
//     order, so results do not depend on timing.
//
// Nothing in this file waits on a flag: the only waits are cp.async
// completions of the warp's own copies.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/b2decode.h"
#include "dev.cuh"

namespace b2 {
namespace {

constexpr int kMvbVec = 8;                    // vectors per column tile (mma N)
constexpr int kMvbMaxNt = 2;                  // column tiles per pass (up to 16 vectors)
constexpr int kMvbWarps = 8;                  // warps per CTA
constexpr int kMvbThreads = kMvbWarps * 32;
constexpr int kMvbKc = 8;                     // 32-blocks per chunk
constexpr int kMvbMaxSlices = 8;
constexpr uint32_t kMvbMagic = 0x4B400000u;   // 1.5 * 2^23 as float bits
constexpr float kMvbMagicF = 12582912.0f;

// One stage holds 16 rows x one chunk of 8 blocks: raw GGUF rows (16 rows of
// rc bytes), or in the tiled layout the chunk's 8 (tile, block) units of
// 16 x qb quant bytes followed by their 8 x 16 f16 scales -- the same bytes.
template <int QT> struct MvbGeom {
    static constexpr int bpb = QT == 8 ? 34 : 18;        // bytes per 32-block
    static constexpr int qb = QT == 8 ? 32 : 16;         // quant bytes of one row's block
    static constexpr int rc = kMvbKc * bpb;              // row bytes of one chunk (16-B multiple)
    static constexpr int tile = 16 * rc;                 // one stage
    static constexpr int tsc = kMvbKc * 16 * qb;         // tiled: offset of the scales in a stage
    static constexpr int stages = QT == 8 ? 3 : 5;
    static constexpr int smem = kMvbWarps * stages * tile;
    static_assert(tsc + kMvbKc * 32 == tile, "tiled stage = raw stage bytes");
};

// Byte position of element k (0..31) of vector v inside one plane record
// (256 bytes = 32 lanes x the 8 bytes of their B fragment {b0, b1}).
// Lane (g, t) holds column g.  The natural order keeps the k slots of the
// fragment (b0: k = 4t..4t+3, b1: 16+4t..): Q4_0 rows and the tiled layout
// (ldmatrix) use it.  PERM assigns lane t the eight contiguous elements
// 8t..8t+7 (b0 then b1), which the A operand of raw Q8_0 rows mirrors.
template <bool PERM> __device__ __forceinline__ int plane_pos(int v, int k) {
    if (PERM) return v * 32 + k;
    const int kk = k & 15;
    return v * 32 + 8 * (kk >> 2) + (k >= 16 ? 4 : 0) + (kk & 3);
}

// One CTA per (32-block kb, column tile n), one warp per vector v of the
// tile, lane = element.  Record gi = kb * NT + n: planes at gi * 768 bytes
// (three 256-byte plane records), scales at gi * 8, and (Q4_0) the
// accumulator starts 1.5 * 2^23 - 8 * sum(plane) at gi * 24 + plane * 8.
// Vectors v >= nvec become zero planes with scale 0.
template <bool PERM, bool STARTS>
__global__ void __launch_bounds__(kMvbThreads)
    mvb_planes_kernel(const float* __restrict__ x, int nvec, int cols, int nt, uint8_t* __restrict__ planes,
                      float* __restrict__ xsc, uint32_t* __restrict__ xst) {
    const int gi = blockIdx.x, kb = gi / nt, n = gi - kb * nt;
    const int vl = threadIdx.x >> 5, lane = threadIdx.x & 31, v = n * kMvbVec + vl;
    const float val = v < nvec ? x[(size_t)v * cols + (size_t)kb * 32 + lane] : 0.0f;
    float amax = fabsf(val);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    const float M = kMvbMagicF;
    const float q = val * inv;
    const float f0 = q + M, r0 = f0 - M;
    const float q1 = (q - r0) * 128.0f;
    const float f1 = q1 + M, r1 = f1 - M;
    const float f2 = (q1 - r1) * 128.0f + M, r2 = f2 - M;
    const int pos = plane_pos<PERM>(vl, lane);
    uint8_t* rec = planes + (size_t)gi * 3 * 256;
    rec[pos] = (uint8_t)__float_as_uint(f0);
    rec[256 + pos] = (uint8_t)__float_as_uint(f1);
    rec[512 + pos] = (uint8_t)__float_as_uint(f2);
    if (lane == 0) xsc[gi * kMvbVec + vl] = amax * (1.0f / 127.0f);
    if (STARTS) {
        int s0 = (int)r0, s1 = (int)r1, s2 = (int)r2;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (lane == 0) {
            uint32_t* st = xst + (size_t)gi * 3 * kMvbVec + vl;
            st[0] = kMvbMagic - 8u * (uint32_t)s0;
            st[kMvbVec] = kMvbMagic - 8u * (uint32_t)s1;
            st[2 * kMvbVec] = kMvbMagic - 8u * (uint32_t)s2;
        }
    }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool U4>
__device__ __forceinline__ void mma_i8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                                       uint32_t c0, uint32_t c1, uint32_t& d0, uint32_t& d1, uint32_t& d2,
                                       uint32_t& d3) {
    if (U4) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %11, %12, %13};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %11, %12, %13};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
    }
}

// Two A-operand words of one row of block b from its raw bytes in shared
// memory (blk = the block's first byte, the fp16 scale).  Q8_0: elements
// 8t..8t+7 (quants start 2 bytes in); Q4_0: the nibble bytes 4t..4t+3,
// low nibbles = elements 4t.., high nibbles = 16+4t..  A stage row starts
// on a 16-byte boundary, so the quants of even blocks start 2 bytes off a
// 4-byte boundary: those read the aligned words around them and permute.
template <int QT, int B>
__device__ __forceinline__ void a_words(const uint8_t* blk, int t, uint32_t& lo, uint32_t& hi) {
    if (QT == 8) {
        if (B & 1) {
            lo = *reinterpret_cast<const uint32_t*>(blk + 2 + 8 * t);
            hi = *reinterpret_cast<const uint32_t*>(blk + 6 + 8 * t);
        } else {
            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 8 * t);
            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(blk + 4 + 8 * t);
            const uint32_t w2 = *reinterpret_cast<const uint32_t*>(blk + 8 + 8 * t);
            lo = __byte_perm(w0, w1, 0x5432);
            hi = __byte_perm(w1, w2, 0x5432);
        }
    } else {
        uint32_t w;
        if (B & 1) {
            w = *reinterpret_cast<const uint32_t*>(blk + 2 + 4 * t);
        } else {
            const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 4 * t);
            const uint32_t w1 = *reinterpret_cast<const uint32_t*>(blk + 4 + 4 * t);
            w = __byte_perm(w0, w1, 0x5432);
        }
        lo = w & 0x0F0F0F0Fu;
        hi = (w >> 4) & 0x0F0F0F0Fu;
    }
}

// The sequence of (unit, chunk) items of one warp: units u = first,
// first + stride, ... in slice-major order (u = slice * ntiles + tile), the
// chunks of the unit's slice in order.
struct MvbIter {
    int u, tile, slice, c, c1;
    __device__ __forceinline__ void enter(int total, int ntiles, int nch, int ks) {
        if (u >= total) return;
        slice = u / ntiles;
        tile = u - slice * ntiles;
        c = (int)((long long)slice * nch / ks);
        c1 = (int)((long long)(slice + 1) * nch / ks);
    }
    __device__ __forceinline__ void next(int stride, int total, int ntiles, int nch, int ks) {
        if (++c < c1) return;
        u += stride;
        enter(total, ntiles, nch, ks);
    }
};

// Output of one lane for one column tile: rows g, g + 8 of the tile,
// vectors 2t, 2t + 1 of the column tile.
__device__ __forceinline__ void mvb_store(float* y, int rows, int nvec, int r0, int v0, float a, float b, float c,
                                          float d) {
    const int r1 = r0 + 8, v1 = v0 + 1;
    if (r0 < rows) {
        if (v0 < nvec) y[(size_t)v0 * rows + r0] = a;
        if (v1 < nvec) y[(size_t)v1 * rows + r0] = b;
    }
    if (r1 < rows) {
        if (v0 < nvec) y[(size_t)v0 * rows + r1] = c;
        if (v1 < nvec) y[(size_t)v1 * rows + r1] = d;
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// The matrix: raw GGUF rows (w, row bytes rb), or (TILED) the decode
// kernel's tiled layout -- quants at w, scales at ws, nb blocks per row --
// of which this call reads the `rows` rows from tile tile0 on.
struct MvbMat {
    const uint8_t* w;
    const uint8_t* ws;
    int rows, rb, nb, tile0;
};

template <int QT, int NT, bool TILED>
__global__ void __launch_bounds__(kMvbThreads, 1)
    mvb_kernel(const MvbMat mat, int nch, int ntiles, int ks,
               const uint8_t* __restrict__ planes, const float* __restrict__ xsc, const uint32_t* __restrict__ xst,
               float* __restrict__ y, int nvec, float* __restrict__ part, int* __restrict__ cnt) {
    const uint8_t* __restrict__ w = mat.w;
    const int rows = mat.rows, rb = mat.rb, nb = mat.nb;
    using G = MvbGeom<QT>;
    constexpr int NV = NT * kMvbVec;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* stage0 = smem + (size_t)warp * G::stages * G::tile;
    const uint32_t stage0_s = smem_u32(stage0);
    const int stride = gridDim.x * kMvbWarps;
    const int total = ntiles * ks;
    const int rows_pad = ntiles * 16;

    MvbIter pf, cs;
    pf.u = blockIdx.x * kMvbWarps + warp;
    pf.tile = pf.slice = pf.c = pf.c1 = 0;
    pf.enter(total, ntiles, nch, ks);
    cs = pf;

    // 16-byte copies of one stage.  Raw: 16 rows x G::rc / 16 pieces (rows
    // past the end repeat the last row; their outputs are dropped).  Tiled:
    // the chunk's units (nblk x 16 x qb bytes) and scales (nblk x 32 bytes),
    // each one contiguous range.
    constexpr int kPieces = G::rc / 16;
    auto issue = [&](const MvbIter& it, int st) {
        if (it.u < total) {
            const uint32_t dst0 = stage0_s + (uint32_t)(st * G::tile);
            if (TILED) {
                const int kb0 = it.c * kMvbKc, nblk = min(kMvbKc, nb - kb0);
                const size_t unit0 = (size_t)(mat.tile0 + it.tile) * nb + kb0;
                const uint8_t* qsrc = w + unit0 * 16 * G::qb;
                const uint8_t* ssrc = mat.ws + unit0 * 32;
                for (int j = lane; j < nblk * G::qb; j += 32) cp_async16(dst0 + (uint32_t)(j * 16), qsrc + (size_t)j * 16);
                for (int j = lane; j < nblk * 2; j += 32)
                    cp_async16(dst0 + (uint32_t)(G::tsc + j * 16), ssrc + (size_t)j * 16);
            } else {
                const size_t coff = (size_t)it.c * G::rc;
                for (int j = lane; j < 16 * kPieces; j += 32) {
                    const int row = j / kPieces, piece = j - row * kPieces;
                    const int r = min(it.tile * 16 + row, rows - 1);
                    cp_async16(dst0 + (uint32_t)(row * G::rc + piece * 16), w + (size_t)r * rb + coff + piece * 16);
                }
            }
        }
        cp_async_commit();
    };
    // tiled Q8_0: this lane's ldmatrix row address in a unit (rows with bit 2
    // set hold their 16-byte halves swapped); Q4_0: rows 0..15, one 16-byte row each
    uint32_t lo8;
    {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8, half = (lane >> 4) & 1;
        lo8 = (uint32_t)(row * 32 + ((half ^ ((row >> 2) & 1)) << 4));
    }
    const uint32_t lo4 = (uint32_t)((lane & 15) * 16);

#pragma unroll
    for (int i = 0; i < G::stages - 1; i++) {
        issue(pf, i);
        pf.next(stride, total, ntiles, nch, ks);
    }

    const unsigned long long mneg = f2_pack(-kMvbMagicF, -kMvbMagicF);
    const unsigned long long c7 = f2_pack(0.0078125f, 0.0078125f);
    const unsigned long long c14 = f2_pack(6.103515625e-05f, 6.103515625e-05f);
    unsigned long long acc_g[NT], acc_h[NT];
#pragma unroll
    for (int n = 0; n < NT; n++) acc_g[n] = acc_h[n] = f2_pack(0.0f, 0.0f);
    int st = 0;
#pragma unroll 1
    while (cs.u < total) {
        issue(pf, st == 0 ? G::stages - 1 : st - 1);
        pf.next(stride, total, ntiles, nch, ks);
        cp_async_wait<G::stages - 1>();
        __syncwarp();

        const uint8_t* rg = stage0 + st * G::tile + g * G::rc;
        const uint8_t* rh = rg + 8 * G::rc;
        const uint32_t sq = stage0_s + (uint32_t)(st * G::tile);
        const uint8_t* ssc = stage0 + st * G::tile + G::tsc;
        const int kb0 = cs.c * kMvbKc;
        const int nblk = TILED ? min(kMvbKc, nb - kb0) : kMvbKc;
        // one 32-block of the chunk: A fragments, scales, the NT x 3 mma and
        // their fp32 accumulation
        auto block = [&](const int bb) {
            const int kb = kb0 + bb;
            uint32_t a0, a1, a2, a3;
            float dg, dh;
            if (TILED) {
                if (QT == 8) {
                    ldsm_x4(sq + (uint32_t)(bb * 16 * G::qb) + lo8, a0, a1, a2, a3);
                } else {
                    uint32_t w0, w1;
                    ldsm_x2(sq + (uint32_t)(bb * 16 * G::qb) + lo4, w0, w1);
                    a0 = w0 & 0x0F0F0F0Fu;         // row g, elements 4t.. (low nibbles)
                    a1 = w1 & 0x0F0F0F0Fu;         // row g + 8
                    a2 = (w0 >> 4) & 0x0F0F0F0Fu;  // row g, elements 16+4t.. (high nibbles)
                    a3 = (w1 >> 4) & 0x0F0F0F0Fu;
                }
                // scales of rows g and g + 8: one word (order 0, 8, 1, 9, ...)
                const float2 d2 = __half22float2(*reinterpret_cast<const __half2*>(ssc + bb * 32 + 4 * g));
                dg = d2.x;
                dh = d2.y;
            } else {
                const uint8_t* bg = rg + bb * G::bpb;
                const uint8_t* bh = rh + bb * G::bpb;
                switch (bb) {  // bb is a constant after unrolling: the parity picks the load pattern
                    case 0: a_words<QT, 0>(bg, t, a0, a2); a_words<QT, 0>(bh, t, a1, a3); break;
                    case 1: a_words<QT, 1>(bg, t, a0, a2); a_words<QT, 1>(bh, t, a1, a3); break;
                    case 2: a_words<QT, 2>(bg, t, a0, a2); a_words<QT, 2>(bh, t, a1, a3); break;
                    case 3: a_words<QT, 3>(bg, t, a0, a2); a_words<QT, 3>(bh, t, a1, a3); break;
                    case 4: a_words<QT, 4>(bg, t, a0, a2); a_words<QT, 4>(bh, t, a1, a3); break;
                    case 5: a_words<QT, 5>(bg, t, a0, a2); a_words<QT, 5>(bh, t, a1, a3); break;
                    case 6: a_words<QT, 6>(bg, t, a0, a2); a_words<QT, 6>(bh, t, a1, a3); break;
                    default: a_words<QT, 7>(bg, t, a0, a2); a_words<QT, 7>(bh, t, a1, a3); break;
                }
                dg = __half2float(*reinterpret_cast<const __half*>(bg));
                dh = __half2float(*reinterpret_cast<const __half*>(bh));
            }
            const unsigned long long dgp = f2_pack(dg, dg), dhp = f2_pack(dh, dh);
#pragma unroll
            for (int n = 0; n < NT; n++) {
                const int gi = kb * NT + n;
                const uint2* rec = reinterpret_cast<const uint2*>(planes + (size_t)gi * 3 * 256) + lane;
                const uint2 p0 = __ldg(rec), p1 = __ldg(rec + 32), p2 = __ldg(rec + 64);
                const float2 sx = __ldg(reinterpret_cast<const float2*>(xsc + gi * kMvbVec + 2 * t));
                uint32_t s0a = kMvbMagic, s0b = kMvbMagic, s1a = kMvbMagic, s1b = kMvbMagic, s2a = kMvbMagic,
                         s2b = kMvbMagic;
                if (QT != 8) {
                    const uint2* sp = reinterpret_cast<const uint2*>(xst + (size_t)gi * 3 * kMvbVec + 2 * t);
                    const uint2 v0 = __ldg(sp), v1 = __ldg(sp + 4), v2 = __ldg(sp + 8);
                    s0a = v0.x; s0b = v0.y; s1a = v1.x; s1b = v1.y; s2a = v2.x; s2b = v2.y;
                }
                uint32_t e0, e1, e2, e3, f0, f1, f2, f3, h0, h1, h2, h3;
                mma_i8<QT != 8>(a0, a1, a2, a3, p0.x, p0.y, s0a, s0b, e0, e1, e2, e3);
                mma_i8<QT != 8>(a0, a1, a2, a3, p1.x, p1.y, s1a, s1b, f0, f1, f2, f3);
                mma_i8<QT != 8>(a0, a1, a2, a3, p2.x, p2.y, s2a, s2b, h0, h1, h2, h3);
                const unsigned long long sxp = f2_pack(sx.x, sx.y);
                // rows g (d0, d1) and g + 8 (d2, d3), vectors 2t and 2t + 1 of column tile n
                unsigned long long tg = f2_add(f2_pack(__uint_as_float(e0), __uint_as_float(e1)), mneg);
                tg = f2_fma(f2_add(f2_pack(__uint_as_float(f0), __uint_as_float(f1)), mneg), c7, tg);
                tg = f2_fma(f2_add(f2_pack(__uint_as_float(h0), __uint_as_float(h1)), mneg), c14, tg);
                unsigned long long th = f2_add(f2_pack(__uint_as_float(e2), __uint_as_float(e3)), mneg);
                th = f2_fma(f2_add(f2_pack(__uint_as_float(f2), __uint_as_float(f3)), mneg), c7, th);
                th = f2_fma(f2_add(f2_pack(__uint_as_float(h2), __uint_as_float(h3)), mneg), c14, th);
                acc_g[n] = f2_fma(f2_mul(dgp, sxp), tg, acc_g[n]);
                acc_h[n] = f2_fma(f2_mul(dhp, sxp), th, acc_h[n]);
            }
        };
        if (nblk == kMvbKc) {
            // a full chunk: unrolled, so the loads of later blocks issue early
#pragma unroll
            for (int bb = 0; bb < kMvbKc; bb++) block(bb);
        } else {
#pragma unroll 1
            for (int bb = 0; bb < nblk; bb++) block(bb);  // tiled layout only: a short last chunk
        }

        if (cs.c + 1 == cs.c1) {
            // unit done: rows tile*16 + g, + 8; vectors n*8 + 2t, + 1
            const int r0 = cs.tile * 16 + g, r1 = r0 + 8;
            if (ks == 1) {
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    const float2 vg = f2_unpack(acc_g[n]), vh = f2_unpack(acc_h[n]);
                    mvb_store(y, rows, nvec, r0, n * kMvbVec + 2 * t, vg.x, vg.y, vh.x, vh.y);
                }
            } else {
                float* ps = part + (size_t)cs.slice * NV * rows_pad;
#pragma unroll
                for (int n = 0; n < NT; n++) {
                    const float2 vg = f2_unpack(acc_g[n]), vh = f2_unpack(acc_h[n]);
                    const int v0 = n * kMvbVec + 2 * t, v1 = v0 + 1;
                    ps[(size_t)v0 * rows_pad + r0] = vg.x;
                    ps[(size_t)v1 * rows_pad + r0] = vg.y;
                    ps[(size_t)v0 * rows_pad + r1] = vh.x;
                    ps[(size_t)v1 * rows_pad + r1] = vh.y;
                }
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(cnt + cs.tile, 1) == ks - 1;
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        const int v0 = n * kMvbVec + 2 * t, v1 = v0 + 1;
                        float s00 = 0.0f, s01 = 0.0f, s10 = 0.0f, s11 = 0.0f;
                        for (int s = 0; s < ks; s++) {
                            const float* q = part + (size_t)s * NV * rows_pad;
                            s00 += __ldcg(q + (size_t)v0 * rows_pad + r0);
                            s01 += __ldcg(q + (size_t)v1 * rows_pad + r0);
                            s10 += __ldcg(q + (size_t)v0 * rows_pad + r1);
                            s11 += __ldcg(q + (size_t)v1 * rows_pad + r1);
                        }
                        mvb_store(y, rows, nvec, r0, v0, s00, s01, s10, s11);
                    }
                    if (lane == 0) cnt[cs.tile] = 0;  // every unit of the tile has arrived
                }
            }
#pragma unroll
            for (int n = 0; n < NT; n++) acc_g[n] = acc_h[n] = f2_pack(0.0f, 0.0f);
        }
        __syncwarp();  // every lane is done with this stage before it is refilled
        st = st + 1 == G::stages ? 0 : st + 1;
        cs.next(stride, total, ntiles, nch, ks);
    }
    cp_async_wait<0>();
}

// Scratch of the batched matvec, one per (device, stream): the per-tile
// arrival counters (zero between calls: the last unit of a tile resets its
// counter), the x planes, their scales and Q4_0 accumulator starts, the slice
// partials.  Calls on one stream run in order, so they never share it while
// it is in use; calls on different streams (two models, or two batches of
// one model on different threads) each get their own.
struct MvbScratch {
    uint8_t* buf = nullptr;
    size_t bytes = 0;
    unsigned long long gen = 0;  // bumped whenever buf moves (CUDA graphs hold its address)
    int sms = 0;
    bool attr_set = false;
};
std::mutex g_mvb_mu;
std::map<std::pair<int, cudaStream_t>, MvbScratch> g_mvb;

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

template <int QT, bool TILED>
cudaError_t set_smem_attrs() {
    using G = MvbGeom<QT>;
    cudaError_t e = cudaFuncSetAttribute(mvb_kernel<QT, 1, TILED>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(mvb_kernel<QT, 2, TILED>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::smem);
    // the rest of the 256 KB stays L1 for the x planes (read through the
    // texture path).  Only a hint: a refusal is cleared so that the launch
    // check does not report it.
    if (cudaFuncSetAttribute(mvb_kernel<QT, 1, TILED>, cudaFuncAttributePreferredSharedMemoryCarveout, 0) != cudaSuccess)
        (void)cudaGetLastError();
    if (cudaFuncSetAttribute(mvb_kernel<QT, 2, TILED>, cudaFuncAttributePreferredSharedMemoryCarveout, 0) != cudaSuccess)
        (void)cudaGetLastError();
    return e;
}

template <int QT, bool TILED>
void launch_mvb(int nt, int grid, cudaStream_t s, const MvbMat& mat, int nch, int ntiles, int ks,
                const uint8_t* planes, const float* xsc, const uint32_t* xst, float* y, int nvec, float* part,
                int* cnt) {
    using G = MvbGeom<QT>;
    if (nt == 1)
        mvb_kernel<QT, 1, TILED><<<grid, kMvbThreads, G::smem, s>>>(mat, nch, ntiles, ks, planes, xsc, xst, y, nvec,
                                                                    part, cnt);
    else
        mvb_kernel<QT, 2, TILED><<<grid, kMvbThreads, G::smem, s>>>(mat, nch, ntiles, ks, planes, xsc, xst, y, nvec,
                                                                    part, cnt);
}

// Both layouts: plane split of x, then the tile dots.  nb = 32-blocks per row.
int mvb_run(bool q8, bool tiled, const MvbMat& mat, const float* x, float* y, int nvec, cudaStream_t s,
            std::string* err) {
    const int nbk = mat.nb;
    const int nch = (nbk + kMvbKc - 1) / kMvbKc;
    const int ntiles = (mat.rows + 15) / 16;
    const int nt = (nvec + kMvbVec - 1) / kMvbVec;  // column tiles: 1 or 2
    const int cols = nbk * 32;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *err = "no CUDA device";
        return B2_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lk(g_mvb_mu);
    MvbScratch* sc = &g_mvb[{dev, s}];
    if (!sc->sms && cudaDeviceGetAttribute(&sc->sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        *err = "cudaDeviceGetAttribute failed";
        return B2_ERR_CUDA;
    }
    if (!sc->attr_set) {
        const cudaError_t es[4] = {set_smem_attrs<8, false>(), set_smem_attrs<2, false>(), set_smem_attrs<8, true>(),
                                   set_smem_attrs<2, true>()};
        for (cudaError_t e : es) {
            if (e != cudaSuccess) {
                *err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
                return B2_ERR_CUDA;
            }
        }
        sc->attr_set = true;
    }
    // slices: the fewest (up to 8, at most one per chunk) giving every
    // warp of the grid two units
    const int warps = sc->sms * kMvbWarps;
    int ks = 1;
    while (ks < kMvbMaxSlices && ks < nch && (long long)ntiles * ks < 2LL * warps) ks++;
    // Arrival counters first: ks > 1 only when ntiles * (ks - 1) < 2 * warps,
    // so 2 * warps counters cover every split call.  They are zeroed when
    // the buffer is allocated and each split call leaves them zero.
    const size_t b_cnt = align256((size_t)2 * warps * 4);
    const size_t ng = (size_t)nbk * nt;  // plane record groups
    const size_t b_planes = align256(ng * 3 * 256);
    const size_t b_xsc = align256(ng * kMvbVec * 4);
    const size_t b_xst = align256(ng * 3 * kMvbVec * 4);
    const size_t b_part = ks > 1 ? align256((size_t)ks * nt * kMvbVec * ntiles * 16 * 4) : 0;
    const size_t need = b_cnt + b_planes + b_xsc + b_xst + b_part;
    if (sc->bytes < need) {
        if (sc->buf) cudaFree(sc->buf);
        sc->buf = nullptr;
        sc->bytes = 0;
        if (cudaMalloc(&sc->buf, need) != cudaSuccess) {
            *err = "scratch allocation failed";
            return B2_ERR_OOM;
        }
        if (cudaMemsetAsync(sc->buf, 0, b_cnt, s) != cudaSuccess) {
            *err = "scratch clear failed";
            return B2_ERR_CUDA;
        }
        sc->bytes = need;
        sc->gen++;
    }
    uint8_t* base = sc->buf;
    int* cnt = reinterpret_cast<int*>(base);
    uint8_t* planes = base + b_cnt;
    float* xsc = reinterpret_cast<float*>(planes + b_planes);
    uint32_t* xst = reinterpret_cast<uint32_t*>(planes + b_planes + b_xsc);
    float* part = ks > 1 ? reinterpret_cast<float*>(planes + b_planes + b_xsc + b_xst) : nullptr;
    const int units = ntiles * ks;
    const int grid = std::min(sc->sms, (units + kMvbWarps - 1) / kMvbWarps);
    const int ngrid = (int)ng;
    // plane order: raw Q8_0 rows take the permuted order, everything else the natural one
    if (q8 && !tiled)
        mvb_planes_kernel<true, false><<<ngrid, kMvbThreads, 0, s>>>(x, nvec, cols, nt, planes, xsc, xst);
    else if (q8)
        mvb_planes_kernel<false, false><<<ngrid, kMvbThreads, 0, s>>>(x, nvec, cols, nt, planes, xsc, xst);
    else
        mvb_planes_kernel<false, true><<<ngrid, kMvbThreads, 0, s>>>(x, nvec, cols, nt, planes, xsc, xst);
    if (q8 && tiled) launch_mvb<8, true>(nt, grid, s, mat, nch, ntiles, ks, planes, xsc, xst, y, nvec, part, cnt);
    else if (q8) launch_mvb<8, false>(nt, grid, s, mat, nch, ntiles, ks, planes, xsc, xst, y, nvec, part, cnt);
    else if (tiled) launch_mvb<2, true>(nt, grid, s, mat, nch, ntiles, ks, planes, xsc, xst, y, nvec, part, cnt);
    else launch_mvb<2, false>(nt, grid, s, mat, nch, ntiles, ks, planes, xsc, xst, y, nvec, part, cnt);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *err = std::string("batched matvec launch: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

}  // namespace
}  // namespace b2

using namespace b2;

int b2_matvec_batch_impl(int qtype, const void* w, const float* x, float* y, int rows, int cols, int nvec,
                         cudaStream_t s, std::string* err) {
    if (reinterpret_cast<uintptr_t>(w) & 15) {
        *err = "weight pointer must be 16-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    if (reinterpret_cast<uintptr_t>(x) & 3 || reinterpret_cast<uintptr_t>(y) & 3) {
        *err = "x and y must be 4-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    if (nvec < 1 || nvec > kMvbMaxNt * kMvbVec || cols % (32 * kMvbKc)) {
        *err = "batched matvec takes 1 to 16 vectors and cols a multiple of 256";
        return B2_ERR_BAD_ARG;
    }
    const bool q8 = qtype == 8;
    const int nbk = cols / 32;
    const MvbMat mat{static_cast<const uint8_t*>(w), nullptr, rows, nbk * (q8 ? 34 : 18), nbk, 0};
    return mvb_run(q8, false, mat, x, y, nvec, s, err);
}

// The same dots over a matrix resident in the decode kernel's tiled layout
// (base = the tiled matrix, rp = its padded row count): rows [row0, row0 +
// rows) of it, row0 a multiple of 16.
int b2_tiled_matvec_batch_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols,
                               const float* x, float* y, int nvec, cudaStream_t s, std::string* err) {
    if (reinterpret_cast<uintptr_t>(x) & 3 || reinterpret_cast<uintptr_t>(y) & 3) {
        *err = "x and y must be 4-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    if (nvec < 1 || nvec > kMvbMaxNt * kMvbVec || cols % 32 || cols <= 0 || rows <= 0) {
        *err = "batched matvec takes 1 to 16 vectors and cols a multiple of 32";
        return B2_ERR_BAD_ARG;
    }
    if (row0 % 16 || row0 + rows > rp) {
        *err = "tensor does not start on a 16-row tile of its matrix";
        return B2_ERR_BAD_ARG;
    }
    const bool q8 = qtype == 8;
    const int nbk = cols / 32;
    const uint8_t* w = static_cast<const uint8_t*>(base);
    const MvbMat mat{w, w + (size_t)rp * nbk * (q8 ? 32 : 16), rows, 0, nbk, (int)(row0 / 16)};
    return mvb_run(q8, true, mat, x, y, nvec, s, err);
}

// Generation of the scratch buffer of stream s on the current device: a CUDA
// graph that captured batched matvecs on s is valid while this is unchanged.
// Frees the batched matvec's scratch of stream s on device dev (a stream
// about to be destroyed; nothing of it may still run).
void b2_mvb_release(int dev, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_mvb_mu);
    const auto it = g_mvb.find({dev, s});
    if (it != g_mvb.end()) {
        if (it->second.buf) cudaFree(it->second.buf);
        g_mvb.erase(it);
    }
}

unsigned long long b2_mvb_scratch_generation(cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_mvb_mu);
    const auto it = g_mvb.find({dev, s});
    return it == g_mvb.end() ? 0 : it->second.gen;
}
