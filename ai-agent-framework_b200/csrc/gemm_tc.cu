// Tensor-core GEMM over the resident quantised weights (Blackwell tcgen05).
//
// Y[t][r] = sum_k X[t][k] W[r][k] for many tokens t at once: the prefill of
// a prompt (the forward of transformer.go:519-739 with seqLen > 1, the
// batched form of the C++ sibling's Transformer::forward_batch,
// Local-LLM/src/transformer.cpp:540-575, whose mat_mat_mul_tensor
// Local-LLM/include/tensor.h:354-387 dequantises and multiplies) and the
// batched decode steps.  W stays in the decode kernel's tiled Q8_0 / Q4_0
// layout (dev.cuh); nothing is dequantised in HBM.
//
// One CTA computes a 128-row x BN-token tile of Y over its K range (BN 16,
// 32, 64, 128 or 256: the token count rounded up):
//   warp 0      producer: TMA tensor loads (cp.async.bulk.tensor.2d, this
//               GPU's own memory, no multicast) of each K stage's raw quant
//               and scale blocks of the 128 weight rows and of the BN x 64
//               fp16 activation tile (128-byte swizzle) into a ring of raw
//               stages as deep as shared memory allows; the first ring's
//               weights before the wait on the previous kernel (the launch
//               is a programmatic dependent launch), the activations after;
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16 (M 128,
//               N BN, K 16) four times per stage, A from tensor memory, B
//               (the activation tile) from shared memory by descriptor, the
//               fp32 accumulator in tensor memory (BN columns);
//               tcgen05.commit frees the A stage and the raw stage;
//   warps 2..9  dequantisers, two per tensor-memory lane quadrant (one Q
//               block of the stage each): thread (lane) r decodes its weight
//               row (f16 scale x int8 or nibble - 8, rounded once to fp16)
//               and stores it with tcgen05.st into its lane of a 4-deep ring
//               of A stages in tensor memory (the dequantised tile never
//               touches shared memory); then the epilogue: tcgen05.ld of its
//               accumulator row, times the token's activation scale, to Y
//               (coalesced over rows).
// Activations arrive in fp16 with a power-of-two scale per token (its
// largest magnitude maps into [2^14, 2^15); converted by the call, or by the
// kernel before it), so they keep 11 significant bits without overflow;
// products accumulate in fp32.  The
// weight d * q is rounded to fp16 once (at most 2^-12 relative error per
// weight).  Every wait is bounded (globaltimer) and reports B2_ERR_TIMEOUT
// through the device error flag; a CTA that gave up stops issuing work,
// waits (bounded) for the copies and products it issued and frees its
// tensor memory before it exits.
//
// When the row tiles are fewer than the SMs, the K range is split over up to
// kMaxKSplit CTAs per tile; their partial sums go to a scratch buffer and one
// more kernel adds them in split order (results do not depend on timing).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "gemm.h"

namespace b2 {
namespace {

constexpr int kDqWarps = 8;             // dequantising / epilogue warps: two per TMEM lane quadrant
constexpr int kGemmThreads = 64 + 32 * kDqWarps;  // + producer warp, MMA warp
constexpr int kBM = 128;                // weight rows per CTA (MMA M)
constexpr int kStageBlocks = 2;         // Q blocks (of 32) per K stage: 64 elements
constexpr int kMaxKSplit = 8;
constexpr uint64_t kGemmWaitNs = 2000000000ull;
constexpr int kGemmSmemMax = 232448;

template <int QT>
struct QShape {
    static constexpr int QB = QT == 8 ? 32 : 16;                       // quant bytes per row and block
    static constexpr int kRawQ = kBM / kTileRows * kStageBlocks * kTileRows * QB;  // quants of a stage
    static constexpr int kRawS = kBM / kTileRows * kStageBlocks * kTileRows * 2;   // scales of a stage
};

// Shared-memory plan of one CTA (byte offsets from a 1024-aligned base): a
// deep ring of raw stages (the activation tile and the raw quant and scale
// blocks of one K stage, filled by TMA) and a double-buffered dequantised A
// tile.  The raw stages are what is in flight from HBM, so that ring is as
// deep as shared memory allows.  The dequantised A tiles (16 KB of fp16 a
// stage, four times the Q4_0 bytes they come from) never touch shared
// memory: the dequantising warps store them into tensor memory, where the
// MMA reads its A operand, in a ring four deep so they run ahead of the
// MMA's round trip (issue, completion, commit).
template <int QT, int BN>
struct GemmSmem {
    static constexpr int kA = kBM * 128;  // fp16, 128 rows x 64 K, 128-byte swizzle
    static constexpr int kB = BN * 128;   // fp16, BN rows x 64 K
    // raw slot [B | raw q | raw s], a multiple of 1024 so each B tile stays 1024-aligned
    static constexpr int kSlot = (kB + QShape<QT>::kRawQ + QShape<QT>::kRawS + 1023) & ~1023;
    static constexpr int kAStages = 4;
    static constexpr int kFixed = 2048;  // alignment slack, then barriers and the TMEM slot
    // the decode-step forms (BN <= 32) run two CTAs per SM, so twice the
    // warps decode weights; the prefill forms one CTA
    static constexpr int kCtas = BN <= 32 ? 2 : 1;
    // per CTA: the opt-in maximum, or an equal share of the SM's 228 KB less
    // the 1 KB the hardware reserves per resident CTA
    static constexpr int kBudget = kCtas == 1 ? kGemmSmemMax : 233472 / kCtas - 1024;
    static constexpr int kFit = (kBudget - kFixed) / kSlot;
    static constexpr int kStages = kFit > 24 ? 24 : kFit;  // raw stages
    static_assert(kStages >= 2, "two raw stages must fit");
    static constexpr int kTotal = kFixed + kStages * kSlot;
    // tensor memory: the accumulator (BN columns, at least 32), then the A
    // ring (32 columns a stage: 128 lanes x 64 fp16); 256 columns in all, so
    // two CTAs of an SM fit its 512
    static constexpr uint32_t kAccCols = BN < 32 ? 32 : BN;
    static constexpr uint32_t kTmemCols = BN <= 128 ? 256 : 512;
    static_assert(kAccCols + 32 * kAStages <= kTmemCols && kCtas * kTmemCols <= 512, "tensor memory plan");
};

struct GemmArgs {
    int nst;            // K stages per CTA (kStageBlocks blocks each)
    int kst_split;      // stages per split (the last split may take fewer)
    int ksplit;         // splits of K (gridDim.z)
    int tiles_q;        // first 16-row Q tile of the matrix share (row0 / 16)
    int rows;           // output rows (weight rows) of the share
    int ntok;           // tokens (valid columns of X)
    int ldy;            // row stride of Y (floats)
    float* y;           // [ntok][ldy]
    float* part;        // split partials [split][ntok][rows] (ksplit > 1)
    const float* tok_scale;  // [ntok_pad] activation scale per token
    int* err;
};

__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kGemmWaitNs) {
            atomicCAS(err, 0, B2_ERR_TIMEOUT);
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (sm_100 shared
// memory descriptor: start >> 4 in bits 0-13, leading offset (unused with
// this swizzle) 16-29, stride offset >> 4 in 32-45, version 1 in 46-47,
// layout type 2 = 128-byte swizzle in 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), A
// and B fp16 (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 in
// bits 17-22, M >> 4 in bits 24-28.
template <int BN>
__device__ __forceinline__ uint32_t f16_idesc() {
    return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// A from tensor memory (M = 128 lanes, K = 16: 8 columns), B from shared memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 4 signed bytes -> 2 half2 of the exact integers: (b ^ 0x80) in the low
// byte of the fp16 0x6400 (1024) is 1024 + b + 128.
__device__ __forceinline__ void s8x4_to_h2(uint32_t w, __half2& lo, __half2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x5140), b = __byte_perm(u, 0x64646464u, 0x7362);
    const __half2 off = __floats2half2_rn(1152.0f, 1152.0f);
    lo = __hsub2(*reinterpret_cast<const __half2*>(&a), off);
    hi = __hsub2(*reinterpret_cast<const __half2*>(&b), off);
}
// 4 nibbles (one per byte, 0..15) -> 2 half2 of nibble - 8.
__device__ __forceinline__ void u4x4_to_h2(uint32_t w, __half2& lo, __half2& hi) {
    const uint32_t a = __byte_perm(w, 0x64646464u, 0x5140), b = __byte_perm(w, 0x64646464u, 0x7362);
    const __half2 off = __floats2half2_rn(1032.0f, 1032.0f);
    lo = __hsub2(*reinterpret_cast<const __half2*>(&a), off);
    hi = __hsub2(*reinterpret_cast<const __half2*>(&b), off);
}

// 16 consecutive 32-bit tensor-memory columns of this thread's lane (one
// lane per thread of the warp, the warp's 32-lane quadrant in taddr).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Row r (0..127) of a stage: Q blocks kb0 .. kb0 + NKB - 1 of its two -> 32
// fp16 (d * q) each, written to the row's tensor-memory lane as the A operand
// of the MMA: element k of the stage in column k / 2 (low half for even k)
// from the stage's first column a_col.
template <int QT, int NKB>
__device__ __forceinline__ void dequant_row(const uint8_t* rawq, const uint8_t* raws, uint32_t a_col, int r, int kb0) {
    constexpr int QB = QShape<QT>::QB;
    const int t = r >> 4, rr = r & 15;
#pragma unroll
    for (int kk = 0; kk < NKB; kk++) {
        const int kb = kb0 + kk;
        // TMA box layout: [tile][block][16 rows][QB]; scales [tile][block][16] in (g, g + 8) order
        const uint8_t* q = rawq + ((t * kStageBlocks + kb) * kTileRows + rr) * QB;
        const uint16_t dbits =
            *reinterpret_cast<const uint16_t*>(raws + ((t * kStageBlocks + kb) * kTileRows + 2 * (rr & 7) + (rr >> 3)) * 2);
        const __half2 d2 = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
        uint32_t w[8], out[16];
        if (QT == 8) {
            // rows with bit 2 set hold their two 16-byte halves swapped
            const uint4 h0 = *reinterpret_cast<const uint4*>(q + ((rr & 4) ? 16 : 0));
            const uint4 h1 = *reinterpret_cast<const uint4*>(q + ((rr & 4) ? 0 : 16));
            w[0] = h0.x; w[1] = h0.y; w[2] = h0.z; w[3] = h0.w;
            w[4] = h1.x; w[5] = h1.y; w[6] = h1.z; w[7] = h1.w;
        } else {
            // byte i: low nibble = element i, high nibble = element i + 16
            const uint4 h = *reinterpret_cast<const uint4*>(q);
            w[0] = h.x & 0x0F0F0F0Fu; w[1] = h.y & 0x0F0F0F0Fu; w[2] = h.z & 0x0F0F0F0Fu; w[3] = h.w & 0x0F0F0F0Fu;
            w[4] = (h.x >> 4) & 0x0F0F0F0Fu; w[5] = (h.y >> 4) & 0x0F0F0F0Fu;
            w[6] = (h.z >> 4) & 0x0F0F0F0Fu; w[7] = (h.w >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int c = 0; c < 4; c++) {  // chunk c of this block: elements 8c .. 8c + 7
            __half2 h[4];
            if (QT == 8) {
                s8x4_to_h2(w[2 * c], h[0], h[1]);
                s8x4_to_h2(w[2 * c + 1], h[2], h[3]);
            } else {
                u4x4_to_h2(w[2 * c], h[0], h[1]);
                u4x4_to_h2(w[2 * c + 1], h[2], h[3]);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                h[i] = __hmul2(h[i], d2);
                out[4 * c + i] = *reinterpret_cast<const uint32_t*>(&h[i]);
            }
        }
        tmem_st16(a_col + (uint32_t)(16 * kb), out);  // block kb: columns 16 kb .. 16 kb + 15
    }
}

template <int QT, int BN>
__global__ void __launch_bounds__(kGemmThreads, GemmSmem<QT, BN>::kCtas)
    qgemm_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_s,
                 const __grid_constant__ CUtensorMap map_x, const GemmArgs a) {
    using SM = GemmSmem<QT, BN>;
    constexpr int NS = SM::kStages;
    extern __shared__ __align__(1024) uint8_t gsm_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    constexpr int NA = SM::kAStages;
    uint8_t* rawr = base + 1024;  // [NS][B | raw q | raw s]
    uint64_t* full = reinterpret_cast<uint64_t*>(base);  // raw stage landed (TMA)
    uint64_t* rempty = full + NS;                        // raw stage free (MMA done with its B)
    uint64_t* afull = rempty + NS;                       // [NA] A tile decoded
    uint64_t* aempty = afull + NA;                       // [NA] A tile free (MMA done)
    uint64_t* accum = aempty + NA;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, nt = blockIdx.y, ks = blockIdx.z;
    const int st0 = ks * a.kst_split;
    const int nst = max(0, min(a.kst_split, a.nst - st0));
    constexpr uint32_t kTmemCols = SM::kTmemCols;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&rempty[s], 1);
        }
        for (int j = 0; j < NA; j++) {
            mbar_init(&afull[j], kDqWarps);
            mbar_init(&aempty[j], 1);
        }
        mbar_init(accum, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // The kernel after this one may launch now.  Only after the tensor
    // memory is held: a dependent GEMM's CTA placed on this SM early must
    // not take the columns a CTA of this grid still waits to allocate.
    pdl_trigger();

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            const uint32_t bytes = QShape<QT>::kRawQ + QShape<QT>::kRawS + SM::kB;
            auto load_w = [&](int it) {  // the stage's weight blocks and scales
                const int s = it % NS, kb = (st0 + it) * kStageBlocks;  // first Q block of the stage
                uint8_t* st = rawr + (size_t)s * SM::kSlot;
                mbar_arrive_expect_tx(&full[s], bytes);
                tma_load_2d(st + SM::kB, &map_q, kb * (kTileRows * QShape<QT>::QB / 8),
                            a.tiles_q + mt * (kBM / kTileRows), &full[s]);
                tma_load_2d(st + SM::kB + QShape<QT>::kRawQ, &map_s, kb * (kTileRows * 2 / 8),
                            a.tiles_q + mt * (kBM / kTileRows), &full[s]);
            };
            auto load_x = [&](int it) {  // the stage's activation tile
                const int s = it % NS, kb = (st0 + it) * kStageBlocks;
                tma_load_2d(rawr + (size_t)s * SM::kSlot, &map_x, kb * 32, nt * BN, &full[s]);
            };
            // The weights depend on nothing a previous kernel writes: the first
            // ring's worth streams before the wait on the kernel this launch
            // follows (a programmatic dependent launch overlaps its tail);
            // the activations, and everything after them, come after it.
            const int pre = min(nst, NS);
            for (int it = 0; it < pre; it++) load_w(it);
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int it = 0; it < pre; it++) load_x(it);
            int issued = pre;
            for (int it = pre; it < nst; it++) {
                if (!gemm_wait(&rempty[it % NS], ((it / NS) - 1) & 1, a.err, abort_flag)) break;
                load_w(it);
                load_x(it);
                issued = it + 1;
            }
            // every copy issued has landed before the CTA may exit
            for (int it = max(0, issued - NS); it < issued; it++)
                if (!gemm_wait(&full[it % NS], (it / NS) & 1, a.err, abort_flag)) {
                    // (already aborted: give the copies a bounded time of their own)
                    const uint64_t t0 = global_ns();
                    while (!mbar_try_wait(&full[it % NS], (it / NS) & 1) && global_ns() - t0 < kGemmWaitNs) {
                    }
                }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------------- MMA
        if (lane == 0) {
            const uint32_t idesc = f16_idesc<BN>();
            int done = 0;
            for (int it = 0; it < nst; it++) {
                const int s = it % NS, j = it % NA;
                if (!gemm_wait(&afull[j], (it / NA) & 1, a.err, abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ta = tmem + SM::kAccCols + 32u * (uint32_t)j, sb = smem_u32(rawr + (size_t)s * SM::kSlot);
#pragma unroll
                for (int k = 0; k < 4; k++)  // K = 16 per MMA: 8 columns of A, 32 bytes along B's swizzled row
                    mma_f16_ts(tmem, ta + 8u * (uint32_t)k, sw128_desc(sb + 32 * k), idesc, (it | k) != 0);
                mma_commit(&aempty[j]);   // the A buffer, and
                mma_commit(&rempty[s]);   // the raw stage (its B tile) are free once these products are done
                done = it + 1;
            }
            mma_commit(accum);  // after every MMA issued above
            (void)done;
        }
    } else {
        // ---------------------------------------------- dequantisers, epilogue
        // thread: weight row r of the tile; with eight warps the two halves of
        // the row's stage (one Q block each) go to threads 128 apart
        constexpr int kRowThreads = kDqWarps * 32 / kBM;  // 1 or 2
        // (row = tensor-memory lane: a warp reaches lanes 32 (warp % 4) .. + 31)
        const int dt = threadIdx.x - 64, r = 32 * (warp & 3) + lane, kb0 = (dt / kBM) * (kStageBlocks / kRowThreads);
        for (int it = 0; it < nst; it++) {
            const int s = it % NS, j = it % NA;
            bool ok = gemm_wait(&full[s], (it / NS) & 1, a.err, abort_flag);
            if (ok && it >= NA) ok = gemm_wait(&aempty[j], ((it / NA) - 1) & 1, a.err, abort_flag);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const uint8_t* st = rawr + (size_t)s * SM::kSlot;
            // this warp's lane quadrant of A stage j
            const uint32_t ta = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + SM::kAccCols + 32u * (uint32_t)j;
            dequant_row<QT, kStageBlocks / kRowThreads>(st + SM::kB, st + SM::kB + QShape<QT>::kRawQ, ta, r, kb0);
            // raw stage s is free once every dequantising warp has read it;
            // its B tile still feeds the MMA, which releases the stage
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[j]);
        }
        // epilogue: accumulator row r (TMEM lane r; warp w reads lanes 32 (w % 4) ..);
        // the warps of one lane quadrant split the columns
        const int q = warp & 3, grp = (warp - 2) >> 2;
        constexpr int kGroups = kDqWarps / 4;
        constexpr int kColsPer = BN / kGroups < 16 ? 16 : BN / kGroups;
        const int row = 32 * q + lane;
        bool ok = gemm_wait(accum, 0, a.err, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        // one decision for all four epilogue warps (each arrives here whatever
        // its waits returned), so the barriers below are met by all or none
        volatile int* ep_ok = reinterpret_cast<volatile int*>(tmem_slot + 4);  // [kDqWarps]
        if (lane == 0) ep_ok[warp - 2] = ok ? 1 : 0;
        named_bar_sync(1, 32 * kDqWarps);
#pragma unroll
        for (int w = 0; w < kDqWarps; w++) ok = ok && ep_ok[w];
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok && nst > 0) {
            const int grow = mt * kBM + row;  // output row within the share
            const size_t plane = (size_t)a.ntok * a.rows;
            float* yb = a.ksplit > 1 ? a.part + (size_t)ks * plane : a.y;
            const int ld = a.ksplit > 1 ? a.rows : a.ldy;
#pragma unroll 1
            for (int c0 = grp * kColsPer; c0 < BN && c0 < (grp + 1) * kColsPer; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int tok = nt * BN + c0 + j;
                    if (grow < a.rows && tok < a.ntok)
                        yb[(size_t)tok * ld + grow] = __uint_as_float(v[j]) * a.tok_scale[tok];
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        // the MMAs this CTA issued are complete (accum barrier, bounded) before
        // its tensor memory goes back
        if (lane == 0) {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait(accum, 0) && global_ns() - t0 < kGemmWaitNs) {
            }
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// X fp32 [ntok][cols] -> fp16 [ntok_pad][cols] scaled by 2^e per token (the
// largest magnitude into [2^14, 2^15)), scale[t] = 2^-e; rows past ntok zero.
// One CTA of kCvtThreads per token; the row is read once (float4 loads kept
// in registers for the scaling pass), cols a multiple of 64.
constexpr int kCvtThreads = 512;
constexpr int kCvtVec = 8;  // float4 per thread: cols up to 16384 in one pass
__global__ void __launch_bounds__(kCvtThreads) to_f16_scaled_kernel(const float* __restrict__ x, int ntok, int cols,
                                                                      __half* __restrict__ xh, float* __restrict__ scale) {
    __shared__ float red[kCvtThreads / 32];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x, n4 = cols / 4;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * cols);
    float4 v[kCvtVec];
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < kCvtVec; k++) {
        const int i = threadIdx.x + k * kCvtThreads;
        v[k] = (t < ntok && i < n4) ? __ldg(xr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
    }
    // (columns past kCvtVec * kCvtThreads * 4: a second, rare pass below)
    for (int i = threadIdx.x + kCvtVec * kCvtThreads; t < ntok && i < n4; i += kCvtThreads) {
        const float4 w = __ldg(xr + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(w.x), fabsf(w.y)), fmaxf(fabsf(w.z), fabsf(w.w))));
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kCvtThreads / 32; i++) mx = fmaxf(mx, red[i]);
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
        int ex;
        frexpf(mx, &ex);  // mx in [2^(ex-1), 2^ex)
        e = 15 - ex;
    }
    const float up = ldexpf(1.0f, e);
    if (threadIdx.x == 0) scale[t] = ldexpf(1.0f, -e);
    uint2* xo = reinterpret_cast<uint2*>(xh + (size_t)t * cols);
#pragma unroll
    for (int k = 0; k < kCvtVec; k++) {
        const int i = threadIdx.x + k * kCvtThreads;
        if (i < n4) {
            const __half2 a = __floats2half2_rn(v[k].x * up, v[k].y * up), b = __floats2half2_rn(v[k].z * up, v[k].w * up);
            xo[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
        }
    }
    for (int i = threadIdx.x + kCvtVec * kCvtThreads; i < n4; i += kCvtThreads) {
        float4 w = t < ntok ? __ldg(xr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const __half2 a = __floats2half2_rn(w.x * up, w.y * up), b = __floats2half2_rn(w.z * up, w.w * up);
        xo[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
}

// Split-K partials [ks][ntok][rows] -> y [ntok][rows], summed in split order
// (the same sums whatever order the CTAs finished in): float4 elements when
// y is 16-byte aligned and the count divides by 4, single floats otherwise.
__global__ void splitk_sum4_kernel(const float* __restrict__ part, int ks, size_t n4, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const float4* p = reinterpret_cast<const float4*>(part);
    float4* o = reinterpret_cast<float4*>(y);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 v = __ldcg(p + i);
        for (int s = 1; s < ks; s++) {
            const float4 w = __ldcg(p + (size_t)s * n4 + i);
            v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
        }
        o[i] = v;
    }
}
__global__ void splitk_sum1_kernel(const float* __restrict__ part, int ks, size_t n, float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = __ldcg(part + i);
        for (int s = 1; s < ks; s++) v += __ldcg(part + (size_t)s * n + i);
        y[i] = v;
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn(std::string* err) {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) *err = "cuTensorMapEncodeTiled is not available from the driver";
    return fn;
}

bool make_map_2d(EncodeTiledFn enc, CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Per (device, stream) scratch: fp16 activations, token scales, split
// partials, the error flag.  Calls on one stream run in order.
struct GemmScratch {
    uint8_t* buf = nullptr;
    size_t bytes = 0;
    int* err = nullptr;
    int sms = 0;
    unsigned long long gen = 0;
};
std::mutex g_gemm_mu;
std::map<std::pair<int, cudaStream_t>, GemmScratch> g_gemm;
constexpr int kMaxDevices = 64;
// the whole gate/up product of b2_tiled_gemm_half_impl, per (device, stream)
std::map<std::pair<int, cudaStream_t>, std::pair<float*, size_t>> g_gemm_fused;

size_t al256(size_t n) { return (n + 255) & ~size_t(255); }

template <int QT, int BN>
int launch_qgemm(const CUtensorMap& mq, const CUtensorMap& ms, const CUtensorMap& mx, const GemmArgs& a, dim3 grid,
                 cudaStream_t s, std::string* err) {
    // the attribute belongs to a device: set once per device (under g_gemm_mu)
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *err = "no usable CUDA device";
        return B2_ERR_CUDA;
    }
    if (!attr[dev]) {
        if (cudaFuncSetAttribute(qgemm_kernel<QT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GemmSmem<QT, BN>::kTotal) != cudaSuccess) {
            *err = "cudaFuncSetAttribute (tensor-core GEMM) failed";
            return B2_ERR_CUDA;
        }
        attr[dev] = true;
    }
    // programmatic dependent launch: the CTAs may start (and stream their
    // first weights) while the previous kernel on the stream finishes; the
    // kernel waits for it (griddepcontrol.wait) before it reads activations
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmSmem<QT, BN>::kTotal;
    cfg.stream = s;
    cudaLaunchAttribute attr_pdl[1];
    attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr_pdl;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, qgemm_kernel<QT, BN>, mq, ms, mx, a) != cudaSuccess) {
        *err = "tensor-core GEMM launch failed";
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

template <int QT>
int launch_bn(int bn, const CUtensorMap& mq, const CUtensorMap& ms, const CUtensorMap& mx, const GemmArgs& a,
              dim3 grid, cudaStream_t s, std::string* err) {
    switch (bn) {
        case 16: return launch_qgemm<QT, 16>(mq, ms, mx, a, grid, s, err);
        case 32: return launch_qgemm<QT, 32>(mq, ms, mx, a, grid, s, err);
        case 64: return launch_qgemm<QT, 64>(mq, ms, mx, a, grid, s, err);
        case 128: return launch_qgemm<QT, 128>(mq, ms, mx, a, grid, s, err);
        default: return launch_qgemm<QT, 256>(mq, ms, mx, a, grid, s, err);
    }
}

}  // namespace
}  // namespace b2

using namespace b2;

// Y = W X over rows [row0, row0 + rows) of a tiled Q8_0 / Q4_0 matrix
// (base: the tiled matrix, rp its padded rows, cols = K) for ntok tokens:
// x [ntok][cols] fp32, y [ntok][rows] fp32, device memory, stream s.
namespace {
// N tile: the token count rounded up, 256 at most (the widest MMA: each
// dequantised A tile then feeds twice the products of a 128-token tile)
int bn_for(int ntok) { return ntok <= 16 ? 16 : ntok <= 32 ? 32 : ntok <= 64 ? 64 : ntok <= 128 ? 128 : 256; }

// Both entry points: x (fp32, converted here) or xh / tsc (already fp16).
int gemm_run(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols, const float* x,
             const __half* xh_in, const float* tsc_in, float* y, int ntok, GemmParts* parts, cudaStream_t s,
             std::string* err) {
    if (qtype != 8 && qtype != 2) {
        *err = "tensor-core GEMM takes Q8_0 or Q4_0 weights";
        return B2_ERR_UNSUPPORTED_TYPE;
    }
    if (ntok < 1 || rows < 1 || cols < 64 || cols % 64 || row0 % kTileRows || row0 + rows > rp) {
        *err = "tensor-core GEMM: cols must be a multiple of 64 and rows inside the matrix";
        return B2_ERR_BAD_ARG;
    }
    if ((x ? (reinterpret_cast<uintptr_t>(x) & 15) : (!xh_in || !tsc_in || (reinterpret_cast<uintptr_t>(xh_in) & 15))) ||
        (reinterpret_cast<uintptr_t>(y) & 3)) {
        *err = "x must be 16-byte aligned and y 4-byte aligned";
        return B2_ERR_BAD_ARG;
    }
    std::string e2;
    EncodeTiledFn enc = encode_fn(&e2);
    if (!enc) {
        *err = e2;
        return B2_ERR_CUDA;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *err = "no CUDA device";
        return B2_ERR_CUDA;
    }
    const int bn = bn_for(ntok);
    const int n_tiles = (ntok + bn - 1) / bn;
    const int ntok_pad = n_tiles * bn;
    const int nb = cols / 32;
    const int nst = nb / kStageBlocks;
    const int m_tiles = (rows + kBM - 1) / kBM;
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    GemmScratch* sc = &g_gemm[{dev, s}];
    if (!sc->sms && cudaDeviceGetAttribute(&sc->sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        *err = "cudaDeviceGetAttribute failed";
        return B2_ERR_CUDA;
    }
    // split K until the tiles cover the SMs (at least 4 stages per split)
    int ksplit = 1;
    while (ksplit < kMaxKSplit && (long long)m_tiles * n_tiles * ksplit < sc->sms && nst / (2 * ksplit) >= 4) ksplit *= 2;
    const int kst = (nst + ksplit - 1) / ksplit;
    ksplit = (nst + kst - 1) / kst;
    const size_t b_x = x ? al256((size_t)ntok_pad * cols * 2) : 0, b_sc = x ? al256((size_t)ntok_pad * 4) : 0;
    const size_t b_part = ksplit > 1 ? al256((size_t)ksplit * ntok * rows * 4) : 0;
    const size_t need = 256 + b_x + b_sc + b_part;
    if (sc->bytes < need) {
        if (sc->buf) cudaFree(sc->buf);
        sc->buf = nullptr;
        sc->bytes = 0;
        if (cudaMalloc(&sc->buf, need) != cudaSuccess) {
            *err = "tensor-core GEMM scratch allocation failed";
            return B2_ERR_OOM;
        }
        cudaMemsetAsync(sc->buf, 0, 256, s);
        sc->bytes = need;
        sc->err = reinterpret_cast<int*>(sc->buf);
        sc->gen++;
    }
    __half* xh = x ? reinterpret_cast<__half*>(sc->buf + 256) : const_cast<__half*>(xh_in);
    const float* tsc = x ? reinterpret_cast<float*>(sc->buf + 256 + b_x) : tsc_in;
    float* part = ksplit > 1 ? reinterpret_cast<float*>(sc->buf + 256 + b_x + b_sc) : nullptr;

    const bool q8 = qtype == 8;
    const int QB = q8 ? 32 : 16;
    const int64_t tiles_total = rp / kTileRows;
    const uint8_t* wq = static_cast<const uint8_t*>(base);
    const uint8_t* ws = wq + (size_t)rp * nb * QB;
    CUtensorMap mq, ms, mx;
    if (!make_map_2d(enc, &mq, CU_TENSOR_MAP_DATA_TYPE_UINT64, wq, (uint64_t)nb * kTileRows * QB / 8, tiles_total,
                     (uint64_t)nb * kTileRows * QB, kStageBlocks * kTileRows * QB / 8, kBM / kTileRows,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(enc, &ms, CU_TENSOR_MAP_DATA_TYPE_UINT64, ws, (uint64_t)nb * kTileRows * 2 / 8, tiles_total,
                     (uint64_t)nb * kTileRows * 2, kStageBlocks * kTileRows * 2 / 8, kBM / kTileRows,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(enc, &mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, (uint64_t)cols, (uint64_t)ntok_pad,
                     (uint64_t)cols * 2, 64, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)) {
        *err = "tensor map encoding failed (alignment)";
        return B2_ERR_BAD_ARG;
    }
    if (x)
        launch_pdl(to_f16_scaled_kernel, dim3(ntok_pad), dim3(kCvtThreads), 0, s, x, ntok, cols, xh,
                   const_cast<float*>(tsc));
    GemmArgs a{};
    a.nst = nst;
    a.kst_split = kst;
    a.tiles_q = (int)(row0 / kTileRows);
    a.rows = rows;
    a.ntok = ntok;
    a.ldy = rows;
    a.y = y;
    a.ksplit = ksplit;
    a.part = part;
    a.tok_scale = tsc;
    a.err = sc->err;
    const dim3 grid(m_tiles, n_tiles, ksplit);
    int rc = q8 ? launch_bn<8>(bn, mq, ms, mx, a, grid, s, err) : launch_bn<2>(bn, mq, ms, mx, a, grid, s, err);
    if (rc) return rc;
    if (parts) {
        parts->p = ksplit > 1 ? part : y;
        parts->k = ksplit;
        parts->plane = (size_t)ntok * rows;
    } else if (ksplit > 1) {
        const size_t n = (size_t)ntok * rows;
        const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;  // (part is 256-aligned)
        const size_t units = vec ? n / 4 : n;
        const int blocks = (int)std::min<size_t>((size_t)sc->sms * 8, (units + 255) / 256);
        if (vec) launch_pdl(splitk_sum4_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, s, part, ksplit, units, y);
        else launch_pdl(splitk_sum1_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, s, part, ksplit, units, y);
    }
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
        *err = std::string("tensor-core GEMM launch: ") + cudaGetErrorString(ce);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}
}  // namespace

int b2_tiled_gemm_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols, const float* x,
                       float* y, int ntok, cudaStream_t s, std::string* err) {
    if (!x) {
        *err = "null argument";
        return B2_ERR_BAD_ARG;
    }
    return gemm_run(qtype, base, rp, row0, rows, cols, x, nullptr, nullptr, y, ntok, nullptr, s, err);
}

int b2_tiled_gemm_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols, const float* x,
                       float* y, int ntok, GemmParts* parts, cudaStream_t s, std::string* err) {
    if (!x) {
        *err = "null argument";
        return B2_ERR_BAD_ARG;
    }
    return gemm_run(qtype, base, rp, row0, rows, cols, x, nullptr, nullptr, y, ntok, parts, s, err);
}

int b2_tiled_gemm_f16_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols,
                           const void* xh, const float* tok_scale, int ntok, float* y, GemmParts* parts,
                           cudaStream_t s, std::string* err) {
    return gemm_run(qtype, base, rp, row0, rows, cols, nullptr, static_cast<const __half*>(xh), tok_scale, y, ntok,
                    parts, s, err);
}

int b2_gemm_pad_tokens(int ntok) {
    const int bn = bn_for(ntok);
    return (ntok + bn - 1) / bn * bn;
}

namespace b2 {
namespace {
// y[t][j] = fused[t][16 (j / 8) + j % 8 + 8 (half - 1)]: one half (gate 1,
// up 2) of a gate/up product computed over the interleaved resident matrix.
__global__ void gather_half_kernel(const float* __restrict__ fused, int ntok, int rows, int half,
                                   float* __restrict__ y) {
    pdl_trigger();
    pdl_wait();
    const size_t n = (size_t)ntok * rows;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / rows;
        const int j = (int)(i - t * rows);
        y[i] = fused[t * 2 * rows + (size_t)(j >> 3) * 16 + (j & 7) + (half == 2 ? 8 : 0)];
    }
}
}  // namespace
}  // namespace b2

// The gate or up half (half 1 or 2) of the interleaved gate/up matrix (2 *
// rows resident rows): the product over the whole matrix into a buffer kept
// per (device, stream) and grown as needed, then that half's rows.
int b2_tiled_gemm_half_impl(int qtype, const void* base, int64_t rp, int half, int rows, int cols, const float* x,
                            float* y, int ntok, cudaStream_t s, std::string* err) {
    float* fused = nullptr;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) {
            *err = "no CUDA device";
            return B2_ERR_CUDA;
        }
        const size_t need = sizeof(float) * (size_t)ntok * 2 * rows;
        std::lock_guard<std::mutex> lk(g_gemm_mu);
        auto& f = g_gemm_fused[{dev, s}];
        if (f.second < need) {
            if (f.first) {
                cudaStreamSynchronize(s);  // earlier calls on s may still read it
                cudaFree(f.first);
            }
            f = {nullptr, 0};
            if (cudaMalloc(reinterpret_cast<void**>(&f.first), need) != cudaSuccess) {
                *err = "allocation of the gate/up product failed";
                return B2_ERR_OOM;
            }
            f.second = need;
        }
        fused = f.first;
    }
    int rc = b2_tiled_gemm_impl(qtype, base, rp, 0, 2 * rows, cols, x, fused, ntok, s, err);
    if (!rc) {
        const int blocks = (int)std::min<size_t>(4096, ((size_t)ntok * rows + 255) / 256);
        launch_pdl(gather_half_kernel, dim3(std::max(blocks, 1)), dim3(256), 0, s, fused, ntok, rows, half, y);
        if (cudaGetLastError() != cudaSuccess) {
            *err = "gate/up gather launch failed";
            rc = B2_ERR_CUDA;
        }
    }
    return rc;
}

// Device error flag of the GEMM scratch of stream s (0 if none); clears it.
int b2_gemm_status(cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B2_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    auto it = g_gemm.find({dev, s});
    if (it == g_gemm.end() || !it->second.err) return 0;
    int v = 0;
    cudaMemcpyAsync(&v, it->second.err, sizeof(int), cudaMemcpyDeviceToHost, s);
    cudaStreamSynchronize(s);
    if (v) cudaMemsetAsync(it->second.err, 0, sizeof(int), s);
    return v;
}

// Generation of the GEMM scratch of stream s (a CUDA graph that captured a
// GEMM on s stays valid while it is unchanged).
void b2_gemm_release(int dev, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    const auto it = g_gemm.find({dev, s});
    if (it != g_gemm.end()) {
        if (it->second.buf) cudaFree(it->second.buf);
        g_gemm.erase(it);
    }
    const auto f = g_gemm_fused.find({dev, s});
    if (f != g_gemm_fused.end()) {
        if (f->second.first) cudaFree(f->second.first);
        g_gemm_fused.erase(f);
    }
}

unsigned long long b2_gemm_scratch_generation(cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_gemm_mu);
    const auto it = g_gemm.find({dev, s});
    return it == g_gemm.end() ? 0 : it->second.gen;
}
