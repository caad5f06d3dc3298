// Device-side model description and PTX helpers shared by the decode kernels.
#pragma once
#include <stdint.h>
#ifdef __CUDACC__
#include <cuda_fp16.h>
#include <utility>
#endif

namespace b2 {

// One decode token is a fixed sequence of phases; phase p of layer l is
// 4*l + k with k below, and the lm_head phase is 4*L.  Phases hand their
// outputs to the next phase through "LL" words in global memory: 8 bytes =
// {fp32 value, 32-bit tag}, written with one 8-byte store, so a reader that
// sees the expected tag also sees the value.  Polling the data itself is the
// synchronisation; there is no grid barrier.  Weight bytes of later phases
// stream into shared memory ahead of time because they never depend on
// activations.
enum PhaseKind : int {
    PH_QA = 0,      // rmsnorm(x) -> q rows of one head + attention over the cached context (q CTAs);
                    //   k, v rows + KV-cache append (kv CTAs)
    PH_WO = 1,      // merge attention splits and the new position -> Wo rows, residual add
    PH_GATEUP = 2,  // rmsnorm(x) -> gate & up rows, SwiGLU -> act
    PH_DOWN = 3,    // act -> Wd rows, residual add
    PH_LMHEAD = 4,  // rmsnorm(x) -> lm_head rows, logits + argmax
    PH_MATVEC = 5,  // plain y = W x (kernel-level entry point)
};

constexpr int kPhasesPerLayer = 4;
constexpr int kConsumerWarps = 12;
constexpr int kThreads = 32 * (kConsumerWarps + 1);  // warp 0 = producer
constexpr int kMaxSplits = 8;                         // attention context splits per KV head
constexpr int kMaxTp = 8;                             // tensor-parallel ranks (GPUs of one box)
constexpr int kAttnTileBytes = 16384;                 // bytes of cached K (and of V) per attention tile
constexpr int kMaxAttnTile = 128;                     // positions per attention tile, at most
constexpr int kMaxOwnRows = 64;                       // residual rows one CTA keeps (H / grid)
constexpr int kMaxQkvRows = 256;                      // QA-phase rows one CTA computes (hd, or its k/v share)
// Phase trace slots: consumer phase start, input ready, input staged, work
// done; producer first and last weight copy issued (globaltimer ns); total ns
// the consumer warps spent waiting for weight chunks, and how many of those
// waits took longer than 256 ns; ns the producer waited for free ring slots,
// and the chunks it issued; consumer rows loop done (before the epilogue);
// total ns the consumer warps spent in tile dot products; epilogue constants
// ready.
constexpr int kTraceSlots = 13;

// Weight matrices live in HBM in a tiled form of their ggml blocks, made at
// load time (same bytes per weight as the GGUF file):
//   quants [Rp/16 tiles][nb blocks][16 rows][QB bytes]   QB = 32 (Q8_0) or 16 (Q4_0)
//   scales [Rp/16 tiles][nb blocks][16] f16              right after the quants
// Rp = rows rounded up to 16 (padding rows are zero).  A (tile, block) unit
// is contiguous, so any range of tiles x blocks is two 16-byte aligned copies,
// and in shared memory it is the 16 x 32-byte A operand of one int8
// mma.m16n8k32 (ldmatrix).  For Q8_0, rows with bit 2 set store their two
// 16-byte halves swapped, so ldmatrix reads any 8 rows of either half
// without bank conflicts.  The 16 scales of a unit are stored in the order
// rows 0, 8, 1, 9, ..., 7, 15: the mma lane that owns rows g and g + 8 reads
// both with one 32-bit load.
constexpr int kTileRows = 16;

inline
#ifdef __CUDACC__
__host__ __device__
#endif
int tile_qb(int qtype) { return qtype == 8 ? 32 : 16; }

inline
#ifdef __CUDACC__
__host__ __device__
#endif
int64_t tiled_rows(int64_t rows) { return (rows + kTileRows - 1) / kTileRows * kTileRows; }

inline
#ifdef __CUDACC__
__host__ __device__
#endif
size_t tiled_bytes(int64_t rows, int64_t cols, int qtype) {
    return (size_t)(tiled_rows(rows) * (cols / 32) * (tile_qb(qtype) + 2));
}

// Byte offset of quant byte e (0..31 for Q8_0, 0..15 for Q4_0) of row r, block b.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
size_t tiled_qoff(int64_t r, int64_t b, int e, int64_t nb, int qtype) {
    const int qb = tile_qb(qtype);
    const int rr = (int)(r & (kTileRows - 1));
    const int ee = qtype == 8 ? (e ^ ((rr & 4) << 2)) : e;
    return (size_t)((((r / kTileRows) * nb + b) * kTileRows + rr) * qb + ee);
}
// Byte offset of the f16 scale of row r, block b (rp = tiled_rows(rows)).
inline
#ifdef __CUDACC__
__host__ __device__
#endif
size_t tiled_soff(int64_t r, int64_t b, int64_t nb, int64_t rp, int qtype) {
    const int rr = (int)(r & (kTileRows - 1));
    const int pos = 2 * (rr & 7) + (rr >> 3);
    return (size_t)(rp * nb * tile_qb(qtype) + (((r / kTileRows) * nb + b) * kTileRows + pos) * 2);
}

// Static work plan of one CTA in one weight phase: its tiles [u0, u0 + n),
// cut into chunks of nt tiles x one K-slice of bpk blocks (nks slices), each
// chunk small enough for one ring slot.  K is split when a tile's blocks do
// not fit a slot, or to give more warps work when the CTA has few tiles.
// Producer, consumers and the host evaluate the same function.
struct TPlan {
    int u0, n;      // tiles of this CTA
    int nks, bpk;   // K-slices and blocks per slice
    int nt;         // tiles per chunk
    int nchunks;    // = ceil(n / nt) * nks
    int kb0, kbn;   // the row blocks [kb0, kb0 + kbn) the plan covers (all of them but in a K-split phase)
};

// Plan of the tile range [u0, u0 + n) (see TPlan).
inline
#ifdef __CUDACC__
__host__ __device__
#endif
TPlan tile_plan_range(int u0, int n, int nb, int tbb, int slot_bytes, int warps) {
    // tbb: bytes of one (tile, block) unit incl. scales (x2 for gate + up)
    TPlan t;
    t.u0 = u0;
    t.n = n;
    t.kb0 = 0;
    t.kbn = nb;
    if (t.n <= 0) {
        t.n = 0; t.nks = 1; t.bpk = nb; t.nt = 1; t.nchunks = 0;
        return t;
    }
    const int fit = slot_bytes / tbb;                 // blocks per slot
    int nks = (nb + fit - 1) / fit;                   // slices needed to fit a slot
    int want = (warps + t.n - 1) / t.n;               // slices that keep the warps busy
    const int cap = nb / 4 > 0 ? nb / 4 : 1;          // at least 4 blocks per slice
    if (want > cap) want = cap;
    if (want > nks) nks = want;
    t.bpk = (nb + nks - 1) / nks;
    t.nks = (nb + t.bpk - 1) / t.bpk;
    if (t.nks == 1) {
        int nt = fit / nb;                            // whole tiles per slot
        const int spread = (t.n + warps - 1) / warps;
        if (nt > spread) nt = spread;
        t.nt = nt < 1 ? 1 : nt;
    } else {
        t.nt = 1;
    }
    t.nchunks = (t.n + t.nt - 1) / t.nt * t.nks;
    return t;
}

// Even split of `tiles` over the grid.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
TPlan tile_plan(int tiles, int nb, int tbb, int cta, int grid, int slot_bytes, int warps) {
    const int u0 = (int)((long long)cta * tiles / grid);
    const int n = (int)((long long)(cta + 1) * tiles / grid) - u0;
    return tile_plan_range(u0, n, nb, tbb, slot_bytes, warps);
}

// The residual-stream rows a CTA owns (the tiles of the H-row phases, Wo
// and down, and the rows it keeps in shared memory across them).  With no
// more tiles than CTAs they go to the last CTAs of the grid, one each, so the
// first CTAs (the QA phase's q CTAs, whose attention ends the QA phase last)
// own none and the Wo phase does not wait for them twice; otherwise an even
// split.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
void own_tiles(int tiles, int cta, int grid, int* u0, int* n) {
    if (tiles <= grid) {
        const int first = grid - tiles;
        *n = cta >= first ? 1 : 0;
        *u0 = cta >= first ? cta - first : 0;
        return;
    }
    *u0 = (int)((long long)cta * tiles / grid);
    *n = (int)((long long)(cta + 1) * tiles / grid) - *u0;
}
inline
#ifdef __CUDACC__
__host__ __device__
#endif
TPlan own_plan(int tiles, int nb, int tbb, int cta, int grid, int slot_bytes, int warps) {
    int u0 = 0, n = 0;
    own_tiles(tiles, cta, grid, &u0, &n);
    return tile_plan_range(u0, n, nb, tbb, slot_bytes, warps);
}

// The down phase split over K (single GPU, when the grid has at least two
// CTAs per residual tile): tile t of the H / kTileRows down tiles goes to
// CTAs first + 2t and first + 2t + 1 (first = grid - 2 * h_tiles, so the
// residual-row owners at the end of the grid take part), each with one half
// of the row's blocks; they publish partial sums, which the consumers of the
// residual stream add.  kDownSplit is the number of halves.
constexpr int kDownSplit = 2;
inline
#ifdef __CUDACC__
__host__ __device__
#endif
int dn_slice_of(int cta, int grid, int h_tiles) {
    const int c = cta - (grid - kDownSplit * h_tiles);
    return c < 0 ? -1 : c % kDownSplit;
}
inline
#ifdef __CUDACC__
__host__ __device__
#endif
TPlan dn_split_plan(int h_tiles, int nb, int tbb, int cta, int grid, int slot_bytes, int warps) {
    const int c = cta - (grid - kDownSplit * h_tiles);
    if (c < 0) return tile_plan_range(0, 0, nb, tbb, slot_bytes, warps);
    const int t = c / kDownSplit, s = c % kDownSplit;
    const int kb0 = s * nb / kDownSplit, kb1 = (s + 1) * nb / kDownSplit;
    TPlan p = tile_plan_range(t, 1, kb1 - kb0, tbb, slot_bytes, warps);
    p.kb0 = kb0;
    return p;
}

// Gate/up tiles of one CTA.  The CTAs that own residual rows (own_tiles of
// the H / kTileRows Wo and down tiles) also stream those two matrices every
// layer, so they take own_pct percent of the gate/up share of the others:
// the bytes per layer come out close on every CTA, and the owners' ring
// slots are free to prefetch their down tiles during the gate/up phase.
// own_pct = 100 is the even split.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
TPlan gu_plan(int tiles, int nb, int tbb, int cta, int grid, int slot_bytes, int warps, int h_tiles, int own_pct) {
    if (h_tiles > grid || own_pct == 100) return tile_plan(tiles, nb, tbb, cta, grid, slot_bytes, warps);
    const int first = grid - h_tiles;  // first owner CTA
    const long long W = (long long)first * 100 + (long long)h_tiles * own_pct;
    auto cum = [&](int c) {
        return c <= first ? (long long)c * 100 : (long long)first * 100 + (long long)(c - first) * own_pct;
    };
    const int u0 = (int)(tiles * cum(cta) / W);
    const int n = (int)(tiles * cum(cta + 1) / W) - u0;
    return tile_plan_range(u0, n, nb, tbb, slot_bytes, warps);
}

// QA phase rows.  Fused form: q CTAs 0 .. nh*S - 1 (head h = cta / S, split
// cta % S) each compute the hd / kTileRows q tiles of their head and keep
// them; the kv CTAs nh*S .. grid - 1 share the k and v tiles evenly.
// Distributed form (`dist`, for heads whose q rows are too much work for one
// CTA): every CTA takes an even share of all q, k, v tiles and publishes
// them; the q CTAs then read their head's q back.  Returns the tile range.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
void qa_tiles(int nh, int hd, int qd, int kvd, int S, int cta, int grid, int* u0, int* n, int dist) {
    const int nq = nh * S, tph = hd / kTileRows;
    if (dist) {
        const int tiles = (qd + 2 * kvd) / kTileRows;
        *u0 = (int)((long long)cta * tiles / grid);
        *n = (int)((long long)(cta + 1) * tiles / grid) - *u0;
        return;
    }
    if (cta < nq) {
        *u0 = (cta / S) * tph;
        *n = tph;
        return;
    }
    const int kv0 = qd / kTileRows, nkv = 2 * kvd / kTileRows, J = grid - nq, j = cta - nq;
    if (nkv <= J) {
        // one tile each on the first CTAs after the q CTAs: the residual-row
        // owners sit at the end of the grid and enter this phase last (they
        // finish the previous down phase), while every q CTA's last split
        // waits for these rows
        *u0 = kv0 + (j < nkv ? j : 0);
        *n = j < nkv ? 1 : 0;
        return;
    }
    *u0 = kv0 + (int)((long long)j * nkv / J);
    *n = kv0 + (int)((long long)(j + 1) * nkv / J) - *u0;
}

// Work plans of one CTA, computed on the host at load time (no divisions in
// the kernel): Wo, gate/up, down, the lm_head's sub-phases 0 .. kMaxLmSub - 1
// (consecutive parts of the CTA's lm_head tiles, so that one part's K-slice
// results fit the phase buffer), then QA for S = 1 .. kMaxSplits.
constexpr int kMaxLmSub = 8;
constexpr int kPlanSlots = 3 + kMaxLmSub + kMaxSplits;
// S: the QA phase's split count (1 ..), or the lm_head's sub-phase (0 ..)
inline
#ifdef __CUDACC__
__host__ __device__
#endif
int plan_slot(int kind, int S) {
    return kind == PH_QA ? 3 + kMaxLmSub + S - 1 : (kind == PH_LMHEAD ? 3 + S : kind - 1);
}

struct LayerDev {
    const uint8_t* wqkv;  // tiled [(qd + 2*kvd) rows][H]: Wq rows, then Wk, then Wv
    const uint8_t* wo;    // tiled [H rows][qd]
    const uint8_t* wgu;   // tiled [2*FF rows][H]: gate and up interleaved 8 rows at a time
    const uint8_t* wd;    // tiled [H rows][FF]
    const float* attn_norm;
    const float* ffn_norm;
    const float* bqkv;    // [qd + 2*kvd] or null
};

struct ModelDev {
    int H, FF, V, L, nh, nkv, hd, qd, kvd, max_seq;
    int qtype;            // 8 = Q8_0, 2 = Q4_0 (ggml layout)
    int rb_h, rb_q, rb_f; // row bytes for inputs of width H, qd, FF
    float eps;
    int kv_fp32;
    int slot_bytes, nslots;   // shared-memory ring geometry
    int xs_floats;            // phase input / attention scratch (floats)
    int ybuf_floats;          // phase outputs of one CTA: even phases' buffer (QA, gate/up, LM head)
    int ybuf_odd;             // ... and the odd phases' buffer (Wo, down) right after it
    int cfloats;              // phase constants: norm gains, QKV bias, RoPE row
    int attn_tile;            // positions per attention tile
    int qa_dist;              // QA rows spread over all CTAs (q published, read back by the q CTAs)
    int n_lm;                 // lm_head sub-phases (phases 4L .. 4L + n_lm - 1)
    int nbx;                  // 32-blocks of the widest phase input (xq planes)
    const TPlan* plans;       // [grid][kPlanSlots] work plans (plan_slot)
    int Vp;                   // lm_head rows (this rank's vocab share) rounded up to kTileRows
    int Vemb, Vp_emb;         // embedding rows (the whole vocab) and rounded up
    int v_off;                // first vocab row of this rank's lm_head share
    const uint8_t* tok_embd;  // tiled [Vemb rows][H]
    const uint8_t* lm_head;   // tiled [V rows][H] (tok_embd when tied on one GPU)
    const float* out_norm;
    const float* rope_cos;    // [max_seq][hd/2]
    const float* rope_sin;
    void* kcache;             // [L][max_seq][kvd] fp16 or fp32
    void* vcache;
    const LayerDev* layers;   // device array [L]
    // phase hand-off buffers of LL words (uint2 = {value bits, tag})
    uint2* ll_x1;             // [H]   x after the attention residual
    uint2* ll_x2;             // [H]   x after the FFN residual
    uint2* ll_qkv;            // [qd + 2*kvd] q, k (after RoPE), v of the new token
    uint2* ll_part;           // [nh][kMaxSplits][hd + 2] attention split partials (o, m, l)
    uint2* ll_act;            // [FF]  SwiGLU output
    uint2* ll_dnp;            // [2 (layer parity)][kDownSplit][H] down-phase partial sums (split mode)
    int dn_split;             // 1: down rows on their residual owners; kDownSplit: split over K (dn_split_plan)
    float* logits;            // [V]
    unsigned long long* am_key;  // [1] argmax so far: order-preserving value bits << 32 | ~index (self-resetting)
    int* token;               // [1] last argmax
    unsigned* am_ctr;         // [1] argmax arrivals (self-resetting)
    int* err;                 // device error flag (B2_ERR_* codes)
    // tensor parallelism: this rank's heads, FFN rows and vocab share are the
    // dims above; the Wo and down partial sums and the argmax keys go through
    // every rank's exchange buffer (xpeer[tp_rank] is this rank's own)
    int tp, tp_rank;
    uint8_t* xpeer[kMaxTp];
};

// Tensor-parallel exchange buffer (one per rank, the same layout on all;
// peers map it through CUDA IPC): the Wo and the down partial rows of every
// rank [tp][H] LL words each, then every rank's LM-head argmax key (16 bytes:
// order-preserving value bits, tag, ~index, tag).
inline
#ifdef __CUDACC__
__host__ __device__
#endif
size_t xch_dn(int H, int tp) { return (size_t)tp * H * 8; }
inline
#ifdef __CUDACC__
__host__ __device__
#endif
size_t xch_am(int H, int tp) { return 2 * (size_t)tp * H * 8; }
inline size_t xch_bytes(int H, int tp) { return xch_am(H, tp) + 16 * (size_t)tp; }

// Per-launch arguments of the decode kernel.
struct StepArgs {
    const int* tok;      // device pointer to this step's input token
    int pos;             // cache position written by this step
    int p_begin, p_end;  // phase range to run
    unsigned epoch;      // launch number: LL tags are epoch * 256 + layer + 1
    unsigned skew;       // added to every awaited tag (test hook; 0 normally)
    int splits;          // attention context splits per KV head
    int* out_ids;        // argmax also written to out_ids[step] when non-null
    int step;
    int eos;             // with done: an argmax equal to eos sets *done
    int* done;           // device flag; a launch that finds it set does no work
    unsigned long long* trace;  // [phases][kTraceSlots][grid] timestamps, or null
    // PH_MATVEC only
    const uint8_t* mv_w;
    const float* mv_x;
    float* mv_y;
    int mv_rows, mv_cols, mv_rb;
};

// Dynamic shared-memory layout of the decode kernel (byte offsets).
//   ring   [nslots][slot_bytes]   weight slots filled by the producer
//   xs     [xs_floats]            the matvec mode's input vector, or the
//                                 QA phase's attention scratch
//   xres   [kMaxOwnRows]          residual rows this CTA owns
//   ybuf   [ybuf_floats]          dot results of the phase (parity buffers,
//                                 even phases first, then the odd ones)
//   cbuf   [cfloats]              phase constants (norm gains, bias, RoPE)
//   full, empty [nslots] mbarriers; red [64] floats; misc [32] ints
//   dnp    [kDownSplit][16] LL    the down partials of an owner's rows (split mode)
//   plan   [kPlanSlots] TPlan     this CTA's work plans (copied at launch)
//   lay    [L] LayerDev           the layer table (copied at launch)
struct SmemOffsets {
    uint32_t xs, xq, xsc, xsm, xres, ybuf, cbuf, full, empty, red, misc, dnp, plan, lay, total;
};

// xq holds the phase input as three int8 planes in the operand layout of
// mma.m16n8k32: per 32-element block, 12 lanes x {a0, a2} words (96 bytes);
// xsc the per-block scales (fp32) and xsm, for Q4_0, the per-block int32
// accumulator starts of planes 0-2 (1.5 * 2^23 - 8 * plane sum) and 1.5 * 2^23.
inline
#ifdef __CUDACC__
__host__ __device__
#endif
SmemOffsets smem_offsets(int nslots, int slot_bytes, int xs_floats, int ybuf_floats, int cfloats, int nbx,
                         int nlayers) {
    SmemOffsets o;
    uint32_t p = (uint32_t)nslots * (uint32_t)slot_bytes + 128u;
    o.xs = p;    p += 4u * (uint32_t)xs_floats;
    o.xq = p;    p += 96u * (uint32_t)nbx;
    o.xsc = p;   p += 4u * (uint32_t)nbx;
    p = (p + 15u) & ~15u;
    o.xsm = p;   p += 16u * (uint32_t)nbx;
    p = (p + 15u) & ~15u;
    o.xres = p;  p += 4u * kMaxOwnRows;
    o.ybuf = p;  p += 4u * (uint32_t)ybuf_floats;
    o.cbuf = p;  p += 4u * (uint32_t)cfloats;
    p = (p + 15u) & ~15u;
    o.full = p;  p += 8u * (uint32_t)nslots;
    o.empty = p; p += 8u * (uint32_t)nslots;
    o.red = p;   p += 4u * 64u;
    o.misc = p;  p += 4u * 32u;
    p = (p + 15u) & ~15u;
    o.dnp = p;   p += 8u * kTileRows * kDownSplit;
    o.plan = p;  p += (uint32_t)(kPlanSlots * sizeof(TPlan));
    p = (p + 15u) & ~15u;
    o.lay = p;   p += (uint32_t)(nlayers * sizeof(LayerDev));
    p = (p + 15u) & ~15u;
    o.total = p;
    return o;
}

// Constant buffer layout (floats): the QKV bias of this CTA's rows from row
// (16 * u0) & ~3 (kMaxQkvRows + 4); then hd/2 cos and hd/2 sin of the RoPE
// row at the current position.
inline int cb_floats(int hd) { return (kMaxQkvRows + 4 + hd + 31) & ~31; }

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// 1-D bulk copy global -> shared (TMA), completing on an mbarrier.  src, dst
// and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Lets the kernel launched after this one on the stream with programmatic
// dependent launch start now (it waits for this grid's completion, with
// griddepcontrol.wait, before it reads anything this grid writes).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Waits until the grid this one was launched after (programmatic dependent
// launch) has completed and its writes are visible; returns at once for a
// grid launched without the attribute.  A kernel launched by launch_pdl
// calls it before its first global read or write, in every thread, so its
// own completion still implies its predecessor's (the chain of launches
// stays ordered for the kernels after it).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launches kern<<<grid, block, smem, s>>>(args...) as a programmatic
// dependent launch: its CTAs may be scheduled while the kernel before it on
// the stream finishes (once that one has called pdl_trigger in every CTA, or
// exited), and wait in pdl_wait for its completion.  Hides the launch and
// the prologue of a short kernel behind its predecessor's tail; inside a
// captured graph the dependency becomes a programmatic edge.
template <typename... P, typename... A>
cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_acq_rel_add(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// 16-byte global -> shared copies, completed per thread with cp_async_wait().
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// all but the most recent committed group
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}


// ---- LL words: {fp32 value, tag} in one 8-byte store -----------------------
__device__ __forceinline__ void ll_store(uint2* p, float v, unsigned tag) {
    asm volatile("st.relaxed.gpu.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag)
                 : "memory");
}
// Two adjacent LL words with one 16-byte store (p 16-byte aligned).
__device__ __forceinline__ void ll_store2(uint2* p, float v0, float v1, unsigned tag) {
    asm volatile("st.relaxed.gpu.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(v0)), "r"(tag),
                 "r"(__float_as_uint(v1)), "r"(tag)
                 : "memory");
}
// System-scope LL words for the tensor-parallel exchange buffers (written by
// peer GPUs over NVLink, polled by the owner).
__device__ __forceinline__ void ll_store_sys(uint2* p, float v, unsigned tag) {
    asm volatile("st.relaxed.sys.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag)
                 : "memory");
}
__device__ __forceinline__ uint2 ll_load_sys(const uint2* p) {
    uint2 r;
    asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ void st4_sys(uint4* p, uint4 v) {
    asm volatile("st.relaxed.sys.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld4_sys(const uint4* p) {
    uint4 r;
    asm volatile("ld.relaxed.sys.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ uint2 ll_load1(const uint2* p) {
    uint2 r;
    asm volatile("ld.relaxed.gpu.global.v2.b32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ uint4 ll_load2(const uint2* p) {
    uint4 r;
    asm volatile("ld.relaxed.gpu.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

// ---- packed fp32x2 arithmetic (sm_100a) -------------------------------------
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Four bytes -> two exact float pairs via the 2^23 magic: the byte placed in
// the low mantissa byte of 0x4B000000 is the float 2^23 + byte.  sub is the
// pair (2^23 + 128) for int8 after ^0x80, or (2^23 + 8) for Q4_0 nibbles.
__device__ __forceinline__ void bytes_to_f2(uint32_t u, unsigned long long sub, unsigned long long& p01,
                                            unsigned long long& p23) {
    p01 = f2_add(f2_pack(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                         __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))), sub);
    p23 = f2_add(f2_pack(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                         __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))), sub);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Four signed bytes -> four exact floats.  (b ^ 0x80) placed in the low
// mantissa byte of 2^23 gives the float 2^23 + b + 128; subtracting
// 2^23 + 128 leaves b exactly.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}

// Four nibbles (0..15, one per byte) -> four exact floats of (nibble - 8).
__device__ __forceinline__ void u4x4_to_f32(uint32_t w, float* f) {
    f[0] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)) - 8388616.0f;
    f[1] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)) - 8388616.0f;
    f[2] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)) - 8388616.0f;
    f[3] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)) - 8388616.0f;
}

#endif  // __CUDACC__

}  // namespace b2
