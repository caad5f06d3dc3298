// Device-side sampling: repetition penalty, temperature, top-K, top-P and
// the multinomial draw of transformer.go:981-1114 (sample, topKFilter,
// topPFilter, softmax) on the logits the decode step left in HBM, so a
// sampled token costs one small launch and a 4-byte read instead of a copy
// of the whole vocabulary's logits to the host and a host sort.
//
// A cooperative launch of a group of CTAs per sequence, each owning a slice
// of the vocabulary, joined by bounded group barriers; after top-K the
// survivors (usually a few dozen) are compacted in vocabulary order and one
// CTA finishes over them in shared memory.  The selections are radix selects
// on an order-preserving 32-bit key of the float logit (four 8-bit digits,
// most significant first), never a sort:
//   - top-K: the k-th largest key by counts (topKFilter keeps every logit
//     >= the k-th largest value, ties included);
//   - top-P: the cut of topPFilter's stable descending sort by probability
//     mass, the mass of a key bucket being an integer (2^40 fixed point of
//     exp(logit - max)), so the sums are exact and do not depend on the
//     order of the atomics; among equal logits the stable sort keeps index
//     order, and so does the tie rank here;
//   - the draw: the first index (in vocabulary order) whose inclusive
//     prefix of the kept masses reaches r times their total.
//
// The host code sums float probabilities one after another; these sums are
// exact fixed-point sums of the same float terms, so the two agree except
// where r (or top_p) lies within float rounding of a cumulative boundary.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <string>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "sample.h"

namespace b2 {
namespace {

constexpr int kSampleThreads = 512;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kSampleCap = 4096;  // survivors of top-K kept in shared memory
constexpr double kMassScale = 1099511627776.0;  // 2^40: exp(v - max) in (0, 1] -> integer mass

__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (float)exp((double)(v - mx)) as the host computes it, in fixed point.
__device__ __forceinline__ float e_of(float v, float mx) { return (float)exp((double)(v - mx)); }
__device__ __forceinline__ uint64_t q_of(float e) { return __double2ull_rn((double)e * kMassScale); }

struct SampleSmem {
    uint32_t hc[256];             // digit histogram: counts
    unsigned long long hm[256];   // digit histogram: masses
    unsigned long long wsum[kSampleWarps];
    float wf[kSampleWarps];
    int wi[kSampleWarps];
    int lidx[kSampleCap];         // compacted set: vocabulary index (ascending)
    float lval[kSampleCap];       //                logit
    float le[kSampleCap];         //                exp(logit - max)
    unsigned long long gsum[160];  // a group's per-CTA values, staged from global memory
    float gmax[160];
    int gcnt[160];
    int sel, nlist, tie_last, out, ok;
    uint32_t thr_key;
    unsigned long long above;
};

__device__ float block_max(float v, SampleSmem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (l == 0) s.wf[w] = v;
    __syncthreads();
    v = s.wf[0];
    for (int i = 1; i < kSampleWarps; i++) v = fmaxf(v, s.wf[i]);
    return v;
}

__device__ unsigned long long block_sum_u64(unsigned long long v, SampleSmem& s) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (l == 0) s.wsum[w] = v;
    __syncthreads();
    v = 0;
    for (int i = 0; i < kSampleWarps; i++) v += s.wsum[i];
    return v;
}



// The top-K survivors compacted into shared memory (positions j in
// ascending vocabulary order), the set the single-CTA stages work on.
struct ListSet {
    SampleSmem* s;
    int n;
    __device__ int size() const { return n; }
    __device__ int idx(int j) const { return s->lidx[j]; }
    __device__ float val(int j) const { return s->lval[j]; }
    __device__ float e(int j) const { return s->le[j]; }
    __device__ void set_e(int j, float x) const { s->le[j] = x; }
};

// What the top-P cut keeps: key > key_star, or key == key_star at a
// position <= tie_last.
struct Cut {
    uint32_t key_star;
    int tie_last;
    __device__ bool keep(uint32_t key, int j) const { return key > key_star || (key == key_star && j <= tie_last); }
};

// topPFilter (transformer.go:1071-1114): walking the keys from the largest,
// the first place where the kept mass reaches P (= top_p x total mass).
template <class Set>
__device__ Cut top_p_cut(const Set& S, double P, SampleSmem& s) {
    const int n = S.size();
    uint32_t prefix = 0, pmask = 0;
    unsigned long long above = 0;
    int ties = 0;
    unsigned long long tie_mass = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (threadIdx.x < 256) {
            s.hc[threadIdx.x] = 0;
            s.hm[threadIdx.x] = 0;
        }
        __syncthreads();
        for (int j = threadIdx.x; j < n; j += kSampleThreads) {
            const uint32_t key = fkey(S.val(j));
            if ((key & pmask) == prefix) {
                const int b = (key >> shift) & 255;
                atomicAdd(&s.hc[b], 1u);
                atomicAdd(&s.hm[b], (unsigned long long)q_of(S.e(j)));
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long acc = above;
            int sel = -1;
            for (int b = 255; b >= 0; b--) {
                if ((double)(acc + s.hm[b]) >= P) { sel = b; break; }
                acc += s.hm[b];
            }
            s.sel = sel;
            s.above = acc;
        }
        __syncthreads();
        const int sel = s.sel;
        if (sel < 0) return Cut{0u, 0x7fffffff};  // the mass never reaches P: keep everything
        above = s.above;
        prefix |= (uint32_t)sel << shift;
        pmask |= 255u << shift;
        ties = (int)s.hc[sel];
        tie_mass = s.hm[sel];
        __syncthreads();
    }
    // equal logits have equal masses: the first m of them (index order) are kept
    const double q = (double)(tie_mass / (unsigned long long)ties);
    long long m = (long long)ceil((P - (double)above) / q);
    if (m < 1) m = 1;
    if (m >= ties) return Cut{prefix, 0x7fffffff};
    if (threadIdx.x < 32) {
        const int l = threadIdx.x;
        int seen = 0, last = 0x7fffffff;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + l;
            const bool f = j < n && fkey(S.val(j)) == prefix;
            const unsigned bal = __ballot_sync(0xffffffffu, f);
            const int c = __popc(bal);
            if (seen + c >= m) {
                // lane of the m-th tie: the (m - seen)-th set bit of bal
                unsigned b = bal;
                for (int t = 1; t < m - seen; t++) b &= b - 1;
                last = j0 + __ffs(b) - 1;
                break;
            }
            seen += c;
        }
        if (l == 0) s.tie_last = last;
    }
    __syncthreads();
    return Cut{prefix, s.tie_last};
}

// The multinomial draw (transformer.go:1027-1035) over the kept masses: the
// first position whose inclusive prefix reaches r x total; the last
// vocabulary index when rounding leaves r above every prefix.
template <class Set>
__device__ int draw(const Set& S, const Cut& cut, float r, int n_vocab, SampleSmem& s) {
    if (!(r > 0.0f)) return 0;  // r <= cum already holds at index 0
    const int n = S.size();
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int seg = (n + kSampleWarps - 1) / kSampleWarps;
    const int b0 = min(n, w * seg), b1 = min(n, b0 + seg);
    unsigned long long sum = 0;
    for (int j = b0 + l; j < b1; j += 32) {
        const float v = S.val(j);
        if (cut.keep(fkey(v), j)) sum += q_of(S.e(j));
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();
    if (l == 0) s.wsum[w] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long tot = 0;
        for (int i = 0; i < kSampleWarps; i++) tot += s.wsum[i];
        const double R = (double)r * (double)tot;
        unsigned long long acc = 0;
        int sel = -1;
        for (int i = 0; i < kSampleWarps; i++) {
            if ((double)(acc + s.wsum[i]) >= R && s.wsum[i] > 0) { sel = i; break; }
            acc += s.wsum[i];
        }
        s.sel = sel;
        s.above = acc;
        s.out = n_vocab - 1;
        s.hm[0] = __double_as_longlong(R);
    }
    __syncthreads();
    if (w == s.sel) {
        const double R = __longlong_as_double((long long)s.hm[0]);
        unsigned long long acc = s.above;
        for (int j0 = b0; j0 < b1; j0 += 32) {
            const int j = j0 + l;
            unsigned long long q = 0;
            if (j < b1) {
                const float v = S.val(j);
                if (cut.keep(fkey(v), j)) q = q_of(S.e(j));
            }
            unsigned long long inc = q;  // inclusive scan across the warp
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
                if (l >= o) inc += t;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, q > 0 && (double)(acc + inc) >= R);
            if (bal) {
                const int ln = __ffs(bal) - 1;
                if (l == ln) s.out = S.idx(j);
                break;
            }
            acc += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
    __syncthreads();
    return s.out;
}



// ---------------------------------------------------------------------------
// The row split over a group of G CTAs (a cooperative launch: all resident).
// CTA g of a row owns the vocabulary slice [g seg, (g + 1) seg); the stages
// over the whole row combine their slices through the row's scratch in
// global memory at group barriers (bounded waits: a barrier that is not met
// within kSampleWaitNs sets the row's error and every CTA returns).

constexpr int kMcMaxG = 160;  // (the group arrays of SampleSmem hold this many)
constexpr int kSliceLogits = 4096;
constexpr uint64_t kSampleWaitNs = 1000000000ull;

struct McRow {
    // zeroed before every launch (the first kMcZeroBytes)
    unsigned bar;
    int err;
    int tie_last;
    unsigned pad_[61];
    unsigned hk[4][256];            // top-K digit counts, one table per round
    unsigned hc[4][256];            // top-P digit counts
    unsigned long long hm[4][256];  // top-P digit masses
    // written before they are read
    float pmax[kMcMaxG];
    int pidx[kMcMaxG];
    int pcnt[kMcMaxG];
    int ptie[kMcMaxG];
    unsigned long long psum_s[kMcMaxG];
    unsigned long long psum_d[kMcMaxG];
    int lidx[kSampleCap];
    float lval[kSampleCap];
};
constexpr size_t kMcZeroBytes = offsetof(McRow, pmax);
constexpr size_t kMcRowBytes = (sizeof(McRow) + 255) & ~size_t(255);

struct Grp {
    McRow* sc;
    int G, g;
    int b0, b1;       // this CTA's slice
    unsigned target;  // barrier arrivals awaited next (thread 0's copy)
};

__device__ bool grp_sync(Grp& G, SampleSmem& s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        G.target += (unsigned)G.G;
        __threadfence();
        atomicAdd(&G.sc->bar, 1u);
        if (ld_acquire(&G.sc->bar) < G.target) {
            const uint64_t t0 = global_ns();
            while (ld_acquire(&G.sc->bar) < G.target) {
                if (*reinterpret_cast<volatile int*>(&G.sc->err)) { ok = 0; break; }
                if (global_ns() - t0 > kSampleWaitNs) {
                    atomicExch(&G.sc->err, 1);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        s.ok = ok;
    }
    __syncthreads();
    return s.ok != 0;
}

// Global tables and per-CTA values are read once, by many threads in
// parallel, into shared memory before one thread walks them (a walk over
// global memory would be a chain of L2 round trips).
__device__ void stage_u32(const unsigned* src, int n, unsigned* dst) {
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kSampleThreads) dst[i] = __ldcg(src + i);
    __syncthreads();
}
__device__ void stage_u64(const unsigned long long* src, int n, unsigned long long* dst) {
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kSampleThreads) dst[i] = __ldcg(src + i);
    __syncthreads();
}

// The digit selection every CTA of the group makes from the same table
// (walking the digits from the largest key): the count form of top-K.
__device__ void select_count(const unsigned* h, int krem, SampleSmem& s) {
    stage_u32(h, 256, s.hc);
    if (threadIdx.x == 0) {
        int c = 0, sel = 0;
        for (int b = 255; b >= 0; b--) {
            if (c + (int)s.hc[b] >= krem) { sel = b; break; }
            c += s.hc[b];
        }
        s.sel = sel;
        s.above = (unsigned long long)c;
    }
    __syncthreads();
}

// topKFilter (transformer.go:1053-1069) over the group: the k-th largest key
// by four rounds of digit counts (each CTA counts its slice in shared memory
// and adds the nonzero bins to the round's table).  *n_keep = keys >= it.
__device__ bool mc_kth_key(Grp& G, const float* L, int k, SampleSmem& s, uint32_t* thr, int* n_keep) {
    uint32_t prefix = 0, pmask = 0;
    int krem = k, greater = 0;
    for (int rd = 0; rd < 4; rd++) {
        const int shift = 24 - 8 * rd;
        if (threadIdx.x < 256) s.hc[threadIdx.x] = 0;
        __syncthreads();
        for (int i = G.b0 + threadIdx.x; i < G.b1; i += kSampleThreads) {
            const uint32_t key = fkey(L[i]);
            if ((key & pmask) == prefix) atomicAdd(&s.hc[(key >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 256 && s.hc[threadIdx.x]) atomicAdd(&G.sc->hk[rd][threadIdx.x], s.hc[threadIdx.x]);
        if (!grp_sync(G, s)) return false;
        select_count(G.sc->hk[rd], krem, s);
        const int sel = s.sel, c = (int)s.above;
        krem -= c;
        greater += c;
        prefix |= (uint32_t)sel << shift;
        pmask |= 255u << shift;
        if (rd == 3) *n_keep = greater + (int)s.hc[sel];
        __syncthreads();
    }
    *thr = prefix;
    return true;
}

// Ordered compaction of the row's keys >= thr into the scratch list (group
// order = vocabulary order): slice counts, a barrier, then each CTA writes
// its survivors at its offset (warp slices within the CTA, as compact_ge).
__device__ bool mc_compact_ge(Grp& G, const float* L, uint32_t thr, SampleSmem& s, int* n_list) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int n = G.b1 - G.b0;
    const int seg = (n + kSampleWarps - 1) / kSampleWarps;
    const int c0 = G.b0 + min(n, w * seg), c1 = G.b0 + min(n, w * seg + seg);
    int cnt = 0;
    for (int i = c0 + l; i < c1; i += 32) cnt += fkey(L[i]) >= thr;
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    __syncthreads();
    if (l == 0) s.wi[w] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int i = 0; i < kSampleWarps; i++) t += s.wi[i];
        G.sc->pcnt[G.g] = t;
    }
    if (!grp_sync(G, s)) return false;
    stage_u32(reinterpret_cast<const unsigned*>(G.sc->pcnt), G.G, reinterpret_cast<unsigned*>(s.gcnt));
    int base = 0, total = 0;
    for (int h = 0; h < G.G; h++) {
        const int c = s.gcnt[h];
        if (h < G.g) base += c;
        total += c;
    }
    for (int i = 0; i < w; i++) base += s.wi[i];
    for (int i0 = c0; i0 < c1; i0 += 32) {
        const int i = i0 + l;
        const float v = i < c1 ? L[i] : -INFINITY;
        const bool f = i < c1 && fkey(v) >= thr;
        const unsigned bal = __ballot_sync(0xffffffffu, f);
        if (f) {
            const int at = base + __popc(bal & ((1u << l) - 1));
            G.sc->lidx[at] = i;
            G.sc->lval[at] = v;
        }
        base += __popc(bal);
    }
    *n_list = total;
    return grp_sync(G, s);
}

// topPFilter (transformer.go:1071-1114) over the group: four rounds of digit
// counts and masses (E = exp(logit - max) of this CTA's slice), every CTA
// making the same selection; a cut inside a run of equal logits keeps the
// first ones in vocabulary order (the tie rank crosses the slices).
__device__ bool mc_top_p_cut(Grp& G, const float* L, const float* E, double P, SampleSmem& s, Cut* cut) {
    uint32_t prefix = 0, pmask = 0;
    unsigned long long above = 0, tie_mass = 0;
    int ties = 0;
    for (int rd = 0; rd < 4; rd++) {
        const int shift = 24 - 8 * rd;
        if (threadIdx.x < 256) {
            s.hc[threadIdx.x] = 0;
            s.hm[threadIdx.x] = 0;
        }
        __syncthreads();
        for (int i = G.b0 + threadIdx.x; i < G.b1; i += kSampleThreads) {
            const uint32_t key = fkey(L[i]);
            if ((key & pmask) == prefix) {
                const int b = (key >> shift) & 255;
                atomicAdd(&s.hc[b], 1u);
                atomicAdd(&s.hm[b], (unsigned long long)q_of(E[i]));
            }
        }
        __syncthreads();
        if (threadIdx.x < 256 && s.hc[threadIdx.x]) {
            atomicAdd(&G.sc->hc[rd][threadIdx.x], s.hc[threadIdx.x]);
            atomicAdd(&G.sc->hm[rd][threadIdx.x], s.hm[threadIdx.x]);
        }
        if (!grp_sync(G, s)) return false;
        stage_u32(G.sc->hc[rd], 256, s.hc);
        stage_u64(G.sc->hm[rd], 256, s.hm);
        if (threadIdx.x == 0) {
            unsigned long long acc = above;
            int sel = -1;
            for (int b = 255; b >= 0; b--) {
                if ((double)(acc + s.hm[b]) >= P) { sel = b; break; }
                acc += s.hm[b];
            }
            s.sel = sel;
            s.above = acc;
        }
        __syncthreads();
        const int sel = s.sel;
        if (sel < 0) {  // the mass never reaches P: keep everything
            *cut = Cut{0u, 0x7fffffff};
            return true;
        }
        above = s.above;
        prefix |= (uint32_t)sel << shift;
        pmask |= 255u << shift;
        ties = (int)s.hc[sel];
        tie_mass = s.hm[sel];
        __syncthreads();
    }
    const double q = (double)(tie_mass / (unsigned long long)ties);
    long long m = (long long)ceil((P - (double)above) / q);
    if (m < 1) m = 1;
    if (m >= ties) {
        *cut = Cut{prefix, 0x7fffffff};
        return true;
    }
    // the m-th tie in vocabulary order: slice counts, then the CTA holding it
    int cnt = 0;
    for (int i = G.b0 + threadIdx.x; i < G.b1; i += kSampleThreads) cnt += fkey(L[i]) == prefix;
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) s.wi[threadIdx.x >> 5] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int i = 0; i < kSampleWarps; i++) t += s.wi[i];
        G.sc->ptie[G.g] = t;
    }
    if (!grp_sync(G, s)) return false;
    stage_u32(reinterpret_cast<const unsigned*>(G.sc->ptie), G.G, reinterpret_cast<unsigned*>(s.gcnt));
    long long before = 0;
    for (int h = 0; h < G.g; h++) before += s.gcnt[h];
    const long long mine = s.gcnt[G.g];
    if (before < m && m <= before + mine && threadIdx.x < 32) {
        const int l = threadIdx.x;
        long long seen = before;
        for (int i0 = G.b0; i0 < G.b1; i0 += 32) {
            const int i = i0 + l;
            const bool f = i < G.b1 && fkey(L[i]) == prefix;
            const unsigned bal = __ballot_sync(0xffffffffu, f);
            const int c = __popc(bal);
            if (seen + c >= m) {
                unsigned b = bal;
                for (long long t = 1; t < m - seen; t++) b &= b - 1;
                if (l == 0) G.sc->tie_last = i0 + __ffs(b) - 1;
                break;
            }
            seen += c;
        }
    }
    if (!grp_sync(G, s)) return false;
    *cut = Cut{prefix, __ldcg(&G.sc->tie_last)};
    return true;
}

// The multinomial draw (transformer.go:1027-1035) over the group: slice sums
// of the kept masses, then the slice (and in it the warp, then the lane)
// where the prefix reaches r x total; the last vocabulary index when
// rounding leaves r above every prefix.  Returns the id in the CTA that
// decides (-2 in the others).
__device__ int mc_draw(Grp& G, const float* L, const float* E, const Cut& cut, float r, int n, SampleSmem& s,
                       bool* ok) {
    *ok = true;
    if (!(r > 0.0f)) return G.g == 0 ? 0 : -2;  // r <= cum already holds at index 0
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    const int len = G.b1 - G.b0;
    const int seg = (len + kSampleWarps - 1) / kSampleWarps;
    const int c0 = G.b0 + min(len, w * seg), c1 = G.b0 + min(len, w * seg + seg);
    unsigned long long sum = 0;
    for (int i = c0 + l; i < c1; i += 32)
        if (cut.keep(fkey(L[i]), i)) sum += q_of(E[i]);
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();
    if (l == 0) s.wsum[w] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long t = 0;
        for (int i = 0; i < kSampleWarps; i++) t += s.wsum[i];
        G.sc->psum_d[G.g] = t;
    }
    if (!grp_sync(G, s)) {
        *ok = false;
        return -2;
    }
    stage_u64(G.sc->psum_d, G.G, s.gsum);
    if (threadIdx.x == 0) {
        unsigned long long tot = 0;
        for (int h = 0; h < G.G; h++) tot += s.gsum[h];
        const double R = (double)r * (double)tot;
        unsigned long long acc = 0;
        int hsel = -1;
        for (int h = 0; h < G.G; h++) {
            const unsigned long long v = s.gsum[h];
            if (v > 0 && (double)(acc + v) >= R) { hsel = h; break; }
            acc += v;
        }
        s.out = -2;
        if (hsel < 0) {
            if (G.g == 0) s.out = n - 1;
            s.sel = -1;
        } else if (hsel == G.g) {
            s.out = n - 1;  // (kept unless the scan below finds the index)
            int wsel = -1;
            for (int i = 0; i < kSampleWarps; i++) {
                if (s.wsum[i] > 0 && (double)(acc + s.wsum[i]) >= R) { wsel = i; break; }
                acc += s.wsum[i];
            }
            s.sel = wsel;
            s.above = acc;
            s.hm[0] = __double_as_longlong(R);
        } else {
            s.sel = -1;
        }
    }
    __syncthreads();
    if (w == s.sel) {
        const double R = __longlong_as_double((long long)s.hm[0]);
        unsigned long long acc = s.above;
        for (int i0 = c0; i0 < c1; i0 += 32) {
            const int i = i0 + l;
            unsigned long long q = 0;
            if (i < c1 && cut.keep(fkey(L[i]), i)) q = q_of(E[i]);
            unsigned long long inc = q;
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
                if (l >= o) inc += t;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, q > 0 && (double)(acc + inc) >= R);
            if (bal) {
                if (l == __ffs(bal) - 1) s.out = i;
                break;
            }
            acc += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
    __syncthreads();
    return s.out;
}

// First maximum (transformer.go:1038-1046 argmax) of the slice [b0, b1):
// the largest value, the smallest index among equals; (value, index) to
// thread 0.
__device__ void slice_argmax(const float* L, int b0, int b1, SampleSmem& s, float* bv_out, int* bi_out) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    float bv = -INFINITY;
    int bi = -1;
    for (int i = b0 + threadIdx.x; i < b1; i += kSampleThreads) {
        const float v = L[i];
        if (bi < 0 || v > bv) { bv = v; bi = i; }  // ascending i: only a larger value replaces
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    __syncthreads();
    if (l == 0) { s.wf[w] = bv; s.wi[w] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        bv = s.wf[0];
        bi = s.wi[0];
        for (int i = 1; i < kSampleWarps; i++)
            if (s.wi[i] >= 0 && (bi < 0 || s.wf[i] > bv || (s.wf[i] == bv && s.wi[i] < bi))) { bv = s.wf[i]; bi = s.wi[i]; }
        *bv_out = bv;
        *bi_out = bi;
    }
}

// Top-P and the draw over the top-K survivors, in one CTA (shared memory).
__device__ int list_filter_and_draw(int nl, float mx, const SampleArgs& a, float r, SampleSmem& s) {
    const ListSet S{&s, nl};
    for (int j = threadIdx.x; j < nl; j += kSampleThreads) S.set_e(j, e_of(S.val(j), mx));
    __syncthreads();  // (exp(logit - max) against the row's maximum: top-K keeps it)
    Cut cut{0u, 0x7fffffff};
    if (a.top_p > 0.0f && a.top_p < 1.0f) {
        unsigned long long tot = 0;
        for (int j = threadIdx.x; j < nl; j += kSampleThreads) tot += q_of(S.e(j));
        tot = block_sum_u64(tot, s);
        cut = top_p_cut(S, (double)a.top_p * (double)tot, s);
    }
    return draw(S, cut, r, a.n, s);
}

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(const __grid_constant__ SampleArgs a) {
    extern __shared__ __align__(16) uint8_t ssm_raw[];
    SampleSmem& s = *reinterpret_cast<SampleSmem*>(ssm_raw);
    const int G = a.group, row = blockIdx.x / G, g = blockIdx.x % G, n = a.n;
    const int seg = (n + G - 1) / G;
    McRow* sc = reinterpret_cast<McRow*>(a.scratch + (size_t)row * kMcRowBytes);
    float* E = reinterpret_cast<float*>(a.scratch + (size_t)a.rows * kMcRowBytes) + (size_t)row * a.e_ld;
    Grp grp{sc, G, g, min(n, g * seg), min(n, g * seg + seg), 0u};
    float* L = a.logits + (long long)row * a.ld;
    const int ng = a.ngen[row];
    // transformer.go:984-999: the penalty, once per occurrence in order (each
    // CTA for the ids in its slice)
    if (a.pen > 1.0f && ng > 0 && a.gen && threadIdx.x == 0) {
        const int32_t* gl = a.gen + (long long)row * a.gen_ld;
        for (int i = 0; i < ng; i++) {
            const int t = gl[i];
            if (t >= grp.b0 && t < grp.b1) {
                const float v = L[t];
                L[t] = v > 0.0f ? v / a.pen : v * a.pen;
            }
        }
    }
    __syncthreads();
    int id = -2;
    bool ok = true;
    if (a.greedy) {
        float bv;
        int bi;
        slice_argmax(L, grp.b0, grp.b1, s, &bv, &bi);
        if (threadIdx.x == 0) {
            sc->pmax[g] = bv;
            sc->pidx[g] = bi;
        }
        ok = grp_sync(grp, s);
        if (ok && g == 0) {
            stage_u32(reinterpret_cast<const unsigned*>(sc->pmax), G, reinterpret_cast<unsigned*>(s.gmax));
            stage_u32(reinterpret_cast<const unsigned*>(sc->pidx), G, reinterpret_cast<unsigned*>(s.gcnt));
            if (threadIdx.x == 0) {
                int best = -1;
                float v = -INFINITY;
                for (int h = 0; h < G; h++)  // slices in vocabulary order: a later one wins only if larger
                    if (s.gcnt[h] >= 0 && (best < 0 || s.gmax[h] > v)) { v = s.gmax[h]; best = s.gcnt[h]; }
                id = best < 0 ? 0 : best;
            }
        }
    } else {
        float mx = -INFINITY;
        for (int i = grp.b0 + threadIdx.x; i < grp.b1; i += kSampleThreads) {
            const float v = L[i] / a.temp;
            L[i] = v;
            mx = fmaxf(mx, v);
        }
        mx = block_max(mx, s);
        if (threadIdx.x == 0) sc->pmax[g] = mx;
        ok = grp_sync(grp, s);
        if (ok) {
            stage_u32(reinterpret_cast<const unsigned*>(sc->pmax), G, reinterpret_cast<unsigned*>(s.gmax));
            mx = -INFINITY;
            for (int h = 0; h < G; h++) mx = fmaxf(mx, s.gmax[h]);
        }
        bool full = true;
        if (ok && a.top_k > 0 && a.top_k < n) {
            uint32_t thr = 0;
            int n_keep = 0;
            ok = mc_kth_key(grp, L, a.top_k, s, &thr, &n_keep);
            if (ok && n_keep <= kSampleCap) {
                int nl = 0;
                ok = mc_compact_ge(grp, L, thr, s, &nl);
                full = false;
                if (ok && g == 0) {
                    for (int j = threadIdx.x; j < nl; j += kSampleThreads) {
                        s.lidx[j] = __ldcg(&sc->lidx[j]);
                        s.lval[j] = __ldcg(&sc->lval[j]);
                    }
                    __syncthreads();
                    id = list_filter_and_draw(nl, mx, a, a.r[row], s);
                }
            } else if (ok) {
                for (int i = grp.b0 + threadIdx.x; i < grp.b1; i += kSampleThreads)
                    if (fkey(L[i]) < thr) L[i] = -INFINITY;
            }
        }
        if (ok && full) {
            unsigned long long tot = 0;
            for (int i = grp.b0 + threadIdx.x; i < grp.b1; i += kSampleThreads) {
                const float e = e_of(L[i], mx);
                E[i] = e;
                tot += q_of(e);
            }
            tot = block_sum_u64(tot, s);
            Cut cut{0u, 0x7fffffff};
            if (a.top_p > 0.0f && a.top_p < 1.0f) {
                if (threadIdx.x == 0) sc->psum_s[g] = tot;
                ok = grp_sync(grp, s);
                if (ok) {
                    stage_u64(sc->psum_s, G, s.gsum);
                    tot = 0;
                    for (int h = 0; h < G; h++) tot += s.gsum[h];
                    ok = mc_top_p_cut(grp, L, E, (double)a.top_p * (double)tot, s, &cut);
                }
            }
            if (ok) id = mc_draw(grp, L, E, cut, a.r[row], n, s, &ok);
        }
    }
    if (threadIdx.x == 0) {
        if (!ok) {
            if (g == 0) a.out[row] = -1;
            if (a.err) atomicCAS(a.err, 0, B2_ERR_TIMEOUT);
        } else if (id >= 0) {
            a.out[row] = id;
            if (a.gen_append && ng < a.gen_cap) a.gen_append[(long long)row * a.gen_ld + ng] = id;
        }
    }
}

}  // namespace

size_t sample_scratch_bytes(int n, int rows) {
    return (size_t)rows * (kMcRowBytes + (((size_t)n * 4 + 255) & ~size_t(255)));
}

int launch_sample(const SampleArgs& a0, int rows, cudaStream_t s, std::string* err) {
    if (rows <= 0 || rows > kSampleMaxRows || a0.n <= 0 || !a0.logits || !a0.out || !a0.scratch || a0.ld < a0.n ||
        (!a0.greedy && !(a0.temp > 0.0f))) {
        *err = "sample: bad arguments";
        return B2_ERR_BAD_ARG;
    }
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) ||
        cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SampleSmem)) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sample_kernel, kSampleThreads, sizeof(SampleSmem)) !=
            cudaSuccess ||
        per_sm < 1) {
        *err = "sample: device query failed";
        return B2_ERR_CUDA;
    }
    SampleArgs a = a0;
    a.rows = rows;
    // about 4096 logits a CTA: a group barrier costs more with every CTA it
    // waits for, and a slice that small is a few loads per thread
    a.group = std::max(1, std::min({kMcMaxG, sms * per_sm / rows, (a.n + kSliceLogits - 1) / kSliceLogits}));
    a.e_ld = (long long)((((size_t)a.n * 4 + 255) & ~size_t(255)) / 4);
    // the rows' barrier counters and digit tables start from zero
    for (int r = 0; r < rows; r++)
        if (cudaMemsetAsync(a.scratch + (size_t)r * kMcRowBytes, 0, kMcZeroBytes, s) != cudaSuccess) {
            *err = "sample: scratch reset failed";
            return B2_ERR_CUDA;
        }
    void* args[] = {&a};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(sample_kernel), dim3(rows * a.group),
                                                      dim3(kSampleThreads), args, sizeof(SampleSmem), s);
    if (e != cudaSuccess) {
        *err = std::string("sample: ") + cudaGetErrorString(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

}  // namespace b2
