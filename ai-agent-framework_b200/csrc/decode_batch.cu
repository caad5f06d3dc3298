// Batched greedy decode: up to 16 sequences advance one token per step
// together, each at its own position in a KV cache of its own, so a step
// reads every weight byte once for all of them (transformer.go:519-739, the
// forward of one new token, for B sequences at a time; argmax
// transformer.go:1038-1046).
//
// A step (and each prompt chunk of a slot's prefill) is a sequence of
// launches on the model's stream:
//   embedding rows of the B tokens (the tiled token_embd, decoded on the fly)
//   per layer: RMSNorm -> batched tile dot over [Wq; Wk; Wv] -> bias, RoPE
//   and the KV append at each sequence's position -> attention over each
//   sequence's own length -> Wo tile dot -> residual add -> RMSNorm ->
//   gate/up tile dot (interleaved 8 rows at a time) -> SwiGLU -> down tile dot
//   -> residual add
//   final RMSNorm -> lm_head tile dot -> argmax per sequence (first maximum).
// When every width is a multiple of 64 the products run on the tcgen05
// tensor-core GEMM (gemm_tc.cu) and the norms, RoPE and SwiGLU are fused
// into the kernels between them (forward_rows_tc); otherwise the tile dots
// are the batched matvec over the resident tiled weights (matvec_batch.cu).
// A slot's prompt runs through the same launches in chunks of up to
// kPrefillChunk of its tokens.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <string>
#include <vector>

#include "../../include/b2decode.h"
#include "dev.cuh"
#include "gemm.h"
#include "model.h"

int b2_tiled_matvec_batch_impl(int qtype, const void* base, int64_t rp, int64_t row0, int rows, int cols,
                               const float* x, float* y, int nvec, cudaStream_t s, std::string* err);
unsigned long long b2_mvb_scratch_generation(cudaStream_t s);
int b2_attention_seqs_launch(const float* q, const __half* k, const __half* v, float* part, size_t part_floats,
                             float* out, int batch, int nh, int nkv, int hd, const int* lens, int add, int stride,
                             int max_len, int sms, cudaStream_t s);

constexpr int kBatchMax = 16;
constexpr int kPrefillChunk = 256;  // prompt tokens per weight pass of a prefill (tensor-core GEMM)
constexpr int kBatchSplits = 32;    // attention splits the partial buffer holds (for kBatchMax rows)

struct b2_batch {
    b2_model* m = nullptr;
    int B = 0;
    int max_seq = 0;
    bool model_cache = false;  // kc / vc are the model's own cache (the prompt-prefill workspace)
    void* arena = nullptr;
    __half* kc = nullptr;  // [L][B][max_seq][kvd]
    __half* vc = nullptr;
    float *x = nullptr, *xn = nullptr, *y = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr;
    float *gu = nullptr, *act = nullptr, *logits = nullptr, *part = nullptr;
    __half* xh = nullptr;   // [kPrefillChunk + 16][max(H, FF)]: a product's input in the GEMM's fp16 form
    float* tsc = nullptr;   // [kPrefillChunk + 16] its per-token scales
    int xh_ld = 0;
    size_t part_floats = 0;
    int *d_pos = nullptr, *d_tok = nullptr, *d_next = nullptr;  // [kBatchMax]
    int* d_ppos = nullptr;                                      // [kBatchMax] prefill chunk positions
    float* arg_v = nullptr;                                     // [kBatchMax][kArgParts] argmax parts
    int* arg_i = nullptr;
    int* h_io = nullptr;                                        // pinned [3 * kBatchMax]
    std::vector<int> pos;                                       // positions (host copy)
    bool use_graph = false;                  // replay steps from a captured CUDA graph
    cudaGraphExec_t exec = nullptr;          // the step's launches (tokens and ids copied outside)
    unsigned long long exec_gen = 0;         // scratch generation it captured (scratch_generation)
};

namespace b2 {
namespace {

constexpr int kBdThreads = 256;

// Row `tok` of the tiled embedding (gguf.go:540-582 dequant, Q4_0 in the
// ggml element order); an id outside the vocabulary embeds to zero.
__global__ void bd_embed_kernel(const uint8_t* __restrict__ emb, int V, int64_t rp, int H, int qt,
                                const int* __restrict__ tok, float* __restrict__ x) {
    const int b = blockIdx.x, t = tok[b];
    const int64_t nb = H / 32;
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        float v = 0.0f;
        if (t >= 0 && t < V) {
            const int64_t blk = j >> 5;
            const int e = j & 31;
            const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(emb + tiled_soff(t, blk, nb, rp, qt)));
            if (qt == 8) {
                v = d * (float)(int8_t)emb[tiled_qoff(t, blk, e, nb, 8)];
            } else {
                const uint8_t byte = emb[tiled_qoff(t, blk, e & 15, nb, 2)];
                v = d * (float)(((e < 16) ? (byte & 15) : (byte >> 4)) - 8);
            }
        }
        x[(size_t)b * H + j] = v;
    }
}

// transformer.go:922-932 rmsNorm of each sequence's row: x * r * w with
// r = 1 / sqrt(mean(x^2) + eps) (the root in double, as the Go code).  One
// CTA of kNormThreads per row, the row read once (float4, kept in registers);
// H a multiple of 4 (the batched path needs H % 64 == 0 for its products).
constexpr int kNormThreads = 512;
constexpr int kNormVec = 4;  // float4 per thread in the single pass: H up to 8192
__global__ void __launch_bounds__(kNormThreads) bd_rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                                   float* __restrict__ out, int H, float eps) {
    __shared__ float red[kNormThreads / 32];
    __shared__ float rs;
    const int b = blockIdx.x, n4 = H / 4;
    const float4* xb = reinterpret_cast<const float4*>(x + (size_t)b * H);
    const float4* wv = reinterpret_cast<const float4*>(w);
    float4* ob = reinterpret_cast<float4*>(out + (size_t)b * H);
    float4 v[kNormVec];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < kNormVec; k++) {
        const int i = threadIdx.x + k * kNormThreads;
        v[k] = i < n4 ? xb[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        ss = fmaf(v[k].x, v[k].x, fmaf(v[k].y, v[k].y, fmaf(v[k].z, v[k].z, fmaf(v[k].w, v[k].w, ss))));
    }
    for (int i = threadIdx.x + kNormVec * kNormThreads; i < n4; i += kNormThreads) {
        const float4 u = xb[i];
        ss = fmaf(u.x, u.x, fmaf(u.y, u.y, fmaf(u.z, u.z, fmaf(u.w, u.w, ss))));
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < kNormThreads / 32; i++) t += red[i];
        rs = (float)(1.0 / sqrt((double)(t / (float)H) + (double)eps));
    }
    __syncthreads();
    const float r = rs;
#pragma unroll
    for (int k = 0; k < kNormVec; k++) {
        const int i = threadIdx.x + k * kNormThreads;
        if (i < n4) {
            const float4 g = __ldg(wv + i);
            ob[i] = make_float4(v[k].x * r * g.x, v[k].y * r * g.y, v[k].z * r * g.z, v[k].w * r * g.w);
        }
    }
    for (int i = threadIdx.x + kNormVec * kNormThreads; i < n4; i += kNormThreads) {
        const float4 u = xb[i], g = __ldg(wv + i);
        ob[i] = make_float4(u.x * r * g.x, u.y * r * g.y, u.z * r * g.z, u.w * r * g.w);
    }
}

// Split-K partial planes summed in plane order: the k (<= kMaxPlanes) loads
// are issued together (predicated, unrolled) so they overlap in flight.
constexpr int kMaxPlanes = 8;
__device__ __forceinline__ float4 sum_planes4(const float* p, size_t plane, int k) {
    float4 v[kMaxPlanes];
#pragma unroll
    for (int s = 0; s < kMaxPlanes; s++)
        if (s < k) v[s] = __ldcg(reinterpret_cast<const float4*>(p + s * plane));
    float4 r = v[0];
#pragma unroll
    for (int s = 1; s < kMaxPlanes; s++)
        if (s < k) {
            r.x += v[s].x; r.y += v[s].y; r.z += v[s].z; r.w += v[s].w;
        }
    return r;
}
__device__ __forceinline__ float2 sum_planes2(const float* p, size_t plane, int k) {
    float2 v[kMaxPlanes];
#pragma unroll
    for (int s = 0; s < kMaxPlanes; s++)
        if (s < k) v[s] = __ldcg(reinterpret_cast<const float2*>(p + s * plane));
    float2 r = v[0];
#pragma unroll
    for (int s = 1; s < kMaxPlanes; s++)
        if (s < k) {
            r.x += v[s].x; r.y += v[s].y;
        }
    return r;
}

// The GEMM's input form of one token's row (gemm.h): scaled by 2^e so the
// largest magnitude lies in [2^14, 2^15), fp16, scale 2^-e.
__device__ __forceinline__ void st_f16x4(__half* p, float4 v, float up) {
    const __half2 a = __floats2half2_rn(v.x * up, v.y * up), b = __floats2half2_rn(v.z * up, v.w * up);
    *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

// The residual update and the next RMSNorm in one pass: x += the split-K
// partials of the product that ends the sub-block (k planes, summed in
// plane order, then added: as a separate sum and add would), then
// transformer.go:922-932 rmsNorm of the new x written in the GEMM's input
// form (xh row, scale) for the next product, and as fp32 into xn when xn is
// given.  Each row is spread over a cluster of kRowCtas CTAs (one slice
// each); the row's sum of squares and largest magnitude are combined over
// the cluster through distributed shared memory (every CTA reads every
// partial in rank order, so all agree).  Grid R * kRowCtas; H a multiple of
// 4 kRowCtas, at most 4 kRowCtas kRowThreads kAddVec.
namespace cg = cooperative_groups;
constexpr int kRowCtas = 8;
constexpr int kRowThreads = 128;
constexpr int kAddVec = 4;  // float4 per thread

__device__ float cluster_sum_ranked(cg::cluster_group& cl, float* mine, float v) {
    // v: this CTA's partial (thread 0 writes it); the cluster's sum in rank order
    if (threadIdx.x == 0) *mine = v;
    cl.sync();
    float t = 0.0f;
    for (int r = 0; r < kRowCtas; r++) t += *cl.map_shared_rank(mine, r);
    return t;
}
__device__ float cluster_max_ranked(cg::cluster_group& cl, float* mine, float v) {
    if (threadIdx.x == 0) *mine = v;
    cl.sync();
    float t = 0.0f;
    for (int r = 0; r < kRowCtas; r++) t = fmaxf(t, *cl.map_shared_rank(mine, r));
    return t;
}
__device__ float block_sum128(float v, float* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = 0.0f;
#pragma unroll
    for (int i = 0; i < kRowThreads / 32; i++) v += red[i];
    return v;
}
__device__ float block_max128(float v, float* red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[0];
#pragma unroll
    for (int i = 1; i < kRowThreads / 32; i++) v = fmaxf(v, red[i]);
    return v;
}

__global__ void __cluster_dims__(kRowCtas, 1, 1) __launch_bounds__(kRowThreads)
    bd_add_norm_f16_kernel(float* __restrict__ x, const float* __restrict__ part, int k, size_t plane,
                              const float* __restrict__ w, int H, float eps, __half* __restrict__ xh, int xh_ld,
                              float* __restrict__ tsc, float* __restrict__ xn) {
    __shared__ float red[kRowThreads / 32];
    __shared__ float c_ss, c_mx;
    pdl_trigger();
    pdl_wait();
    cg::cluster_group cl = cg::this_cluster();
    const int b = blockIdx.x / kRowCtas, c = (int)cl.block_rank();
    const int n4 = H / 4 / kRowCtas;  // float4 of this CTA's slice
    float4* xb = reinterpret_cast<float4*>(x + (size_t)b * H);
    float4 u[kAddVec];
    float ss = 0.0f;
#pragma unroll
    for (int v = 0; v < kAddVec; v++) {
        const int t = threadIdx.x + v * kRowThreads, i = c * n4 + t;
        u[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t < n4) {
            u[v] = xb[i];
            if (k > 0) {
                const float4 s = sum_planes4(part + (size_t)b * H + 4 * i, plane, k);
                u[v].x += s.x; u[v].y += s.y; u[v].z += s.z; u[v].w += s.w;
                xb[i] = u[v];
            }
        }
        ss = fmaf(u[v].x, u[v].x, fmaf(u[v].y, u[v].y, fmaf(u[v].z, u[v].z, fmaf(u[v].w, u[v].w, ss))));
    }
    ss = cluster_sum_ranked(cl, &c_ss, block_sum128(ss, red));
    const float r = (float)(1.0 / sqrt((double)(ss / (float)H) + (double)eps));
    float mx = 0.0f;
#pragma unroll
    for (int v = 0; v < kAddVec; v++) {
        const int t = threadIdx.x + v * kRowThreads, i = c * n4 + t;
        if (t < n4) {
            const float4 gg = __ldg(reinterpret_cast<const float4*>(w) + i);
            u[v] = make_float4(u[v].x * r * gg.x, u[v].y * r * gg.y, u[v].z * r * gg.z, u[v].w * r * gg.w);
            if (xn) reinterpret_cast<float4*>(xn + (size_t)b * H)[i] = u[v];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(u[v].x), fabsf(u[v].y)), fmaxf(fabsf(u[v].z), fabsf(u[v].w))));
        }
    }
    mx = cluster_max_ranked(cl, &c_mx, block_max128(mx, red));
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
        int ex;
        frexpf(mx, &ex);
        e = 15 - ex;
    }
    if (c == 0 && threadIdx.x == 0) tsc[b] = ldexpf(1.0f, -e);
    const float up = ldexpf(1.0f, e);
#pragma unroll
    for (int v = 0; v < kAddVec; v++) {
        const int t = threadIdx.x + v * kRowThreads, i = c * n4 + t;
        if (t < n4) st_f16x4(xh + (size_t)b * xh_ld + 4 * i, u[v], up);
    }
    cl.sync();  // no CTA leaves while another may still read its shared memory
}

// transformer.go:725-727, 954-956 SwiGLU over the split-K partials of the
// interleaved gate/up product (output j of tile t: gate at row 16t + j % 8,
// up 8 rows below), written in the GEMM's input form for the down product.
// Each row is spread over a cluster of kRowCtas CTAs (CTA c: outputs
// c FF / kRowCtas onwards, consecutive lanes on consecutive outputs; all of
// a thread's loads issued before any is used); the row's largest magnitude
// through distributed shared memory.  FF a multiple of 8 kRowCtas, at most
// kRowCtas kRowThreads kSwClVec.
constexpr int kSwClVec = 16;
__global__ void __cluster_dims__(kRowCtas, 1, 1) __launch_bounds__(kRowThreads)
    bd_swiglu_f16_kernel(const float* __restrict__ part, int k, size_t plane, int FF, __half* __restrict__ xh,
                            int xh_ld, float* __restrict__ tsc) {
    __shared__ float red[kRowThreads / 32];
    __shared__ float c_mx;
    pdl_trigger();
    pdl_wait();
    cg::cluster_group cl = cg::this_cluster();
    const int b = blockIdx.x / kRowCtas, c = (int)cl.block_rank();
    const float* row = part + (size_t)b * 2 * FF;
    const int per = FF / kRowCtas;  // this CTA's outputs: c per .. (c + 1) per - 1
    float gv[kSwClVec], uv[kSwClVec];
#pragma unroll
    for (int kk = 0; kk < kSwClVec; kk++) {
        const int jj = kk * kRowThreads + threadIdx.x, j = c * per + jj;
        const size_t o = (size_t)(j >> 3) * 16 + (j & 7);
        gv[kk] = jj < per ? __ldcg(row + o) : 0.0f;
        uv[kk] = jj < per ? __ldcg(row + o + 8) : 0.0f;
    }
    for (int s = 1; s < k; s++) {
#pragma unroll
        for (int kk = 0; kk < kSwClVec; kk++) {
            const int jj = kk * kRowThreads + threadIdx.x, j = c * per + jj;
            const size_t o = s * plane + (size_t)(j >> 3) * 16 + (j & 7);
            if (jj < per) {
                gv[kk] += __ldcg(row + o);
                uv[kk] += __ldcg(row + o + 8);
            }
        }
    }
    float mx = 0.0f;
#pragma unroll
    for (int kk = 0; kk < kSwClVec; kk++) {
        const int jj = kk * kRowThreads + threadIdx.x, j = c * per + jj;
        gv[kk] = jj < per ? gv[kk] / (1.0f + expf(-gv[kk])) * uv[kk] : 0.0f;
        mx = fmaxf(mx, fabsf(gv[kk]));
    }
    mx = cluster_max_ranked(cl, &c_mx, block_max128(mx, red));
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
        int ex;
        frexpf(mx, &ex);
        e = 15 - ex;
    }
    const float up = ldexpf(1.0f, e);
    if (c == 0 && threadIdx.x == 0) tsc[b] = ldexpf(1.0f, -e);
#pragma unroll
    for (int kk = 0; kk < kSwClVec; kk++) {
        const int jj = kk * kRowThreads + threadIdx.x, j = c * per + jj;
        if (jj < per) xh[(size_t)b * xh_ld + j] = __float2half_rn(gv[kk] * up);
    }
    cl.sync();  // no CTA leaves while another may still read its shared memory
}

// transformer.go:632-656: bias, RoPE on interleaved pairs of every q and k
// head at the row's position (936-951, the model's cos / sin table), then k
// and v appended to the row's cache slot (rows slot_stride positions apart;
// 0 when all rows are tokens of one sequence); q kept for attention.
// The q / k / v rows are the sum of k split-K planes (plane floats apart).
__global__ void bd_rope_kv_kernel(const float* __restrict__ qkv, int k, size_t plane, const float* __restrict__ bias,
                                  const float* __restrict__ cosT, const float* __restrict__ sinT,
                                  const int* __restrict__ pos, float* __restrict__ q, __half* __restrict__ kc,
                                  __half* __restrict__ vc, int qd, int kvd, int hd, int slot_stride) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, p = pos[b], n = qd + 2 * kvd, hh = hd / 2;
    const float* row = qkv + (size_t)b * n;
    for (int j = blockIdx.y * blockDim.x + threadIdx.x; j < n / 2; j += gridDim.y * blockDim.x) {
        const int r = 2 * j;
        const float2 a = sum_planes2(row + r, plane, k);
        float a0 = a.x, a1 = a.y;
        if (bias) {
            a0 += bias[r];
            a1 += bias[r + 1];
        }
        if (r < qd + kvd) {
            const int pi2 = (r % hd) >> 1;
            const float c = cosT[(size_t)p * hh + pi2], s = sinT[(size_t)p * hh + pi2];
            const float x0 = a0, x1 = a1;
            a0 = x0 * c - x1 * s;
            a1 = x0 * s + x1 * c;
        }
        if (r < qd) {
            q[(size_t)b * qd + r] = a0;
            q[(size_t)b * qd + r + 1] = a1;
        } else {
            const bool isk = r < qd + kvd;
            const int col = r - qd - (isk ? 0 : kvd);
            __half* cache = isk ? kc : vc;
            *reinterpret_cast<__half2*>(cache + ((size_t)b * slot_stride + p) * kvd + col) =
                __floats2half2_rn(a0, a1);
        }
    }
}

__global__ void bd_add_kernel(float* __restrict__ x, const float* __restrict__ y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] += y[i];
}

// transformer.go:725-727, 954-956 SwiGLU over the interleaved gate/up
// output: output j of tile t has its gate at row 16t + j % 8, its up 8 rows
// below.
__global__ void bd_swiglu_kernel(const float* __restrict__ gu, float* __restrict__ act, int FF, int B) {
    const int n = B * FF;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int b = i / FF, j = i - b * FF;
        const float* g = gu + (size_t)b * 2 * FF + (size_t)(j >> 3) * 16 + (j & 7);
        const float gv = g[0], uv = g[8];
        act[i] = gv / (1.0f + expf(-gv)) * uv;
    }
}

// transformer.go:1038-1046 argmax per sequence (the first maximum wins), in
// two levels: kArgParts CTAs per row each keep the best (value, index) of
// their slice, then one warp per row takes the best of the parts (the lowest
// index among equal values, as a left-to-right scan does); then the row's
// position moves past the token just appended.
constexpr int kArgParts = 32;
__global__ void bd_argmax_part_kernel(const float* __restrict__ logits, int V, float* __restrict__ pv,
                                      int* __restrict__ pi) {
    __shared__ float bv[kBdThreads / 32];
    __shared__ int bi[kBdThreads / 32];
    const int b = blockIdx.x / kArgParts, part = blockIdx.x % kArgParts;
    const int j0 = (int)((long long)part * V / kArgParts), j1 = (int)((long long)(part + 1) * V / kArgParts);
    const float* lb = logits + (size_t)b * V;
    float best = -INFINITY;
    int idx = V;
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x)
        if (lb[j] > best) {
            best = lb[j];
            idx = j;
        }
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (v2 > best || (v2 == best && i2 < idx)) {
            best = v2;
            idx = i2;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        bv[threadIdx.x >> 5] = best;
        bi[threadIdx.x >> 5] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kBdThreads / 32; w++)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        // (bv[0], bi[0] is thread 0's own warp result: already in best / idx)
        pv[blockIdx.x] = best;
        pi[blockIdx.x] = idx;
    }
}
__global__ void bd_argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int V,
                                       int* __restrict__ next, int* __restrict__ pos) {
    const int b = blockIdx.x, lane = threadIdx.x;
    float best = lane < kArgParts ? pv[b * kArgParts + lane] : -INFINITY;
    int idx = lane < kArgParts ? pi[b * kArgParts + lane] : V;
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (v2 > best || (v2 == best && i2 < idx)) {
            best = v2;
            idx = i2;
        }
    }
    if (lane == 0) {
        next[b] = idx < V ? idx : 0;
        pos[b] += 1;
    }
}

// positions p0 .. p0 + n - 1 of a prefill chunk
__global__ void bd_iota_kernel(int* __restrict__ pos, int n, int p0) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) pos[i] = p0 + i;
}

bool ok(cudaError_t e, std::string* err, const char* what) {
    if (e == cudaSuccess) return true;
    *err = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
}

}  // namespace
}  // namespace b2

using namespace b2;

namespace {
int batch_create(b2_model* m, int B, bool model_cache, b2_batch** out, std::string* err);
}

int b2_batch_create_impl(b2_model* m, int B, b2_batch** out, std::string* err) {
    return batch_create(m, B, false, out, err);
}

namespace {

// A batch of B slots with KV caches of their own, or (model_cache) one row
// set over the model's own cache: the workspace of the model's prompt
// prefill on the tensor cores.
int batch_create(b2_model* m, int B, bool model_cache, b2_batch** out, std::string* err) {
    const ModelDev& d = m->dev;
    if (B < 1 || B > kBatchMax) {
        *err = "batch size must be 1 to 16";
        return B2_ERR_BAD_ARG;
    }
    if (d.tp > 1 || d.kv_fp32) {
        *err = "batched decode needs a single-GPU model with the fp16 KV cache";
        return B2_ERR_BAD_ARG;
    }
    if ((d.hd != 64 && d.hd != 128 && d.hd != 256) || d.nh / d.nkv > 8) {
        *err = "batched decode attention needs head_dim 64, 128 or 256 and at most 8 query heads per KV head";
        return B2_ERR_UNSUPPORTED_TYPE;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != m->device) {
        *err = "the model's device must be the current device";
        return B2_ERR_BAD_ARG;
    }
    b2_batch* bt = new b2_batch;
    bt->m = m;
    bt->B = B;
    bt->max_seq = d.max_seq;
    bt->model_cache = model_cache;
    bt->pos.assign(B, 0);
    const size_t kv = model_cache ? 0 : (size_t)d.L * B * d.max_seq * d.kvd;
    const int n_qkv = d.qd + 2 * d.kvd;
    // activations for R rows: the B slots of a step, or up to kPrefillChunk
    // tokens of one sequence in a prefill chunk (whose lm_head runs for its
    // last token only, so the logits hold kBatchMax rows)
    const size_t R = std::max(kBatchMax, kPrefillChunk);
    bt->part_floats = (size_t)kBatchMax * d.nh * kBatchSplits * (d.hd + 2);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) & ~size_t(255);
        return o;
    };
    const size_t o_kc = take(kv * 2), o_vc = take(kv * 2);
    const size_t o_x = take(R * d.H * 4), o_xn = take(R * d.H * 4), o_y = take(R * d.H * 4);
    const size_t o_qkv = take(R * n_qkv * 4), o_q = take(R * d.qd * 4);
    const size_t o_att = take(R * d.qd * 4);
    const size_t o_gu = take(R * 2 * d.FF * 4), o_act = take(R * d.FF * 4);
    const size_t o_lg = take((size_t)kBatchMax * d.V * 4), o_part = take(bt->part_floats * 4);
    const size_t o_pos = take(R * 4), o_tok = take(R * 4), o_next = take(R * 4), o_ppos = take(R * 4);
    const size_t o_argv = take((size_t)kBatchMax * kArgParts * 4), o_argi = take((size_t)kBatchMax * kArgParts * 4);
    // (rows past a pass's tokens are read by the GEMM's last N tile, never used)
    const int xh_rows = kPrefillChunk + 16, xh_ld = std::max(d.H, d.FF);
    const size_t o_xh = take((size_t)xh_rows * xh_ld * 2), o_tsc = take((size_t)xh_rows * 4);
    if (cudaMalloc(&bt->arena, off) != cudaSuccess) {
        delete bt;
        *err = "device allocation of the batch state failed";
        return B2_ERR_OOM;
    }
    if (cudaMallocHost(&bt->h_io, sizeof(int) * 3 * kBatchMax) != cudaSuccess) {
        cudaFree(bt->arena);
        delete bt;
        *err = "pinned host allocation failed";
        return B2_ERR_OOM;
    }
    uint8_t* A = static_cast<uint8_t*>(bt->arena);
    bt->kc = model_cache ? static_cast<__half*>(d.kcache) : reinterpret_cast<__half*>(A + o_kc);
    bt->vc = model_cache ? static_cast<__half*>(d.vcache) : reinterpret_cast<__half*>(A + o_vc);
    bt->x = reinterpret_cast<float*>(A + o_x);
    bt->xn = reinterpret_cast<float*>(A + o_xn);
    bt->y = reinterpret_cast<float*>(A + o_y);
    bt->qkv = reinterpret_cast<float*>(A + o_qkv);
    bt->q = reinterpret_cast<float*>(A + o_q);
    bt->att = reinterpret_cast<float*>(A + o_att);
    bt->gu = reinterpret_cast<float*>(A + o_gu);
    bt->act = reinterpret_cast<float*>(A + o_act);
    bt->logits = reinterpret_cast<float*>(A + o_lg);
    bt->part = reinterpret_cast<float*>(A + o_part);
    bt->d_pos = reinterpret_cast<int*>(A + o_pos);
    bt->d_tok = reinterpret_cast<int*>(A + o_tok);
    bt->d_next = reinterpret_cast<int*>(A + o_next);
    bt->d_ppos = reinterpret_cast<int*>(A + o_ppos);
    bt->arg_v = reinterpret_cast<float*>(A + o_argv);
    bt->arg_i = reinterpret_cast<int*>(A + o_argi);
    bt->xh = reinterpret_cast<__half*>(A + o_xh);
    bt->tsc = reinterpret_cast<float*>(A + o_tsc);
    bt->xh_ld = xh_ld;
    if (!ok(cudaMemsetAsync(bt->arena, 0, off, m->stream), err, "clear") ||
        !ok(cudaStreamSynchronize(m->stream), err, "clear")) {
        cudaFreeHost(bt->h_io);
        cudaFree(bt->arena);
        delete bt;
        return B2_ERR_CUDA;
    }
    *out = bt;
    return B2_OK;
}

}  // namespace

// Touches nothing of the model (which may already be freed): cudaFree waits
// for the device's outstanding work before releasing the arena.
void b2_batch_free_impl(b2_batch* bt) {
    if (!bt) return;
    if (bt->exec) cudaGraphExecDestroy(bt->exec);
    if (bt->h_io) cudaFreeHost(bt->h_io);
    if (bt->arena) cudaFree(bt->arena);
    delete bt;
}

namespace {

// Prompt tokens per weight pass: kPrefillChunk when every product can run
// on the tensor-core GEMM (widths a multiple of 64), else the batched
// matvec's kBatchMax.
int prefill_chunk(const ModelDev& d) {
    return (d.H % 64 == 0 && d.qd % 64 == 0 && d.FF % 64 == 0) ? kPrefillChunk : kBatchMax;
}

// Y = W X for the R rows: the tensor-core GEMM from kGemmMinRows rows on,
// the batched matvec (one weight pass, int8 planes against the tiled
// blocks) below.
constexpr int kGemmMinRows = 2;
int matmul_rows(int qt, const uint8_t* w, int64_t rp, int rows, int cols, const float* x, float* y, int R,
                cudaStream_t s, std::string* err) {
    if (R >= kGemmMinRows && cols % 64 == 0) return b2_tiled_gemm_impl(qt, w, rp, 0, rows, cols, x, y, R, s, err);
    return b2_tiled_matvec_batch_impl(qt, w, rp, 0, rows, cols, x, y, R, s, err);
}

// Generation of the scratch buffers a step's launches use (a captured graph
// holds their addresses).
unsigned long long scratch_generation(cudaStream_t s) {
    return b2_mvb_scratch_generation(s) ^ (b2_gemm_scratch_generation(s) << 32);
}

// R rows through the whole model: row r is token d_tok[r] at position
// d_rpos[r], its K / V rows going to kc / vc + r * slot_stride positions
// (per layer, plus kv_off); its attention covers positions 0 .. d_rpos[r].
// With all_logits the lm_head and argmax run for every row (d_next[r],
// d_rpos[r] moved on by one); otherwise for the last row only, into logits
// row 0 and d_next[0] (a prefill chunk needs the argmax after its last token),
// or not at all without any_logits (a prompt's chunks before its last).
// The tensor-core form of forward_rows (every width a multiple of 64, at
// least kGemmMinRows rows): each product takes its input in the GEMM's fp16
// form from the kernel before it and leaves its split-K partials to the
// kernel after it, which sums them: per layer the residual add, RMSNorm and
// conversion are one launch (bd_add_norm_f16), the q/k/v sum rides in the
// RoPE launch and the gate/up sum in the SwiGLU launch.  Every launch of a
// layer is a programmatic dependent launch (launch_pdl): its CTAs are placed
// while the kernel before it drains and wait for it in pdl_wait, so the
// 11 launches of a layer do not each pay a launch and a ramp-up.
bool tc_rows_ok(const ModelDev& d, int R) {
    return R >= kGemmMinRows && R <= kPrefillChunk && d.H % 64 == 0 && d.qd % 64 == 0 && d.FF % 64 == 0 &&
           d.H <= 4 * kRowCtas * kRowThreads * kAddVec && d.FF <= kRowCtas * kRowThreads * kSwClVec;
}

int forward_rows_tc(b2_batch* bt, int R, int* d_rpos, size_t kv_off, int slot_stride, int max_len, std::string* err,
                    bool all_logits, bool any_logits) {
    b2_model* m = bt->m;
    const ModelDev& d = m->dev;
    cudaStream_t s = m->stream;
    // (xh rows are as long as the product that reads them: H, or FF for down)
    const int H = d.H, qt = d.qtype, n_qkv = d.qd + 2 * d.kvd;
    bd_embed_kernel<<<R, kBdThreads, 0, s>>>(d.tok_embd, d.Vemb, d.Vp_emb, H, qt, bt->d_tok, bt->x);
    const size_t kv_layer = (size_t)bt->B * bt->max_seq * d.kvd;
    GemmParts prev;  // the partials still to be added to x (none before layer 0)
    int rc = B2_OK;
    for (int l = 0; l < d.L && rc == B2_OK; l++) {
        const LayerDev& lw = m->layers_host[l];
        launch_pdl(bd_add_norm_f16_kernel, dim3(R * kRowCtas), dim3(kRowThreads), 0, s, bt->x, prev.p, prev.k,
                   prev.plane, lw.attn_norm, H, d.eps, bt->xh, H, bt->tsc, nullptr);
        GemmParts p;
        rc = b2_tiled_gemm_f16_impl(qt, lw.wqkv, tiled_rows(n_qkv), 0, n_qkv, H, bt->xh, bt->tsc, R, bt->qkv, &p, s, err);
        if (rc) break;
        __half* kc = bt->kc + (size_t)l * kv_layer + kv_off;
        __half* vc = bt->vc + (size_t)l * kv_layer + kv_off;
        launch_pdl(bd_rope_kv_kernel, dim3(R, (n_qkv / 2 + kBdThreads - 1) / kBdThreads), dim3(kBdThreads), 0, s,
                   p.p, p.k, p.plane, lw.bqkv, d.rope_cos, d.rope_sin, d_rpos, bt->q, kc, vc, d.qd, d.kvd, d.hd,
                   slot_stride);
        rc = b2_attention_seqs_launch(bt->q, kc, vc, bt->part, bt->part_floats, bt->att, R, d.nh, d.nkv, d.hd, d_rpos,
                                      1, slot_stride, max_len, m->grid, s);
        if (rc) {
            *err = "batched attention launch failed";
            break;
        }
        rc = b2_tiled_gemm_impl(qt, lw.wo, tiled_rows(H), 0, H, d.qd, bt->att, bt->y, R, &p, s, err);
        if (rc) break;
        launch_pdl(bd_add_norm_f16_kernel, dim3(R * kRowCtas), dim3(kRowThreads), 0, s, bt->x, p.p, p.k, p.plane,
                   lw.ffn_norm, H, d.eps, bt->xh, H, bt->tsc, nullptr);
        rc = b2_tiled_gemm_f16_impl(qt, lw.wgu, tiled_rows(2 * d.FF), 0, 2 * d.FF, H, bt->xh, bt->tsc, R, bt->gu, &p, s,
                                    err);
        if (rc) break;
        launch_pdl(bd_swiglu_f16_kernel, dim3(R * kRowCtas), dim3(kRowThreads), 0, s, p.p, p.k, p.plane, d.FF,
                   bt->xh, d.FF, bt->tsc);
        rc = b2_tiled_gemm_f16_impl(qt, lw.wd, tiled_rows(H), 0, H, d.FF, bt->xh, bt->tsc, R, bt->y, &prev, s, err);
    }
    if (rc) return rc;
    if (!any_logits) return ok(cudaGetLastError(), err, "batched decode launch") ? B2_OK : B2_ERR_CUDA;
    // the last down product's partials, the output norm: fp32 rows in xn (for
    // a one-row lm_head on the batched matvec) and the GEMM's form in xh
    launch_pdl(bd_add_norm_f16_kernel, dim3(R * kRowCtas), dim3(kRowThreads), 0, s, bt->x, prev.p, prev.k, prev.plane,
               d.out_norm, H, d.eps, bt->xh, H, bt->tsc, bt->xn);
    const int r_lm = all_logits ? 0 : R - 1, n_lm = all_logits ? R : 1;
    if (n_lm >= kGemmMinRows)
        rc = b2_tiled_gemm_f16_impl(qt, d.lm_head, d.Vp, 0, d.V, H, bt->xh + (size_t)r_lm * H, bt->tsc + r_lm, n_lm,
                                    bt->logits, nullptr, s, err);
    else
        rc = b2_tiled_matvec_batch_impl(qt, d.lm_head, d.Vp, 0, d.V, H, bt->xn + (size_t)r_lm * H, bt->logits, n_lm, s,
                                        err);
    if (rc) return rc;
    bd_argmax_part_kernel<<<n_lm * kArgParts, kBdThreads, 0, s>>>(bt->logits, d.V, bt->arg_v, bt->arg_i);
    bd_argmax_final_kernel<<<n_lm, 32, 0, s>>>(bt->arg_v, bt->arg_i, d.V, bt->d_next, d_rpos + r_lm);
    return ok(cudaGetLastError(), err, "batched decode launch") ? B2_OK : B2_ERR_CUDA;
}

int forward_rows(b2_batch* bt, int R, int* d_rpos, size_t kv_off, int slot_stride, int max_len, std::string* err,
                 bool all_logits = true, bool any_logits = true) {
    if (tc_rows_ok(bt->m->dev, R))
        return forward_rows_tc(bt, R, d_rpos, kv_off, slot_stride, max_len, err, all_logits, any_logits);
    b2_model* m = bt->m;
    const ModelDev& d = m->dev;
    cudaStream_t s = m->stream;
    const int H = d.H, qt = d.qtype, n_qkv = d.qd + 2 * d.kvd;
    bd_embed_kernel<<<R, kBdThreads, 0, s>>>(d.tok_embd, d.Vemb, d.Vp_emb, H, qt, bt->d_tok, bt->x);
    const int ew_blocks = std::max(1, std::min(m->grid * 4, (R * 2 * d.FF + kBdThreads - 1) / kBdThreads));
    const int add_blocks = std::max(1, (R * H + kBdThreads - 1) / kBdThreads);
    const size_t kv_layer = (size_t)bt->B * bt->max_seq * d.kvd;
    int rc = B2_OK;
    for (int l = 0; l < d.L && rc == B2_OK; l++) {
        const LayerDev& ld = m->layers_host[l];
        bd_rmsnorm_kernel<<<R, kNormThreads, 0, s>>>(bt->x, ld.attn_norm, bt->xn, H, d.eps);
        rc = matmul_rows(qt, ld.wqkv, tiled_rows(n_qkv), n_qkv, H, bt->xn, bt->qkv, R, s, err);
        if (rc) break;
        __half* kc = bt->kc + (size_t)l * kv_layer + kv_off;
        __half* vc = bt->vc + (size_t)l * kv_layer + kv_off;
        bd_rope_kv_kernel<<<R, kBdThreads, 0, s>>>(bt->qkv, 1, 0, ld.bqkv, d.rope_cos, d.rope_sin, d_rpos, bt->q, kc, vc,
                                                   d.qd, d.kvd, d.hd, slot_stride);
        rc = b2_attention_seqs_launch(bt->q, kc, vc, bt->part, bt->part_floats, bt->att, R, d.nh, d.nkv, d.hd, d_rpos,
                                      1, slot_stride, max_len, m->grid, s);
        if (rc) {
            *err = "batched attention launch failed";
            break;
        }
        rc = matmul_rows(qt, ld.wo, tiled_rows(H), H, d.qd, bt->att, bt->y, R, s, err);
        if (rc) break;
        bd_add_kernel<<<add_blocks, kBdThreads, 0, s>>>(bt->x, bt->y, R * H);
        bd_rmsnorm_kernel<<<R, kNormThreads, 0, s>>>(bt->x, ld.ffn_norm, bt->xn, H, d.eps);
        rc = matmul_rows(qt, ld.wgu, tiled_rows(2 * d.FF), 2 * d.FF, H, bt->xn, bt->gu, R, s, err);
        if (rc) break;
        bd_swiglu_kernel<<<ew_blocks, kBdThreads, 0, s>>>(bt->gu, bt->act, d.FF, R);
        rc = matmul_rows(qt, ld.wd, tiled_rows(H), H, d.FF, bt->act, bt->y, R, s, err);
        if (rc) break;
        bd_add_kernel<<<add_blocks, kBdThreads, 0, s>>>(bt->x, bt->y, R * H);
    }
    if (rc) return rc;
    if (!any_logits) return ok(cudaGetLastError(), err, "batched decode launch") ? B2_OK : B2_ERR_CUDA;
    const int r_lm = all_logits ? 0 : R - 1, n_lm = all_logits ? R : 1;
    bd_rmsnorm_kernel<<<n_lm, kNormThreads, 0, s>>>(bt->x + (size_t)r_lm * H, d.out_norm, bt->xn, H, d.eps);
    rc = matmul_rows(qt, d.lm_head, d.Vp, d.V, H, bt->xn, bt->logits, n_lm, s, err);
    if (rc) return rc;
    bd_argmax_part_kernel<<<n_lm * kArgParts, kBdThreads, 0, s>>>(bt->logits, d.V, bt->arg_v, bt->arg_i);
    bd_argmax_final_kernel<<<n_lm, 32, 0, s>>>(bt->arg_v, bt->arg_i, d.V, bt->d_next, d_rpos + r_lm);
    return ok(cudaGetLastError(), err, "batched decode launch") ? B2_OK : B2_ERR_CUDA;
}

bool device_current(const b2_model* m, std::string* err) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != m->device) {
        *err = "the model's device must be the current device";
        return false;
    }
    return true;
}

}  // namespace

// The slot's sequence: its prompt in chunks of up to kBatchMax tokens, each
// chunk one pass over the weights (rows = the chunk's tokens, all appending to
// and attending over this slot, token i over positions 0 .. p0 + i).
int b2_batch_prefill_impl(b2_batch* bt, int slot, const int32_t* prompt, int n, int32_t* next_out, std::string* err) {
    b2_model* m = bt->m;
    const ModelDev& d = m->dev;
    if (slot < 0 || slot >= bt->B) {
        *err = "slot outside the batch";
        return B2_ERR_BAD_ARG;
    }
    if (n < 1 || n >= bt->max_seq) {
        *err = "prompt length must be 1 .. max_seq - 1";
        return B2_ERR_CONTEXT;
    }
    if (!device_current(m, err)) return B2_ERR_BAD_ARG;
    cudaStream_t s = m->stream;
    // chunks of equal size (no one-token tail off the tensor-core path)
    const int cmax = prefill_chunk(d), nchunks = (n + cmax - 1) / cmax, chunk = (n + nchunks - 1) / nchunks;
    for (int p0 = 0; p0 < n; p0 += chunk) {
        const int c = std::min(chunk, n - p0);
        if (!ok(cudaMemcpyAsync(bt->d_tok, prompt + p0, sizeof(int) * c, cudaMemcpyHostToDevice, s), err, "tokens"))
            return B2_ERR_CUDA;
        bd_iota_kernel<<<(c + 255) / 256, 256, 0, s>>>(bt->d_ppos, c, p0);
        const int rc = forward_rows(bt, c, bt->d_ppos, (size_t)slot * bt->max_seq * d.kvd, 0, p0 + c, err, false,
                                    p0 + c == n);
        if (rc) return rc;
        // (prompt is pageable host memory: the copy above is complete when the call returns)
    }
    bt->pos[slot] = n;
    bt->h_io[0] = n;
    if (!ok(cudaMemcpyAsync(bt->d_pos + slot, bt->h_io, sizeof(int), cudaMemcpyHostToDevice, s), err, "position") ||
        !ok(cudaMemcpyAsync(bt->h_io + 2 * kBatchMax, bt->d_next, sizeof(int), cudaMemcpyDeviceToHost, s), err, "id") ||
        !ok(cudaStreamSynchronize(s), err, "prefill"))
        return B2_ERR_CUDA;
    if (const int st = b2_gemm_status(s)) {
        *err = "tensor-core GEMM: a bounded wait gave up";
        return st;
    }
    *next_out = bt->h_io[2 * kBatchMax];
    return B2_OK;
}

namespace b2 {

// Prompts from this many tokens on take the tensor-core prefill.
constexpr int kGemmPrefillMin = 16;

bool prefill_gemm_ok(const b2_model* m, int n) {
    const ModelDev& d = m->dev;
    return n >= kGemmPrefillMin && d.tp == 1 && !d.kv_fp32 && (d.hd == 64 || d.hd == 128 || d.hd == 256) &&
           d.nh / d.nkv <= 8 && d.H % 64 == 0 && d.qd % 64 == 0 && d.FF % 64 == 0;
}

void free_prefill_ws(b2_model* m) {
    if (m->prefill_ws) b2_batch_free_impl(m->prefill_ws);
    m->prefill_ws = nullptr;
}

// The prompt in chunks of up to kPrefillChunk tokens, each one pass over the
// weights on the tensor cores, appending to and attending over the model's
// own cache (token i of a chunk sees positions 0 .. its own); then the last
// token's logits and argmax go where the decode kernel leaves them (the
// model's logits buffer and token), so the next decode step and the forward
// entry points read them as after a prefill through the decode kernel.
int prefill_gemm(b2_model* m, const int32_t* tokens, int n, int pos0, std::string* err) {
    const ModelDev& d = m->dev;
    if (!m->prefill_ws) {
        const int rc = batch_create(m, 1, true, &m->prefill_ws, err);
        if (rc) return rc;
    }
    b2_batch* bt = m->prefill_ws;
    cudaStream_t s = m->stream;
    // chunks of equal size (300 tokens: 150 + 150, not 256 + 44): every chunk
    // stays on the tensor-core path
    const int nchunks = (n + kPrefillChunk - 1) / kPrefillChunk, csize = (n + nchunks - 1) / nchunks;
    for (int p0 = 0; p0 < n; p0 += csize) {
        const int c = std::min(csize, n - p0);
        if (!ok(cudaMemcpyAsync(bt->d_tok, tokens + p0, sizeof(int) * c, cudaMemcpyHostToDevice, s), err, "tokens"))
            return B2_ERR_CUDA;
        bd_iota_kernel<<<(c + 255) / 256, 256, 0, s>>>(bt->d_ppos, c, pos0 + p0);
        const int rc = forward_rows(bt, c, bt->d_ppos, 0, 0, pos0 + p0 + c, err, false, p0 + c == n);
        if (rc) return rc;
    }
    if (!ok(cudaMemcpyAsync(d.logits, bt->logits, sizeof(float) * d.V, cudaMemcpyDeviceToDevice, s), err, "logits") ||
        !ok(cudaMemcpyAsync(d.token, bt->d_next, sizeof(int), cudaMemcpyDeviceToDevice, s), err, "token"))
        return B2_ERR_CUDA;
    if (!ok(cudaStreamSynchronize(s), err, "prefill")) return B2_ERR_CUDA;
    if (const int st = b2_gemm_status(s)) {
        *err = "tensor-core GEMM: a bounded wait gave up";
        return st;
    }
    return B2_OK;
}

}  // namespace b2

int b2_batch_step_impl(b2_batch* bt, const int32_t* tokens, int32_t* next_out, std::string* err) {
    b2_model* m = bt->m;
    const ModelDev& d = m->dev;
    const int B = bt->B;
    cudaStream_t s = m->stream;
    if (!device_current(m, err)) return B2_ERR_BAD_ARG;
    int max_len = 0;
    for (int b = 0; b < B; b++) {
        if (bt->pos[b] + 1 > bt->max_seq) {
            *err = "a sequence of the batch is at the KV-cache capacity";
            return B2_ERR_CONTEXT;
        }
        max_len = std::max(max_len, bt->pos[b] + 1);
    }
    for (int b = 0; b < B; b++) bt->h_io[b] = tokens[b];
    if (!ok(cudaMemcpyAsync(bt->d_tok, bt->h_io, sizeof(int) * B, cudaMemcpyHostToDevice, s), err, "tokens"))
        return B2_ERR_CUDA;
    (void)d;
    if (bt->exec && bt->exec_gen != scratch_generation(s)) {  // the scratch moved since the capture
        cudaGraphExecDestroy(bt->exec);
        bt->exec = nullptr;
    }
    if (bt->use_graph && bt->exec) {
        if (!ok(cudaGraphLaunch(bt->exec, s), err, "graph launch")) return B2_ERR_CUDA;
    } else {
        const int rc = forward_rows(bt, B, bt->d_pos, 0, bt->max_seq, max_len, err);
        if (rc) return rc;
    }
    if (!ok(cudaMemcpyAsync(bt->h_io + B, bt->d_next, sizeof(int) * B, cudaMemcpyDeviceToHost, s), err, "ids") ||
        !ok(cudaStreamSynchronize(s), err, "batched decode"))
        return B2_ERR_CUDA;
    if (const int st = b2_gemm_status(s)) {
        *err = "tensor-core GEMM: a bounded wait gave up";
        return st;
    }
    if (bt->use_graph && !bt->exec) {
        // Capture the launches of a step for the next ones (capturing runs
        // nothing).  This step ran them eagerly, so the matvec scratch is
        // already sized and no allocation happens inside the capture.  The
        // attention split count is fixed for the full cache length; every
        // row's length is still read on the device.  A capture that fails
        // leaves the batch stepping eagerly.
        cudaGraph_t graph = nullptr;
        std::string cerr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int crc = forward_rows(bt, B, bt->d_pos, 0, bt->max_seq, bt->max_seq, &cerr);
            const cudaError_t ce = cudaStreamEndCapture(s, &graph);
            if (crc == B2_OK && ce == cudaSuccess && graph &&
                cudaGraphInstantiate(&bt->exec, graph, 0) == cudaSuccess) {
                bt->exec_gen = scratch_generation(s);
            } else {
                bt->exec = nullptr;
            }
            if (graph) cudaGraphDestroy(graph);
        }
        (void)cudaGetLastError();  // a refused capture is not this step's error
    }
    for (int b = 0; b < B; b++) {
        next_out[b] = bt->h_io[B + b];
        bt->pos[b] += 1;
    }
    return B2_OK;
}

int b2_batch_use_graph_impl(b2_batch* bt, int on) {
    bt->use_graph = on != 0;
    if (!bt->use_graph && bt->exec) {
        cudaGraphExecDestroy(bt->exec);
        bt->exec = nullptr;
    }
    return B2_OK;
}

// Logits of the last step, [B][vocab] floats.
int b2_batch_logits_impl(const b2_batch* bt, float* out, std::string* err) {
    const size_t n = (size_t)bt->B * bt->m->dev.V;
    if (!ok(cudaMemcpyAsync(out, bt->logits, n * sizeof(float), cudaMemcpyDeviceToHost, bt->m->stream), err,
            "logits") ||
        !ok(cudaStreamSynchronize(bt->m->stream), err, "logits"))
        return B2_ERR_CUDA;
    return B2_OK;
}
