// Fused mixture-of-experts layer, exact version: router logits, softmax/top-k, token->expert
// permutation, gate/up/SiLU, down and the shared-expert weighted combine, all on the device
// with no host readback of the routing (the reference reads the IDs back on every layer,
// src/engine.js:137, and groups tokens by expert in JavaScript, src/prefill.js:55-61).
//
// Every dot product keeps the reference's reduction order (64 lanes, lane-strided F32
// accumulation, tree s = 32..1; kernels/strata.cu:38-69, 156-165) with no contraction, so
// routing and outputs are bit-identical to the reference's CPU path.
//
// Pipeline (one stream, six launches, capturable in a CUDA graph):
//   k_logits   : router rows (+ the shared-expert gate row) for every token
//   k_topk     : one warp per token (route.cuh)
//   k_permute  : histogram of expert ids, scan, stable token-major scatter of (token, k) pairs
//   k_gate_up  : per (expert slot, 16 row pairs): hidden = silu(gate . x) * (up . x)
//   k_down     : per (expert slot, 16 output rows): parts[t*k + kk] = down . hidden
//   k_combine  : y = shared * sigmoid(sg) + sum_k parts[k] * w[k]   (kernels/strata.cu:470-476)
// Slot 0 of the expert grids is the shared expert (all tokens), slot s > 0 the s-th active
// routed expert; grids are sized for the worst case and slots past the active count exit.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "route.cuh"

namespace strata {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTokChunk = 4;    // tokens staged per pass in k_logits
constexpr int kGuRowPairs = 16; // gate/up row pairs per block in k_gate_up (2 per warp)
constexpr int kDownRows = 16;   // output rows per block in k_down (2 per warp)

struct BlobOffsets {
    long long d_codes;    // words
    long long gu_scales;  // halves
    long long d_scales;   // halves
};
// vendor/strata/tools/pack_layer.py:54-65 with H = width, FF = ff.
__host__ __device__ inline BlobOffsets blob_offsets(int width, int ff) {
    long long hf = (long long)width * ff;
    return BlobOffsets{2 * hf / 16, 3 * hf / 8, 3 * hf / 8 + hf / 32};
}

__global__ void __launch_bounds__(kThreads) k_logits(MoeLayerDev L, const float *__restrict__ x, int tokens, float *logits, float *sg) {
    extern __shared__ float xs[];  // kTokChunk * width
    const int w = threadIdx.x / 32, t = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + w;
    const int width = L.width;
    const float *W = row < L.experts ? L.router + (long long)row * width : (row == L.experts ? L.shared_gate : nullptr);
    for (int t0 = 0; t0 < tokens; t0 += kTokChunk) {
        const int nt = min(kTokChunk, tokens - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * width; i += kThreads) xs[i] = x[(long long)t0 * width + i];
        __syncthreads();
        if (!W) continue;
        for (int j = 0; j < nt; ++j) {
            const float *xv = xs + j * width;
            float lo = 0.0f, hi = 0.0f;
            for (int i = t; i < width; i += STRATA_LANES) {
                lo = __fadd_rn(lo, __fmul_rn(W[i], xv[i]));
                if (i + 32 < width) hi = __fadd_rn(hi, __fmul_rn(W[i + 32], xv[i + 32]));
            }
            float r = tree64(lo, hi);
            if (t == 0) {
                if (row < L.experts) {
                    // strata_elementwise mode 5 (a*1 + b) for the optional logit offset
                    logits[(long long)(t0 + j) * L.experts + row] = L.bias ? __fadd_rn(r, L.bias[row]) : r;
                } else {
                    sg[t0 + j] = r;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(128) k_topk(const float *logits, int tokens, int experts, int topK, int *ids, float *weights) {
    __shared__ float lg[4][512];
    __shared__ float sel[4][32];
    const int w = threadIdx.x / 32, t = threadIdx.x & 31;
    const int token = blockIdx.x * 4 + w;
    if (token >= tokens) return;
    for (int e = t; e < experts; e += 32) lg[w][e] = logits[(long long)token * experts + e];
    __syncwarp();
    route_warp(lg[w], experts, topK, ids + (long long)token * topK, weights + (long long)token * topK, sel[w]);
}

// Stable counting sort of the (token, k) pairs by expert id, token-major inside an expert
// (the order in which src/prefill.js:56-60 appends jobs). One block.
__global__ void __launch_bounds__(1024) k_permute(const int *ids, int tokens, int topK, int experts, int *counts, int *active,
                                                  int *n_active, int *begin, int *pair_token, int *pair_slot, unsigned *err) {
    __shared__ int cnt[512];
    __shared__ int beg[512];
    const int P = tokens * topK;
    for (int e = threadIdx.x; e < experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        int e = ids[p];
        if (e < 0 || e >= experts) raise_error(err, kErrRouting);
        else atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, na = 0;
        for (int e = 0; e < experts; ++e) {
            beg[e] = acc;
            counts[e] = cnt[e];
            if (cnt[e]) {
                active[na] = e;
                begin[na] = acc;
                ++na;
            }
            acc += cnt[e];
        }
        begin[na] = acc;
        *n_active = na;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        int e = ids[p];
        if (e < 0 || e >= experts) continue;
        int rank = 0;
        for (int q = 0; q < p; ++q) rank += ids[q] == e;
        const int pos = beg[e] + rank;
        pair_token[pos] = p / topK;
        pair_slot[pos] = p;
    }
}

__device__ __forceinline__ bool slot_of(int slot, const MoeLayerDev &L, int tokens, const int *n_active, const int *active,
                                        const int *begin, const unsigned *&blob, int &p0, int &np) {
    if (slot == 0) {
        blob = L.shared_blob;
        p0 = 0;
        np = tokens;
        return true;
    }
    const int na = *n_active;
    if (slot > na) return false;
    blob = L.blobs + (long long)active[slot - 1] * L.blob_words;
    p0 = begin[slot - 1];
    np = begin[slot] - p0;
    return true;
}

// hidden row of a pair: routed pairs in permuted order, then the shared expert's tokens.
__global__ void __launch_bounds__(kThreads) k_gate_up(MoeLayerDev L, const float *__restrict__ x, int tokens, const int *n_active,
                                                      const int *active, const int *begin, const int *pair_token, float *hidden) {
    const unsigned *blob;
    int p0, np;
    if (!slot_of(blockIdx.y, L, tokens, n_active, active, begin, blob, p0, np)) return;
    const int width = L.width, ff = L.ff;
    const int wpr = width / 16, gpr = width / 64;  // code words and scale groups per blob row
    extern __shared__ unsigned char smem[];
    unsigned *codes = reinterpret_cast<unsigned *>(smem);              // [2*kGuRowPairs][wpr]
    float *scl = reinterpret_cast<float *>(codes + 2 * kGuRowPairs * wpr);  // [2*kGuRowPairs][gpr]
    float *xs = scl + 2 * kGuRowPairs * gpr;                            // [width]
    const int r0 = blockIdx.x * kGuRowPairs;  // first row pair = blob rows 2*r0 ...
    const BlobOffsets off = blob_offsets(width, ff);
    const unsigned *src = blob + (long long)2 * r0 * wpr;
    for (int i = threadIdx.x; i < 2 * kGuRowPairs * wpr; i += kThreads) codes[i] = src[i];
    for (int i = threadIdx.x; i < 2 * kGuRowPairs * gpr; i += kThreads) {
        long long h = off.gu_scales + (long long)2 * r0 * gpr + i;
        scl[i] = half_bits((blob[h / 2] >> ((h % 2) * 16)) & 65535u);
    }
    const int w = threadIdx.x / 32, t = threadIdx.x & 31;
    const long long shared_base = (long long)tokens * L.topK;
    for (int j = 0; j < np; ++j) {
        const int token = blockIdx.y == 0 ? j : pair_token[p0 + j];
        __syncthreads();
        for (int i = threadIdx.x; i < width; i += kThreads) xs[i] = x[(long long)token * width + i];
        __syncthreads();
        for (int rr = 2 * w; rr < 2 * w + 2; ++rr) {
            const unsigned *gc = codes + (2 * rr) * wpr, *uc = gc + wpr;
            const float *gsc = scl + (2 * rr) * gpr, *usc = gsc + gpr;
            float g[2] = {0.0f, 0.0f}, u[2] = {0.0f, 0.0f};
            for (int i0 = t; i0 < width; i0 += STRATA_LANES)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = i0 + 32 * h;
                    const int sh = (i % 16) * 2;
                    const float xv = xs[i];
                    const float gw = __fmul_rn((float)((int)((gc[i / 16] >> sh) & 3u) - 1), gsc[i / 64]);
                    const float uw = __fmul_rn((float)((int)((uc[i / 16] >> sh) & 3u) - 1), usc[i / 64]);
                    g[h] = __fadd_rn(g[h], __fmul_rn(gw, xv));
                    u[h] = __fadd_rn(u[h], __fmul_rn(uw, xv));
                }
            const float gs = tree64(g[0], g[1]), us = tree64(u[0], u[1]);
            if (t == 0) {
                const long long hrow = blockIdx.y == 0 ? shared_base + token : (long long)(p0 + j);
                hidden[hrow * ff + r0 + rr] = __fmul_rn(ref_silu(gs), us);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) k_down(MoeLayerDev L, int tokens, const int *n_active, const int *active, const int *begin,
                                                   const int *pair_slot, const float *hidden, float *parts, float *shared_out) {
    const unsigned *blob;
    int p0, np;
    if (!slot_of(blockIdx.y, L, tokens, n_active, active, begin, blob, p0, np)) return;
    const int width = L.width, ff = L.ff;
    const int wpr = ff / 16, gpr = ff / 64;
    extern __shared__ unsigned char smem[];
    unsigned *codes = reinterpret_cast<unsigned *>(smem);         // [kDownRows][wpr]
    float *scl = reinterpret_cast<float *>(codes + kDownRows * wpr);  // [kDownRows][gpr]
    float *hs = scl + kDownRows * gpr;                             // [ff]
    const int c0 = blockIdx.x * kDownRows;
    const BlobOffsets off = blob_offsets(width, ff);
    const unsigned *src = blob + off.d_codes + (long long)c0 * wpr;
    for (int i = threadIdx.x; i < kDownRows * wpr; i += kThreads) codes[i] = src[i];
    for (int i = threadIdx.x; i < kDownRows * gpr; i += kThreads) {
        long long h = off.d_scales + (long long)c0 * gpr + i;
        scl[i] = half_bits((blob[h / 2] >> ((h % 2) * 16)) & 65535u);
    }
    const int w = threadIdx.x / 32, t = threadIdx.x & 31;
    const long long shared_base = (long long)tokens * L.topK;
    for (int j = 0; j < np; ++j) {
        const long long hrow = blockIdx.y == 0 ? shared_base + j : (long long)(p0 + j);
        __syncthreads();
        for (int i = threadIdx.x; i < ff; i += kThreads) hs[i] = hidden[hrow * ff + i];
        __syncthreads();
        for (int rr = 2 * w; rr < 2 * w + 2; ++rr) {
            const unsigned *dc = codes + rr * wpr;
            const float *dsc = scl + rr * gpr;
            float a[2] = {0.0f, 0.0f};
            for (int i0 = t; i0 < ff; i0 += STRATA_LANES)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = i0 + 32 * h;
                    const float wv = __fmul_rn((float)((int)((dc[i / 16] >> ((i % 16) * 2)) & 3u) - 1), dsc[i / 64]);
                    a[h] = __fadd_rn(a[h], __fmul_rn(wv, hs[i]));
                }
            const float r = tree64(a[0], a[1]);
            if (t == 0) {
                if (blockIdx.y == 0) shared_out[(long long)j * width + c0 + rr] = r;
                else parts[(long long)pair_slot[p0 + j] * width + c0 + rr] = r;
            }
        }
    }
}

// A pair whose id is outside [0, experts) (a token whose probabilities are all NaN routes to
// -1, which k_permute reports as kErrRouting, src/engine.js:138) has no parts row: it adds
// nothing, so y never depends on what the scratch held before the call.
__global__ void k_combine(const float *parts, const float *weights, const int *ids, const float *shared_out, const float *sg, float *y,
                          int width, int topK, int experts, int tokens) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)width * tokens) return;
    long long token = i / width, d = i % width;
    float value = __fmul_rn(shared_out[i], ref_sigmoid(sg[token]));
    for (int k = 0; k < topK; ++k) {
        if ((unsigned)ids[token * topK + k] >= (unsigned)experts) continue;
        value = __fadd_rn(value, __fmul_rn(parts[(token * topK + k) * width + d], weights[token * topK + k]));
    }
    y[i] = value;
}

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// src/model.js:164 (readExpertBlob): every FP16 scale of a blob, from the gate/up scale plane to
// the end of the down scale plane, must be finite (its exponent bits 0x7c00 not all set). Each
// thread checks one word (two scales); the lowest offending blob index is kept.
__global__ void k_check_scales(const unsigned *blobs, long long blob_words, long long first_word, long long count, int *first_bad) {
    const long long per = blob_words - first_word, n = count * per;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i / per;
        const unsigned v = __ldg(blobs + e * blob_words + first_word + i % per);
        if ((v & 0x7c00u) == 0x7c00u || (v & 0x7c000000u) == 0x7c000000u) atomicMin(first_bad, (int)e);
    }
}

}  // namespace

cudaError_t check_expert_scales(const unsigned *blobs, long long count, int width, int ff, int *first_bad, cudaStream_t s) {
    const long long blob_words = 27LL * ff * width / 128, first_word = 3LL * ff * width / 16;
    STRATA_CUDA_TRY(cudaMemsetAsync(first_bad, 0x7f, sizeof(int), s));  // 0x7f7f7f7f: no blob failed
    const long long n = count * (blob_words - first_word);
    const unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, 148LL * 16);
    if (n > 0) k_check_scales<<<blocks, 256, 0, s>>>(blobs, blob_words, first_word, count, first_bad);
    return cudaGetLastError();
}

size_t moe_scratch_bytes(int tokens, int width, int ff, int experts, int topK) {
    size_t P = (size_t)tokens * topK;
    return align256(sizeof(float) * tokens * experts) + align256(sizeof(float) * tokens) + align256(sizeof(int) * experts) +
           align256(sizeof(int) * experts) + align256(sizeof(int)) + align256(sizeof(int) * (experts + 1)) +
           align256(sizeof(int) * P) * 2 + align256(sizeof(float) * (P + tokens) * ff) + align256(sizeof(float) * P * width) +
           align256(sizeof(float) * (size_t)tokens * width);
}

MoeScratch moe_scratch_carve(void *base, int tokens, int width, int ff, int experts, int topK) {
    char *p = static_cast<char *>(base);
    size_t P = (size_t)tokens * topK;
    auto take = [&](size_t n) {
        char *r = p;
        p += align256(n);
        return r;
    };
    MoeScratch s;
    s.logits = (float *)take(sizeof(float) * tokens * experts);
    s.sg = (float *)take(sizeof(float) * tokens);
    s.counts = (int *)take(sizeof(int) * experts);
    s.active = (int *)take(sizeof(int) * experts);
    s.n_active = (int *)take(sizeof(int));
    s.begin = (int *)take(sizeof(int) * (experts + 1));
    s.pair_token = (int *)take(sizeof(int) * P);
    s.pair_slot = (int *)take(sizeof(int) * P);
    s.hidden = (float *)take(sizeof(float) * (P + tokens) * ff);
    s.parts = (float *)take(sizeof(float) * P * width);
    s.shared_out = (float *)take(sizeof(float) * (size_t)tokens * width);
    return s;
}

cudaError_t moe_forward_exact(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights,
                              const MoeScratch &ws, cudaStream_t s, unsigned *err) {
    const int rows = L.experts + 1;
    const size_t lg_smem = sizeof(float) * kTokChunk * L.width;
    if (lg_smem > 48 * 1024) STRATA_CUDA_TRY(cudaFuncSetAttribute(k_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lg_smem));
    k_logits<<<(rows + kWarps - 1) / kWarps, kThreads, lg_smem, s>>>(L, x, tokens, ws.logits, ws.sg);
    STRATA_CUDA_TRY(cudaGetLastError());
    k_topk<<<(tokens + 3) / 4, 128, 0, s>>>(ws.logits, tokens, L.experts, L.topK, ids, weights);
    STRATA_CUDA_TRY(cudaGetLastError());
    k_permute<<<1, 1024, 0, s>>>(ids, tokens, L.topK, L.experts, ws.counts, ws.active, ws.n_active, ws.begin, ws.pair_token,
                                 ws.pair_slot, err);
    STRATA_CUDA_TRY(cudaGetLastError());
    const int slots = 1 + min(tokens * L.topK, L.experts);
    const size_t gu_smem = sizeof(unsigned) * 2 * kGuRowPairs * (L.width / 16) + sizeof(float) * 2 * kGuRowPairs * (L.width / 64) +
                           sizeof(float) * L.width;
    if (gu_smem > 48 * 1024) STRATA_CUDA_TRY(cudaFuncSetAttribute(k_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gu_smem));
    k_gate_up<<<dim3(L.ff / kGuRowPairs, slots), kThreads, gu_smem, s>>>(L, x, tokens, ws.n_active, ws.active, ws.begin, ws.pair_token,
                                                                        ws.hidden);
    STRATA_CUDA_TRY(cudaGetLastError());
    const size_t dn_smem = sizeof(unsigned) * kDownRows * (L.ff / 16) + sizeof(float) * kDownRows * (L.ff / 64) + sizeof(float) * L.ff;
    if (dn_smem > 48 * 1024) STRATA_CUDA_TRY(cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dn_smem));
    k_down<<<dim3(L.width / kDownRows, slots), kThreads, dn_smem, s>>>(L, tokens, ws.n_active, ws.active, ws.begin, ws.pair_slot,
                                                                      ws.hidden, ws.parts, ws.shared_out);
    STRATA_CUDA_TRY(cudaGetLastError());
    const long long n = (long long)tokens * L.width;
    k_combine<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(ws.parts, weights, ids, ws.shared_out, ws.sg, y, L.width, L.topK, L.experts,
                                                      tokens);
    return cudaGetLastError();
}

}  // namespace strata
