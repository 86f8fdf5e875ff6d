// Mixture-of-experts layer for prompt batches (and decode batches above the fused decode
// kernel's eight tokens): exact routing, then the expert products on tcgen05 tensor cores.
//
//   k_pf_logits  router logits (+ the shared-gate row), bit-identical to the reference
//                (kernels/strata.cu:156-165): thread = one of the reference's 64 lanes for a
//                register block of 8 tokens x 8 rows, lane-strided F32 sums without
//                contraction, then the reference's tree across the two warps of the lane group
//   k_pf_route   softmax / top-k / weights, one warp per token (route.cuh route_warp)
//   k_pf_count   per token-chunk expert histograms
//   k_pf_scan    per-expert offsets, the chunk list of the GEMMs (decreasing size)
//   k_pf_place   stable (token-major) position of every (token, k) pair in its expert's
//                segment, as src/prefill.js:55-61 groups them
//   k_pf_xprep   B rows for the gate/up GEMM: each token's activations as FP16 times 2^k
//                (largest |x| below 2^15), written at its pairs' positions and at row
//                T*topK + t for the shared expert; per row the token, weight and 2^-k
//   k_pf_gemm    gate/up (hidden = silu(gate) * up, FP16) then down (y += weight * D)
// y is zeroed first and receives the shared expert and every routed pair by 16-byte atomic
// adds, so y is not bit-reproducible run to run; it stays within 2e-3 relative L2 of the
// reference (the FP16 tensor-core path's tolerance; tested). Routing is bit-exact.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ep_comm.h"
#include "kernels.h"
#include "pf_gemm.cuh"
#include "route.cuh"

namespace strata {
namespace pf {

// ------------------------------------------------------------------ router logits
// Router logits (+ the shared-gate row as row E), bit-identical to the reference's order: lane
// l of 64 sums x[k] w[k] over k = l mod 64 in increasing k, one rounding per multiply and per
// add (scalar __fmul_rn / __fadd_rn; the paired F32 instructions are slower here than the
// scalar pipe and fuse into a single-rounding multiply-add unless kept apart), then the tree
// partial[l] += partial[l + s], s = 32 .. 1.
//
// Persistent, one CTA per SM: work item = 16 tokens x 3 row tiles of kLgR rows. Warp
// kLgWarps is the producer: per item it loads the 16 tokens' x by 256-column chunks (one TMA
// box each, rows past T read as zero) into a resident buffer, and streams the router rows of
// each (row tile, chunk) step through a ring of stages (one TMA box each; the last row tile,
// which holds the shared-gate row, comes from a per-call tail copy of those rows). Each x
// chunk is released once the item's last row tile has used it, so the next item's x loads
// while the current one finishes. Compute warps: thread i holds the reference's lanes 2i and
// 2i + 1 (one 8-byte shared load gives both lanes' operands) for an 8-token x 4-row tile. The
// tree is a transposing butterfly: at xor distance 16, 8, 4, 2, 1 (lane distance 32 .. 2)
// each thread keeps half of its outputs and adds its partner's pair for them (both lanes at
// once: add.rn.f32x2 rounds each element like __fadd_rn); the last add joins lanes 0 and 1.
// Every add has the reference's operands; thread t ends with output t = 4 token + row.
constexpr int kLgT = 16;                                // tokens per work item
constexpr int kLgKC = 256;                              // K chunk (one 1 KB row segment per box row)
constexpr int kLgGroup = 3;                             // row tiles per work item
constexpr int kLgWarps = 12;                            // compute warps; warp kLgWarps produces
constexpr int kLgWT = 8, kLgWR = 4;                     // warp tile: tokens, rows
constexpr int kLgR = (kLgWarps / (kLgT / kLgWT)) * kLgWR;  // rows per row tile (24)
constexpr int kLgMaxStages = 4, kLgMaxNC = 10;          // router stages; x chunks (H <= 2560)
constexpr int kLgThreads = 32 * (kLgWarps + 1);
constexpr size_t kLgSmemLimit = 227 * 1024;

struct LgMaps {
    CUtensorMap router;  // {H, E} F32, box {256, kLgR}
    CUtensorMap tail;    // {H, kLgR} F32 (rows E / kLgR * kLgR .. : router rows, the gate, zeros), box {256, kLgR}
    CUtensorMap x;       // {H, T} F32, box {256, 16}
};
struct __align__(8) LgBars {
    unsigned long long full[kLgMaxStages], empty[kLgMaxStages], xfull[kLgMaxNC], xempty[kLgMaxNC];
    int abort_flag;
};
inline int logits_stages(int H) {
    const size_t fixed = 1024 + sizeof(LgBars) + (size_t)kLgT * H * 4;
    const size_t stage = (size_t)kLgR * kLgKC * 4;
    return (int)std::min<size_t>(kLgMaxStages, (kLgSmemLimit - fixed) / stage);
}
inline size_t logits_smem(int H) { return 1024 + sizeof(LgBars) + (size_t)kLgT * H * 4 + (size_t)logits_stages(H) * kLgR * kLgKC * 4; }

// The last row tile's rows: router rows [r0, E), the shared gate at E, zeros up to kLgR.
__global__ void k_lg_tail(const float *router, const float *gate, int E, int H, int r0, float *tail) {
    const int i = blockIdx.x, r = r0 + i;
    const float *src = r < E ? router + (long long)r * H : gate;
    for (int k = threadIdx.x; k < H; k += blockDim.x) tail[(long long)i * H + k] = r <= E ? src[k] : 0.0f;
}

__global__ void __launch_bounds__(kLgThreads, 1)
    k_pf_logits(const __grid_constant__ LgMaps M, MoeLayerDev L, int T, int ST, int group, float *logits, float *sg, unsigned *err,
                unsigned long long spin_limit, unsigned long long neg0) {
    extern __shared__ unsigned char lg_raw[];
    unsigned char *base = lg_raw + ((1024 - (su32(lg_raw) & 1023)) & 1023);
    const int H = L.width, E = L.experts, NC = H / kLgKC;
    float *xs = reinterpret_cast<float *>(base);       // [NC][16][256]
    float *ws = xs + (size_t)NC * kLgT * kLgKC;         // [ST][kLgR][256]
    LgBars &B = *reinterpret_cast<LgBars *>(ws + (size_t)ST * kLgR * kLgKC);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_full = E / kLgR, n_rt = n_full + 1, n_grp = (n_rt + group - 1) / group;
    const int n_items = ((T + kLgT - 1) / kLgT) * n_grp;
    if (tid == 0) {
        for (int i = 0; i < ST; ++i) {
            bar_init(&B.full[i], 1);
            bar_init(&B.empty[i], kLgWarps);
        }
        for (int i = 0; i < NC; ++i) {
            bar_init(&B.xfull[i], 1);
            bar_init(&B.xempty[i], kLgWarps);
        }
        B.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    auto wait = [&](unsigned long long *b, unsigned parity) -> bool {
        for (unsigned long long i = 0;; ++i) {
            if (bar_try(b, parity)) return true;
            if (i > spin_limit || *(volatile int *)&B.abort_flag) {
                atomicOr(&B.abort_flag, 1);
                return false;
            }
        }
    };
    if (warp == kLgWarps) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            int g = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
                const int t0 = (item / n_grp) * kLgT, rt0 = (item % n_grp) * group;
                const int nrt = min(group, n_rt - rt0);
                for (int rr = 0; rr < nrt && ok; ++rr)
                    for (int c = 0; c < NC && ok; ++c, ++g) {
                        if (rr == 0) {  // the item's x chunk c, once the previous item released it
                            if (!(ok = wait(&B.xempty[c], (it & 1) ^ 1))) break;
                            bar_expect(&B.xfull[c], kLgT * kLgKC * 4);
                            tma2(xs + (size_t)c * kLgT * kLgKC, &M.x, c * kLgKC, t0, &B.xfull[c]);
                        }
                        const int st = g % ST, rt = rt0 + rr;
                        if (!(ok = wait(&B.empty[st], ((g / ST) & 1) ^ 1))) break;
                        bar_expect(&B.full[st], kLgR * kLgKC * 4);
                        if (rt < n_full) tma2(ws + (size_t)st * kLgR * kLgKC, &M.router, c * kLgKC, rt * kLgR, &B.full[st]);
                        else tma2(ws + (size_t)st * kLgR * kLgKC, &M.tail, c * kLgKC, 0, &B.full[st]);
                    }
            }
            // every issued copy lands before the CTA leaves (bounded)
            for (int k = max(0, g - ST); k < g; ++k)
                for (unsigned long long i = 0; i <= spin_limit && !bar_try(&B.full[k % ST], (k / ST) & 1); ++i) {
                }
        }
    } else {
        // ---------------------------------------------------------------- compute
        const int tb = (warp % (kLgT / kLgWT)) * kLgWT, rb = (warp / (kLgT / kLgWT)) * kLgWR;
        typedef unsigned long long u64;
        int g = 0, it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
            const int t0 = (item / n_grp) * kLgT, rt0 = (item % n_grp) * group;
            const int nrt = min(group, n_rt - rt0);
            for (int rr = 0; rr < nrt && ok; ++rr) {
                // per (token, row): the two reference lanes' partial sums as one f32 pair (low: lane
                // 2 l, high: lane 2 l + 1)
                u64 acc[kLgWT][kLgWR];
#pragma unroll
                for (int i = 0; i < kLgWT; ++i)
#pragma unroll
                    for (int j = 0; j < kLgWR; ++j) acc[i][j] = 0ull;
                for (int c = 0; c < NC; ++c, ++g) {
                    const int st = g % ST;
                    if (!(ok = __all_sync(0xffffffffu, (rr > 0 || wait(&B.xfull[c], it & 1)) && wait(&B.full[st], (g / ST) & 1)))) break;
                    const float *xb = xs + (size_t)c * kLgT * kLgKC + 2 * lane;
                    const float *wb = ws + (size_t)st * kLgR * kLgKC + 2 * lane;
                    u64 xv[2][kLgWT], wv[2][kLgWR];
#pragma unroll
                    for (int i = 0; i < kLgWT; ++i) xv[0][i] = *reinterpret_cast<const u64 *>(xb + (tb + i) * kLgKC);
#pragma unroll
                    for (int j = 0; j < kLgWR; ++j) wv[0][j] = *reinterpret_cast<const u64 *>(wb + (rb + j) * kLgKC);
#pragma unroll
                    for (int m = 0; m < kLgKC / 64; ++m) {  // elements 2 lane + 64 m and + 1: the two lanes' next terms
                        const int cur = m & 1;
                        if (m + 1 < kLgKC / 64) {
#pragma unroll
                            for (int i = 0; i < kLgWT; ++i) xv[cur ^ 1][i] = *reinterpret_cast<const u64 *>(xb + (tb + i) * kLgKC + 64 * (m + 1));
#pragma unroll
                            for (int j = 0; j < kLgWR; ++j) wv[cur ^ 1][j] = *reinterpret_cast<const u64 *>(wb + (rb + j) * kLgKC + 64 * (m + 1));
                        }
                        // the reference's rounded product then rounded add, two lanes per instruction
                        // (mul_rn2: an FMA with the run-time addend neg0 = (-0, -0), never fused with the add)
#pragma unroll
                        for (int i = 0; i < kLgWT; ++i)
#pragma unroll
                            for (int j = 0; j < kLgWR; ++j) acc[i][j] = add2_rn(acc[i][j], mul_rn2(wv[cur][j], xv[cur][i], neg0));
                    }
                    __syncwarp();
                    if (lane == 0) {
                        bar_arrive(&B.empty[st]);
                        if (rr == nrt - 1) bar_arrive(&B.xempty[c]);
                    }
                }
                if (!ok) break;
                // row tile done: the tree and this thread's output
                u64 v[kLgWT * kLgWR];
#pragma unroll
                for (int i = 0; i < kLgWT; ++i)
#pragma unroll
                    for (int j = 0; j < kLgWR; ++j) v[i * kLgWR + j] = acc[i][j];
#pragma unroll
                for (int half = 16; half > 0; half >>= 1) {
                    const bool upper = (lane & half) != 0;
#pragma unroll
                    for (int o = 0; o < half; ++o) {
                        const u64 mine = upper ? v[o + half] : v[o];
                        const u64 theirs = shfl_xor_u64(upper ? v[o] : v[o + half], half);
                        v[o] = add2_rn(mine, theirs);
                    }
                }
                const float a = __fadd_rn(__uint_as_float((unsigned)v[0]), __uint_as_float((unsigned)(v[0] >> 32)));
                const int t = t0 + tb + lane / kLgWR, r = (rt0 + rr) * kLgR + rb + lane % kLgWR;
                if (t < T) {
                    if (r < E) logits[(long long)t * E + r] = L.bias ? __fadd_rn(a, L.bias[r]) : a;
                    else if (r == E) sg[t] = a;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0 && B.abort_flag) raise_error(err, kErrWaitTimeout);
}
static_assert(kLgWT * kLgWR == 32, "the butterfly leaves one output per thread");

// ------------------------------------------------------------------ routing
__global__ void __launch_bounds__(128) k_pf_route(const float *logits, int T, int E, int K, int *ids, float *weights) {
    __shared__ float lg[4][512];
    __shared__ float sel[4][32];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + w;
    if (t >= T) return;
    for (int e = lane; e < E; e += 32) lg[w][e] = logits[(long long)t * E + e];
    __syncwarp();
    route_warp(lg[w], E, K, ids + (long long)t * K, weights + (long long)t * K, sel[w]);
}

// ------------------------------------------------------------------ permutation
constexpr int kTokChunk = 256;  // tokens per counting chunk

__global__ void __launch_bounds__(256) k_pf_count(const int *ids, int T, int E, int K, int *chunk_counts) {
    __shared__ int h[512];
    for (int e = threadIdx.x; e < E; e += 256) h[e] = 0;
    __syncthreads();
    const int c = blockIdx.x;
    const long long p0 = (long long)c * kTokChunk * K, p1 = min((long long)T * K, p0 + (long long)kTokChunk * K);
    for (long long p = p0 + threadIdx.x; p < p1; p += 256) {
        const int e = ids[p];
        if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += 256) chunk_counts[(long long)c * E + e] = h[e];
}

// One block of 512 threads, thread e = bucket (expert) e: it walks the token chunks
// (chunk_base = running count), block scans give the bucket offsets and the positions of every
// bucket's full kMaxN-row chunks; the chunk list is the shared expert's Ts rows starting at
// row shared0, then the full chunks, then the remainders by decreasing size (a counting sort
// over 1 .. kMaxN - 1).
__global__ void __launch_bounds__(512) k_pf_scan(int *chunk_counts, int n_tc, int Ts, int shared0, int E, int *offsets, Chunk *chunks,
                                                 int *n_chunks) {
    __shared__ int wsum[16], wfull[16], total_full;
    __shared__ int rem_hist[kMaxN], rem_start[kMaxN];
    const int e = threadIdx.x, lane = e & 31, w = e >> 5;
    int run = 0;
    if (e < E)
        for (int c = 0; c < n_tc; ++c) {
            const int v = chunk_counts[(long long)c * E + e];
            chunk_counts[(long long)c * E + e] = run;  // becomes the chunk's base within the expert
            run += v;
        }
    const int cnt = e < E ? run : 0, full = cnt / kMaxN, rem = cnt % kMaxN;
    int a = cnt, f = full;  // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ya = __shfl_up_sync(0xffffffffu, a, o), yf = __shfl_up_sync(0xffffffffu, f, o);
        if (lane >= o) {
            a += ya;
            f += yf;
        }
    }
    if (lane == 31) {
        wsum[w] = a;
        wfull[w] = f;
    }
    if (e < kMaxN) rem_hist[e] = 0;
    __syncthreads();
    if (e == 0) {
        int s1 = 0, s2 = 0;
        for (int i = 0; i < 16; ++i) {
            const int t1 = wsum[i], t2 = wfull[i];
            wsum[i] = s1;
            wfull[i] = s2;
            s1 += t1;
            s2 += t2;
        }
        total_full = s2;
    }
    __syncthreads();
    const int off = wsum[w] + a - cnt, fpos = wfull[w] + f - full;
    if (e < E) offsets[e] = off;
    if (e == E - 1) offsets[E] = off + cnt;
    if (e < E && rem) atomicAdd(&rem_hist[rem], 1);
    __syncthreads();
    const int n_shared = (Ts + kMaxN - 1) / kMaxN;
    if (e == 0) {
        int s = n_shared + total_full;
        for (int sz = kMaxN - 1; sz >= 1; --sz) {
            rem_start[sz] = s;
            s += rem_hist[sz];
        }
        *n_chunks = s;
    }
    __syncthreads();
    for (int i = e; i < n_shared; i += 512) chunks[i] = Chunk{-1, shared0 + i * kMaxN, min(kMaxN, Ts - i * kMaxN), 0};
    if (e < E) {
        for (int i = 0; i < full; ++i) chunks[n_shared + fpos + i] = Chunk{e, off + i * kMaxN, kMaxN, 0};
        if (rem) chunks[atomicAdd(&rem_start[rem], 1)] = Chunk{e, off + cnt - rem, rem, 0};
    }
}

// Stable positions: block c handles token chunk c in rounds of 256 pairs in (token, k) order;
// a pair's rank = pairs of its expert in earlier chunks (chunk base) + earlier rounds (running
// count) + earlier warps of the round (per-warp histograms) + earlier lanes (__match_any_sync).
__global__ void __launch_bounds__(256) k_pf_place(const int *ids, int T, int E, int K, const int *chunk_base, const int *offsets,
                                                  int *pos) {
    __shared__ int run[512];
    __shared__ unsigned short wh[8][512];
    const int c = blockIdx.x, tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
    for (int e = tid; e < E; e += 256) run[e] = 0;
    const long long p0 = (long long)c * kTokChunk * K, p1 = min((long long)T * K, p0 + (long long)kTokChunk * K);
    for (long long base = p0; base < p1; base += 256) {
        for (int i = tid; i < 8 * 512; i += 256) (&wh[0][0])[i] = 0;
        __syncthreads();
        const long long p = base + tid;
        const int e = p < p1 ? ids[p] : -1;
        const bool valid = e >= 0 && e < E;
        const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
        const int rank_lane = __popc(same & ((1u << lane) - 1u));
        if (valid && rank_lane == 0) wh[w][e] = (unsigned short)__popc(same);
        __syncthreads();
        if (valid) {
            int before = 0;
            for (int v = 0; v < w; ++v) before += wh[v][e];
            pos[p] = offsets[e] + chunk_base[(long long)c * E + e] + run[e] + before + rank_lane;
        } else if (p < p1) {
            pos[p] = -1;
        }
        __syncthreads();
        for (int e2 = tid; e2 < E; e2 += 256) {
            int s = 0;
#pragma unroll
            for (int v = 0; v < 8; ++v) s += wh[v][e2];
            run[e2] += s;
        }
        __syncthreads();
    }
}

// One block per token: FP16 copies of x times 2^k at the token's pair rows and at its shared
// row shared0 + t (16-byte chunks of 8 elements; H <= 4096). Row metadata: scale 2^-k, the
// token (shared rows: token + token_base) and the weight (shared rows: sigmoid(sg)).
__global__ void __launch_bounds__(256) k_pf_xprep(const float *__restrict__ x, int T, int H, int K, const int *pos, const float *weights,
                                                  const float *sg, int shared0, int token_base, __half *B, float *row_scale, int *row_token,
                                                  float *row_weight) {
    const int t = blockIdx.x, tid = threadIdx.x, nch = H / 8;
    __shared__ float red[8];
    float4 v[2][2];
    float mx = 0.0f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int ch = tid + 256 * u;
        if (ch < nch) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (long long)t * H) + 2 * ch;
            v[u][0] = __ldg(src);
            v[u][1] = __ldg(src + 1);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u][0].x), fabsf(v[u][0].y)), fmaxf(fabsf(v[u][0].z), fabsf(v[u][0].w))));
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u][1].x), fabsf(v[u][1].y)), fmaxf(fabsf(v[u][1].z), fabsf(v[u][1].w))));
        }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    // 2^k * max < 2^15 (FP16 keeps its 11 bits for the largest values)
    const unsigned bits = __float_as_uint(mx);
    int k = 15 - ((int)(bits >> 23) - 126);
    k = (bits >> 23) == 0 ? 0 : k;
    k = (bits >> 23) >= 255 ? 0 : k;
    k = max(-126, min(126, k));
    const float mul = __uint_as_float((unsigned)(k + 127) << 23), inv = __uint_as_float((unsigned)(127 - k) << 23);
    uint4 h[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const __half2 a = __floats2half2_rn(v[u][0].x * mul, v[u][0].y * mul), b = __floats2half2_rn(v[u][0].z * mul, v[u][0].w * mul);
        const __half2 c = __floats2half2_rn(v[u][1].x * mul, v[u][1].y * mul), d = __floats2half2_rn(v[u][1].z * mul, v[u][1].w * mul);
        h[u] = make_uint4(*reinterpret_cast<const unsigned *>(&a), *reinterpret_cast<const unsigned *>(&b),
                          *reinterpret_cast<const unsigned *>(&c), *reinterpret_cast<const unsigned *>(&d));
    }
    for (int kk = 0; kk <= K; ++kk) {
        const long long row = kk < K ? pos[(long long)t * K + kk] : (long long)shared0 + t;
        if (row < 0) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(B + row * H);
#pragma unroll
        for (int u = 0; u < 2; ++u)
            if (tid + 256 * u < nch) dst[tid + 256 * u] = h[u];
        if (tid == 0) {
            row_scale[row] = inv;
            row_token[row] = kk < K ? t : token_base + t;
            row_weight[row] = kk < K ? weights[(long long)t * K + kk] : ref_sigmoid(sg[t]);
        }
    }
}

// ------------------------------------------------------------------ expert parallel
// Rows are deduplicated per (token, destination rank): a token whose experts sit on a rank is
// sent there once, with the list of its pairs on that rank; the rank runs every pair and sums
// the weighted results per received row (pre-combine), so one row per (token, rank) comes back.
// Row metadata, kEpMetaFixed + 2 K ints: source token, pair count, 2^-k bits, 0, then per pair
// (local expert, weight bits); unused pair slots hold local expert -1.
constexpr int kEpMetaFixed = 4;
__host__ __device__ inline int ep_meta_ints(int K) { return kEpMetaFixed + 2 * K; }

// dst[t n + p] = p when token t has an expert on rank p (experts sharded evenly: rank p owns
// [p El, (p + 1) El)), else -1. n <= 32.
__global__ void k_ep_dest_rows(const int *ids, int T, int K, int E, const int *owner, int n, int *dst) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    unsigned mask = 0u;
    for (int kk = 0; kk < K; ++kk) {
        const int e = ids[(long long)t * K + kk];
        if (e >= 0 && e < E) mask |= 1u << owner[e];
    }
    for (int p = 0; p < n; ++p) dst[(long long)t * n + p] = (mask >> p) & 1u ? p : -1;
}

// One block per token: the token's FP16 row (times 2^k, largest |x| < 2^15) at each of its
// send rows, and each row's metadata (the token's pairs on that rank, in k order).
__global__ void __launch_bounds__(256) k_ep_pack(const float *__restrict__ x, int H, int K, const int *ids, const float *weights, int E,
                                                 const int *owner, const int *lidx, int n, const int *pos, __half *send_rows, int *send_meta) {
    const int t = blockIdx.x, tid = threadIdx.x, nch = H / 8, MS = ep_meta_ints(K);
    __shared__ float red[8];
    float4 v[2][2];
    float mx = 0.0f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int ch = tid + 256 * u;
        if (ch < nch) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (long long)t * H) + 2 * ch;
            v[u][0] = __ldg(src);
            v[u][1] = __ldg(src + 1);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u][0].x), fabsf(v[u][0].y)), fmaxf(fabsf(v[u][0].z), fabsf(v[u][0].w))));
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[u][1].x), fabsf(v[u][1].y)), fmaxf(fabsf(v[u][1].z), fabsf(v[u][1].w))));
        }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    const unsigned bits = __float_as_uint(mx);
    int k = 15 - ((int)(bits >> 23) - 126);
    k = (bits >> 23) == 0 ? 0 : k;
    k = (bits >> 23) >= 255 ? 0 : k;
    k = max(-126, min(126, k));
    const float mul = __uint_as_float((unsigned)(k + 127) << 23), inv = __uint_as_float((unsigned)(127 - k) << 23);
    uint4 h[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const __half2 a = __floats2half2_rn(v[u][0].x * mul, v[u][0].y * mul), b = __floats2half2_rn(v[u][0].z * mul, v[u][0].w * mul);
        const __half2 c = __floats2half2_rn(v[u][1].x * mul, v[u][1].y * mul), d = __floats2half2_rn(v[u][1].z * mul, v[u][1].w * mul);
        h[u] = make_uint4(*reinterpret_cast<const unsigned *>(&a), *reinterpret_cast<const unsigned *>(&b),
                          *reinterpret_cast<const unsigned *>(&c), *reinterpret_cast<const unsigned *>(&d));
    }
    for (int p = 0; p < n; ++p) {
        const int row = pos[(long long)t * n + p];
        if (row < 0) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(send_rows + (long long)row * H);
#pragma unroll
        for (int u = 0; u < 2; ++u)
            if (tid + 256 * u < nch) dst[tid + 256 * u] = h[u];
        if (tid == 0) {
            int *m = send_meta + (long long)row * MS;
            int np = 0;
            for (int kk = 0; kk < K; ++kk) {
                const int e = ids[(long long)t * K + kk];
                if (e >= 0 && e < E && owner[e] == p) {
                    m[kEpMetaFixed + 2 * np] = lidx[e];
                    m[kEpMetaFixed + 2 * np + 1] = __float_as_int(weights[(long long)t * K + kk]);
                    ++np;
                }
            }
            for (int j = np; j < K; ++j) {
                m[kEpMetaFixed + 2 * j] = -1;
                m[kEpMetaFixed + 2 * j + 1] = 0;
            }
            m[0] = t;
            m[1] = np;
            m[2] = __float_as_int(inv);
            m[3] = 0;
        }
    }
}

// Send counts per destination rank from the bucket offsets (the counts the ranks exchange).
__global__ void k_ep_send_counts(const int *off, int n, int *cnt) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p < n) cnt[p] = off[p + 1] - off[p];
}

// Local expert of every pair slot of the received rows: lid[i K + j] (-1 for an unused slot).
__global__ void k_ep_pair_experts(const int *meta, int R, int K, int *lid) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (long long)R * K) return;
    const long long i = q / K;
    lid[q] = meta[i * ep_meta_ints(K) + kEpMetaFixed + 2 * (q - i * K)];
}

// One warp per received row: its FP16 row at each of its pairs' positions among the local
// experts' B rows; every pair's GEMM output is added into row i of the result (pre-combine).
__global__ void k_ep_gather(const __half *recv_rows, const int *meta, int R, int K, int H, const int *rpos, __half *B, float *row_scale,
                            int *row_token, float *row_weight) {
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (i >= R) return;
    const int *m = meta + (long long)i * ep_meta_ints(K);
    const uint4 *src = reinterpret_cast<const uint4 *>(recv_rows + (long long)i * H);
    for (int j = 0; j < K; ++j) {
        const int p = rpos[(long long)i * K + j];
        if (p < 0) continue;
        uint4 *dst = reinterpret_cast<uint4 *>(B + (long long)p * H);
        for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
        if (lane == 0) {
            row_scale[p] = __int_as_float(m[2]);
            row_weight[p] = __int_as_float(m[kEpMetaFixed + 2 * j + 1]);
            row_token[p] = i;
        }
    }
}

// y[t] = shared row + the token's returned rows in rank order.
__global__ void k_ep_combine(const float *ret, const int *pos, int n, int H, const float *shared, float *y) {
    const int t = blockIdx.x;
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        float4 a = reinterpret_cast<const float4 *>(shared + (long long)t * H)[c];
        for (int p = 0; p < n; ++p) {
            const int row = pos[(long long)t * n + p];
            if (row < 0) continue;
            const float4 b = reinterpret_cast<const float4 *>(ret + (long long)row * H)[c];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        reinterpret_cast<float4 *>(y + (long long)t * H)[c] = a;
    }
}

}  // namespace pf

// ------------------------------------------------------------------ host
namespace {

struct PfScratch {
    float *logits, *sg;
    int *chunk_counts, *offsets, *pos, *row_token, *n_chunks;
    float *row_scale, *row_weight;
    pf::Chunk *chunks;
    __half *B, *hidden;
    float *tail;  // router logits: the last row tile's rows
};
size_t al(size_t n) { return (n + 255) & ~size_t(255); }
PfScratch carve(void *base, int T, int H, int F, int E, int K) {
    char *p = static_cast<char *>(base);
    PfScratch s;
    const long long rows = (long long)T * K + T;
    const int n_tc = (T + pf::kTokChunk - 1) / pf::kTokChunk;
    const int max_chunks = E + (T * K) / pf::kMaxN + (T + pf::kMaxN - 1) / pf::kMaxN + 1;
    auto take = [&](size_t bytes) {
        char *r = p;
        p += al(bytes);
        return r;
    };
    s.logits = (float *)take(sizeof(float) * T * E);
    s.sg = (float *)take(sizeof(float) * T);
    s.chunk_counts = (int *)take(sizeof(int) * (size_t)n_tc * E);
    s.offsets = (int *)take(sizeof(int) * (E + 1));
    s.pos = (int *)take(sizeof(int) * (size_t)T * K);
    s.row_token = (int *)take(sizeof(int) * rows);
    s.n_chunks = (int *)take(sizeof(int));
    s.row_scale = (float *)take(sizeof(float) * rows);
    s.row_weight = (float *)take(sizeof(float) * rows);
    s.chunks = (pf::Chunk *)take(sizeof(pf::Chunk) * max_chunks);
    s.B = (__half *)take(sizeof(__half) * rows * H);
    s.hidden = (__half *)take(sizeof(__half) * rows * F);
    s.tail = (float *)take(sizeof(float) * pf::kLgR * H);
    return s;
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}
bool encode(CUtensorMap *m, CUtensorMapDataType dt, int rank, const void *base, const unsigned long long *dims,
            const unsigned long long *strides, const unsigned *box, CUtensorMapSwizzle sw) {
    auto fn = encoder();
    if (!fn) return false;
    cuuint64_t d[3] = {0, 0, 0}, st[2] = {0, 0};
    cuuint32_t b[3] = {1, 1, 1}, es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        if (i + 1 < rank) st[i] = strides[i];
    }
    return fn(m, dt, rank, const_cast<void *>(base), d, st, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Router logits: the tail rows, the tensor maps, one persistent launch (one CTA per SM at most).
cudaError_t launch_logits(const MoeLayerDev &L, const float *x, int T, float *logits, float *sg, float *tail, int sms, cudaStream_t s,
                          unsigned *err) {
    const int H = L.width, E = L.experts;
    const int n_full = E / pf::kLgR;
    pf::k_lg_tail<<<pf::kLgR, 256, 0, s>>>(L.router, L.shared_gate, E, H, n_full * pf::kLgR, tail);
    pf::LgMaps M;
    const unsigned long long rdims[2] = {(unsigned long long)H, (unsigned long long)std::max(1, E)},
                             tdims[2] = {(unsigned long long)H, (unsigned long long)pf::kLgR}, xdims[2] = {(unsigned long long)H, (unsigned long long)T};
    const unsigned long long rstr[1] = {(unsigned long long)H * 4};
    const unsigned rbox[2] = {pf::kLgKC, pf::kLgR}, xbox[2] = {pf::kLgKC, pf::kLgT};
    if (!encode(&M.router, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, L.router, rdims, rstr, rbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&M.tail, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, tail, tdims, rstr, rbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode(&M.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, x, xdims, rstr, xbox, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    static int ready_device = -1;
    int dev = 0;
    STRATA_CUDA_TRY(cudaGetDevice(&dev));
    if (ready_device != dev) {
        STRATA_CUDA_TRY(cudaFuncSetAttribute(pf::k_pf_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf::kLgSmemLimit));
        ready_device = dev;
    }
    // row tiles per work item: kLgGroup share one copy of the item's x; with too few items to
    // fill the SMs (small batches), one tile per item
    const int n_rt = n_full + 1, n_tt = (T + pf::kLgT - 1) / pf::kLgT;
    const int group = (long long)n_tt * ((n_rt + pf::kLgGroup - 1) / pf::kLgGroup) >= sms ? pf::kLgGroup : 1;
    const long long n_items = (long long)n_tt * ((n_rt + group - 1) / group);
    const int grid = (int)std::min<long long>(n_items, std::max(1, sms));
    pf::k_pf_logits<<<grid, pf::kLgThreads, pf::logits_smem(H), s>>>(M, L, T, pf::logits_stages(H), group, logits, sg, err, 1ull << 24,
                                                                      kNegZero2);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_gemm(const pf::GemmParams &p, int grid, cudaStream_t s) {
    const size_t smem = sizeof(pf::GemmSmem) + 1024;
    static int ready_device = -1;
    int dev = 0;
    STRATA_CUDA_TRY(cudaGetDevice(&dev));
    if (ready_device != dev) {
        STRATA_CUDA_TRY(cudaFuncSetAttribute(pf::k_pf_gemm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        ready_device = dev;
    }
    pf::k_pf_gemm<MODE><<<grid, pf::kGemmThreads, smem, s>>>(p);
    return cudaGetLastError();
}

// The gate/up and down GEMMs over a chunk list: B rows (FP16, b_rows of them) with their
// scale, token and weight; hidden [b_rows][F]; y[token][H] += weight * down. `experts`
// blobs start at L.blobs. marks (nullable): events after each GEMM.
cudaError_t launch_moe_gemms(const MoeLayerDev &L, int experts, const pf::Chunk *chunks, const int *n_chunks, long long b_rows, const __half *B,
                             __half *hidden, const float *row_scale, const int *row_token, const float *row_weight, float *y, int grid,
                             cudaStream_t s, unsigned *err, cudaEvent_t *marks) {
    const int H = L.width, F = L.ff;
    const long long bb = L.blob_words * 4;
    const long long d_codes = 2LL * F * H / 4, gu_scales = 3LL * F * H / 4, d_scales = gu_scales + 2LL * F * (H / 64) * 2;
    const unsigned char *blobs = reinterpret_cast<const unsigned char *>(L.blobs), *shared = reinterpret_cast<const unsigned char *>(L.shared_blob);
    for (int mode = 0; mode < 2; ++mode) {
        pf::GemmParams p;
        std::memset(&p, 0, sizeof p);
        p.chunks = chunks;
        p.n_chunks = n_chunks;
        p.blobs = blobs;
        p.shared = shared;
        p.blob_bytes = bb;
        p.K = mode == 0 ? H : F;
        p.rows_total = mode == 0 ? 2 * F : H;
        p.NM = p.rows_total / 128;
        p.codes_off = mode == 0 ? 0 : d_codes;
        p.scales_off = mode == 0 ? gu_scales : d_scales;
        p.row_scale = row_scale;
        p.row_token = row_token;
        p.row_weight = row_weight;
        p.hidden = hidden;
        p.y = y;
        p.err = err;
        p.spin_limit = 1ull << 22;
        const unsigned long long cdims[3] = {(unsigned long long)p.K / 4, (unsigned long long)p.rows_total, (unsigned long long)max(1, experts)};
        const unsigned long long cstr[2] = {(unsigned long long)p.K / 4, (unsigned long long)bb};
        const unsigned cbox[3] = {64, 128, 1};
        const unsigned long long sdims[3] = {(unsigned long long)p.K / 4, (unsigned long long)p.rows_total, 1ull};
        if (!encode(&p.tm_codes[0], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (blobs ? blobs : shared) + p.codes_off, cdims, cstr, cbox,
                    CU_TENSOR_MAP_SWIZZLE_64B) ||
            !encode(&p.tm_codes[1], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, shared + p.codes_off, sdims, cstr, cbox, CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
        const void *bmat = mode == 0 ? (const void *)B : (const void *)hidden;
        const unsigned long long bdims[2] = {(unsigned long long)p.K, (unsigned long long)max(1LL, b_rows)};
        const unsigned long long bstr[1] = {(unsigned long long)p.K * 2};
        const unsigned bbox[2] = {64, 16}, bbox64[2] = {64, 64};
        if (!encode(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, bmat, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode(&p.tm_b64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, bmat, bdims, bstr, bbox64, CU_TENSOR_MAP_SWIZZLE_128B))
            return cudaErrorInvalidValue;
        STRATA_CUDA_TRY(mode == 0 ? launch_gemm<pf::kGateUp>(p, grid, s) : launch_gemm<pf::kDown>(p, grid, s));
        if (marks) STRATA_CUDA_TRY(cudaEventRecord(marks[mode], s));
    }
    return cudaSuccess;
}

}  // namespace

size_t moe_prefill_scratch_bytes(int tokens, int width, int ff, int experts, int topK) {
    const long long rows = (long long)tokens * topK + tokens;
    const int n_tc = (tokens + pf::kTokChunk - 1) / pf::kTokChunk;
    const int max_chunks = experts + (tokens * topK) / pf::kMaxN + (tokens + pf::kMaxN - 1) / pf::kMaxN + 1;
    return al(sizeof(float) * tokens * experts) + al(sizeof(float) * tokens) + al(sizeof(int) * (size_t)n_tc * experts) +
           al(sizeof(int) * (experts + 1)) + al(sizeof(int) * (size_t)tokens * topK) + al(sizeof(int) * rows) + al(sizeof(int)) +
           al(sizeof(float) * rows) * 2 + al(sizeof(pf::Chunk) * max_chunks) + al(sizeof(__half) * rows * width) +
           al(sizeof(__half) * rows * ff) + al(sizeof(float) * pf::kLgR * width);
}

size_t moe_logits_tail_bytes(int width) { return sizeof(float) * pf::kLgR * width; }

cudaError_t moe_route_exact(const MoeLayerDev &L, const float *x, int T, float *logits, float *sg, float *tail, int *ids, float *weights,
                            int grid, cudaStream_t s, unsigned *err) {
    STRATA_CUDA_TRY(launch_logits(L, x, T, logits, sg, tail, grid, s, err));
    pf::k_pf_route<<<(T + 3) / 4, 128, 0, s>>>(logits, T, L.experts, L.topK, ids, weights);
    return cudaGetLastError();
}

bool moe_prefill_supported(int width, int ff, int experts, int topK) {
    return ((width == 2048 && ff == 512) || (width == 2560 && ff == 640)) && experts <= 512 && topK <= 32;
}

cudaError_t moe_forward_prefill(const MoeLayerDev &L, const float *x, int T, float *y, int *ids, float *weights, void *scratch, int grid,
                                cudaStream_t s, unsigned *err, cudaEvent_t *marks) {
    auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], s) : cudaSuccess; };
    STRATA_CUDA_TRY(mark(0));
    const int H = L.width, F = L.ff, E = L.experts, K = L.topK;
    const long long rows = (long long)T * K + T;
    PfScratch S = carve(scratch, T, H, F, E, K);
    const int n_tc = (T + pf::kTokChunk - 1) / pf::kTokChunk;
    STRATA_CUDA_TRY(launch_logits(L, x, T, S.logits, S.sg, S.tail, grid, s, err));
    pf::k_pf_route<<<(T + 3) / 4, 128, 0, s>>>(S.logits, T, E, K, ids, weights);
    pf::k_pf_count<<<n_tc, 256, 0, s>>>(ids, T, E, K, S.chunk_counts);
    pf::k_pf_scan<<<1, 512, 0, s>>>(S.chunk_counts, n_tc, T, T * K, E, S.offsets, S.chunks, S.n_chunks);
    pf::k_pf_place<<<n_tc, 256, 0, s>>>(ids, T, E, K, S.chunk_counts, S.offsets, S.pos);
    pf::k_pf_xprep<<<T, 256, 0, s>>>(x, T, H, K, S.pos, weights, S.sg, T * K, 0, S.B, S.row_scale, S.row_token, S.row_weight);
    STRATA_CUDA_TRY(cudaGetLastError());
    STRATA_CUDA_TRY(cudaMemsetAsync(y, 0, sizeof(float) * (size_t)T * H, s));
    STRATA_CUDA_TRY(mark(1));

    STRATA_CUDA_TRY(launch_moe_gemms(L, L.experts, S.chunks, S.n_chunks, rows, S.B, S.hidden, S.row_scale, S.row_token, S.row_weight, y,
                                     grid, s, err, marks ? marks + 2 : nullptr));
    return cudaSuccess;
}


// ------------------------------------------------------------------ expert parallel (host)
// One layer over the ranks of `c`: this rank's T tokens in, its y out; L.blobs holds the
// c->n_local experts this rank owns under the communicator's placement, in ascending id
// (L.experts is the layer's total).
// Stages: exact routing; one row per (token, destination rank) bucketed by rank (stable,
// token-major), packed as an FP16 row with its pair list {local expert, weight} and 2^-k;
// counts, then rows, exchanged by grouped ncclSend/ncclRecv; the received rows' pairs grouped
// by local expert and run through the tensor-core GEMMs together with this rank's shared-
// expert rows, the down GEMM adding each pair's weighted result into its received row (pre-
// combine); one row per received row sent back; y[t] = shared row + the token's returned rows
// in rank order. The receive sizes are read back on the host (as the reference reads its
// routing back, src/engine.js:137). marks (nullable): six events at start, after packing,
// before the GEMMs, after gate/up, after down, after the combine.
int moe_forward_ep(const MoeLayerDev &L, EpComm *c, const float *x, int T, float *y, int *ids, float *weights, int grid, cudaStream_t s,
                   unsigned *err, std::string *msg, cudaEvent_t *marks) {
    const int H = L.width, F = L.ff, E = L.experts, K = L.topK, n = c->n, El = c->n_local;
    cudaError_t e = cudaSuccess;
    if (c->placed_experts != E || El < 1) {
        *msg = "no expert placement for this layer's expert count";
        return 2;
    }
    const int *owner = c->d_place, *lidx = c->d_place + E;
    if (c->failed) {
        *msg = "the expert-parallel communicator failed earlier (" + c->failure + "); call strata_ep_init again";
        return 3;
    }
    auto fail_cuda = [&](cudaError_t ce, const char *what) {
        *msg = std::string(what) + ": " + cudaGetErrorString(ce);
        return 2;
    };
    // a failed exchange leaves the peers in an unknown state: the communicator is aborted
    auto fail_ep = [&](const char *what) {
        *msg = std::string(what) + ": " + *msg;
        c->fail(*msg);
        return 3;
    };
    EpTransport &tr = *c->t;
#define EP_CUDA(x, what)                              \
    do {                                              \
        cudaError_t _c = (x);                         \
        if (_c != cudaSuccess) return fail_cuda(_c, what); \
    } while (0)
#define EP_XCHG(what)                                  \
    do {                                               \
        if (tr.group_end(s, msg)) return fail_ep(what); \
    } while (0)
#define EP_GET(ptr, type, i, count)                                                   \
    type *ptr = static_cast<type *>(c->get(i, sizeof(type) * (size_t)(count) + 16, e)); \
    if (!ptr) return fail_cuda(e, "cudaMalloc");
    const int n_tc = (T + pf::kTokChunk - 1) / pf::kTokChunk;
#define EP_MARK(i)                                                                   \
    do {                                                                             \
        if (marks) EP_CUDA(cudaEventRecord(marks[i], s), "cudaEventRecord");        \
    } while (0)
    // 1. routing
    EP_MARK(0);
    EP_GET(logits, float, 0, (long long)T * E);
    EP_GET(sg, float, 1, T);
    EP_GET(tail, float, 24, (long long)pf::kLgR * H);
    EP_CUDA(launch_logits(L, x, T, logits, sg, tail, grid, s, err), "router logits");
    pf::k_pf_route<<<(T + 3) / 4, 128, 0, s>>>(logits, T, E, K, ids, weights);
    // 2. one row per (token, destination rank): buckets by rank (stable, token-major), packed
    //    FP16 rows and their pair lists
    if (n > 32) {
        *msg = "expert parallelism supports at most 32 ranks";
        return 2;
    }
    const long long TN = (long long)T * n;
    const int MS = pf::ep_meta_ints(K);
    EP_GET(dest, int, 2, TN);
    EP_GET(cc, int, 3, (long long)n_tc * n);
    EP_GET(off, int, 4, n + 1);
    EP_GET(pos, int, 5, TN);
    EP_GET(dchunks, pf::Chunk, 6, TN / pf::kMaxN + n + 2);
    EP_GET(dn, int, 7, 1);
    pf::k_ep_dest_rows<<<(T + 255) / 256, 256, 0, s>>>(ids, T, K, E, owner, n, dest);
    pf::k_pf_count<<<n_tc, 256, 0, s>>>(dest, T, n, n, cc);
    pf::k_pf_scan<<<1, 512, 0, s>>>(cc, n_tc, 0, 0, n, off, dchunks, dn);
    pf::k_pf_place<<<n_tc, 256, 0, s>>>(dest, T, n, n, cc, off, pos);
    EP_GET(send_rows, __half, 8, TN * H);
    EP_GET(send_meta, int, 9, TN * MS);
    pf::k_ep_pack<<<T, 256, 0, s>>>(x, H, K, ids, weights, E, owner, lidx, n, pos, send_rows, send_meta);
    EP_MARK(1);
    // 3. counts exchange; one host read of the send offsets and the receive counts
    EP_GET(d_cnt, int, 10, 2 * n);
    pf::k_ep_send_counts<<<(n + 127) / 128, 128, 0, s>>>(off, n, d_cnt);
    EP_CUDA(cudaGetLastError(), "routing and packing kernels");
    tr.group_start();
    for (int p = 0; p < n; ++p) {
        tr.send(d_cnt + p, sizeof(int), p);
        tr.recv(d_cnt + n + p, sizeof(int), p);
    }
    EP_XCHG("counts exchange");
    EP_CUDA(cudaMemcpyAsync(c->h_off, off, sizeof(int) * (n + 1), cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    EP_CUDA(cudaMemcpyAsync(c->h_off + n + 1, d_cnt + n, sizeof(int) * n, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    if (tr.wait(s, msg)) return fail_ep("waiting for the receive counts");
    std::vector<int> soff(n + 1), sc(n), rc(n), roff(n + 1);
    for (int i = 0; i <= n; ++i) soff[i] = c->h_off[i];
    for (int i = 0; i < n; ++i) sc[i] = soff[i + 1] - soff[i];
    roff[0] = 0;
    for (int i = 0; i < n; ++i) {
        rc[i] = c->h_off[n + 1 + i];
        roff[i + 1] = roff[i] + rc[i];
    }
    const int R = roff[n];
    // 4. rows exchange
    EP_GET(recv_rows, __half, 11, (long long)max(R, 1) * H);
    EP_GET(recv_meta, int, 12, (long long)max(R, 1) * MS);
    tr.group_start();
    for (int p = 0; p < n; ++p) {
        if (sc[p]) {
            tr.send(send_rows + (long long)soff[p] * H, sizeof(__half) * sc[p] * H, p);
            tr.send(send_meta + (long long)soff[p] * MS, sizeof(int) * sc[p] * MS, p);
        }
        if (rc[p]) {
            tr.recv(recv_rows + (long long)roff[p] * H, sizeof(__half) * rc[p] * H, p);
            tr.recv(recv_meta + (long long)roff[p] * MS, sizeof(int) * rc[p] * MS, p);
        }
    }
    EP_XCHG("dispatch");
    // 5. the received rows' pairs grouped by local expert (pair slot i K + j of row i), this
    //    rank's shared-expert rows after them; the GEMMs add every pair of received row i into
    //    Y[i] (pre-combine) and token t's shared expert into Y[R + t]
    const long long QK = (long long)R * K, brows = QK + T;
    const int n_tc2 = max(1, (R + pf::kTokChunk - 1) / pf::kTokChunk);
    const int max_chunks = El + (int)(brows / pf::kMaxN) + 4;
    EP_GET(lid, int, 13, max(QK, 1LL));
    EP_GET(cc2, int, 14, (long long)n_tc2 * El);
    EP_GET(off2, int, 15, El + 1);
    EP_GET(rpos, int, 16, max(QK, 1LL));
    EP_GET(chunks, pf::Chunk, 17, max_chunks);
    EP_GET(nchunks, int, 18, 1);
    EP_GET(B, __half, 19, brows * H);
    EP_GET(hidden, __half, 20, brows * F);
    EP_GET(rmeta, float, 21, 3 * brows);  // row scale, Y row (as int), weight
    EP_GET(Y, float, 22, ((long long)R + T) * H);
    EP_GET(ret, float, 23, max(TN, 1LL) * H);
    float *row_scale = rmeta, *row_weight = rmeta + 2 * brows;
    int *row_token = reinterpret_cast<int *>(rmeta + brows);
    if (R > 0) {
        pf::k_ep_pair_experts<<<(unsigned)((QK + 255) / 256), 256, 0, s>>>(recv_meta, R, K, lid);
        pf::k_pf_count<<<n_tc2, 256, 0, s>>>(lid, R, El, K, cc2);
    }
    pf::k_pf_scan<<<1, 512, 0, s>>>(cc2, R > 0 ? n_tc2 : 0, T, (int)QK, El, off2, chunks, nchunks);
    if (R > 0) {
        pf::k_pf_place<<<n_tc2, 256, 0, s>>>(lid, R, El, K, cc2, off2, rpos);
        pf::k_ep_gather<<<(R + 7) / 8, 256, 0, s>>>(recv_rows, recv_meta, R, K, H, rpos, B, row_scale, row_token, row_weight);
    }
    pf::k_pf_xprep<<<T, 256, 0, s>>>(x, T, H, 0, nullptr, weights, sg, (int)QK, R, B, row_scale, row_token, row_weight);
    EP_CUDA(cudaMemsetAsync(Y, 0, sizeof(float) * ((long long)R + T) * H, s), "cudaMemsetAsync");
    EP_CUDA(cudaGetLastError(), "expert grouping kernels");
    MoeLayerDev Ll = L;
    Ll.experts = El;
    EP_MARK(2);
    EP_CUDA(launch_moe_gemms(Ll, El, chunks, nchunks, brows, B, hidden, row_scale, row_token, row_weight, Y, grid, s, err,
                             marks ? marks + 3 : nullptr),
            "expert GEMMs");
    // 6. one pre-combined row per received row back to its token's rank
    tr.group_start();
    for (int p = 0; p < n; ++p) {
        if (rc[p]) tr.send(Y + (long long)roff[p] * H, sizeof(float) * rc[p] * H, p);
        if (sc[p]) tr.recv(ret + (long long)soff[p] * H, sizeof(float) * sc[p] * H, p);
    }
    EP_XCHG("return");
    // 7. combine: shared row + the returned rows in rank order
    pf::k_ep_combine<<<T, 128, 0, s>>>(ret, pos, n, H, Y + (long long)R * H, y);
    EP_CUDA(cudaGetLastError(), "combine");
    EP_MARK(5);
#undef EP_MARK
#undef EP_CUDA
#undef EP_XCHG
#undef EP_GET
    return 0;
}

}  // namespace strata
