// Reference-compatible entries for strata_run(): the kernels that src/ops.js, src/engine.js
// and src/prefill.js dispatch by name (kernels/strata.cu), with the same parameter names,
// the same dispatch grid of 64-lane workgroups and bit-identical F32 results.
//
// B200 shape: a reference workgroup is one warp (thread t owns virtual lanes t and t+32, the
// s=32 tree step is in-thread, the rest are shuffles), four workgroups per 128-thread block.
// Every global access is bounds-checked against the buffer it came from: an index outside
// the buffer reads 0 / skips the write and sets the context's device error word, which the
// host reports at the next synchronisation. No argument can make these kernels fault.
#include "common.cuh"
#include "kernels.h"
#include "route.cuh"
#include "compat.cuh"
#include "q2mma.cuh"

#include <algorithm>

namespace strata {
namespace {

// ---------------------------------------------------------------- element kernels
// (one reference lane per thread: i = blockIdx.x * 64 + threadIdx.x over the x extent)

__global__ void k_unpack_half(Grid g, UB Packed, FB Values, int count, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (long long)g.x * STRATA_LANES && i < count) Values.set(i, half_of(Packed, i, err), err);
}

__global__ void k_expert_scales(Grid g, UB Blob, FB Scales, int offset, int count, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (long long)g.x * STRATA_LANES && i < count) Scales.set(i, half_of(Blob, offset + i, err), err);
}

__global__ void k_elementwise(Grid g, FB A, FB B, FB Y, int n, int mode, float scale, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g.x * STRATA_LANES || i >= n) return;
    float a = __fmul_rn(A.get(i, err), scale), v = a;
    if (mode == 1) v = ref_silu(a);
    if (mode == 2) v = ref_sigmoid(a);
    if (mode == 3) v = __fmul_rn(ref_silu(a), B.get(i, err));
    if (mode == 4) v = __fmul_rn(a, ref_sigmoid(B.get(i, err)));
    if (mode == 5) v = __fadd_rn(a, B.get(i, err));
    Y.set(i, v, err);
}

__global__ void k_moe_combine(Grid g, FB Parts, FB Weights, FB Shared, FB SharedGate, FB Y, int width, int count, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g.x * STRATA_LANES || i >= width) return;
    float value = __fmul_rn(Shared.get(i, err), ref_sigmoid(SharedGate.get(0, err)));
    for (int k = 0; k < count; ++k) value = __fadd_rn(value, __fmul_rn(Parts.get((long long)k * width + i, err), Weights.get(k, err)));
    Y.set(i, value, err);
}

__global__ void k_moe_combine_batch(Grid g, FB Parts, FB Weights, FB Shared, FB SharedGate, FB Y, int width, int count, int tokens,
                                    unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g.x * STRATA_LANES || i >= (long long)width * tokens) return;
    long long token = i / width, d = i % width;
    float value = __fmul_rn(Shared.get(i, err), ref_sigmoid(SharedGate.get(token, err)));
    for (int k = 0; k < count; ++k)
        value = __fadd_rn(value, __fmul_rn(Parts.get((token * count + k) * width + d, err), Weights.get(token * count + k, err)));
    Y.set(i, value, err);
}

__global__ void k_gather_rows(Grid g, FB X, IB Indices, FB Y, int width, int rows, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g.x * STRATA_LANES || i >= (long long)width * rows) return;
    Y.set(i, X.get((long long)Indices.get(i / width, err) * width + i % width, err), err);
}

__global__ void k_scatter_rows(Grid g, FB X, IB Indices, FB Y, int width, int rows, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)g.x * STRATA_LANES || i >= (long long)width * rows) return;
    Y.set((long long)Indices.get(i / width, err) * width + i % width, X.get(i, err), err);
}

// ---------------------------------------------------------------- workgroup kernels

// kernels/strata.cu:156-165
__global__ void k_project(Grid g, FB X, FB W, FB Y, int cols, int rows, int tokens, int outputStride, int outputOffset, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group_y_first(g, row, token, z)) return;
    if (!((int)row < rows && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    const long long wb = (long long)row * cols, xb = (long long)token * cols;
    float r;
    if (covers(W, wb, cols) && covers(X, xb, cols)) {
        r = lane_dot(W.p + wb, X.p + xb, cols, t);
    } else {  // some index falls outside a buffer: the checked loop reports it
        float lo = 0.0f, hi = 0.0f;
        for (int i = t; i < cols; i += STRATA_LANES) {
            lo = __fadd_rn(lo, __fmul_rn(W.get(wb + i, err), X.get(xb + i, err)));
            if (i + 32 < cols) hi = __fadd_rn(hi, __fmul_rn(W.get(wb + i + 32, err), X.get(xb + i + 32, err)));
        }
        r = tree64(lo, hi);
    }
    if (t == 0) Y.set((long long)token * outputStride + outputOffset + row, r, err);
}

// The same projection for one token (decode), bandwidth-shaped: a half-warp per output row, 16
// rows per block. Thread u of a half-warp holds the reference's lanes 4u .. 4u + 3 (elements
// 4u + 64k .. 4u + 64k + 3 of round k: one 16-byte load of the weights and one of the input
// per round, eight rounds in flight), each lane's products added in round order from 0. The
// tree partial[l] += partial[l + s] (s = 32 .. 4) is a shuffle by s / 4 threads within the
// half-warp; s = 2 and 1 join the lanes of thread 0. Same sums and roundings as k_project.
// The host launches it when cols is a multiple of 64, both rows are 16-byte aligned and the
// buffers cover every row read.
constexpr int kGemvThreads = 256, kGemvRows = kGemvThreads / 16;
__global__ void __launch_bounds__(kGemvThreads) k_project_gemv(FB X, FB W, FB Y, int cols, int rows, int outputOffset, unsigned *err) {
    if (threadIdx.x == 0) {  // the block's weight rows, while the previous kernel finishes
        const int r0 = blockIdx.x * kGemvRows, nr = min(kGemvRows, rows - r0);
        if (nr > 0) prefetch_l2(W.p + (long long)r0 * cols, (unsigned long long)nr * cols * 4);
    }
    dep_enter();
    const int hw = threadIdx.x >> 4, u = threadIdx.x & 15;
    const int row = blockIdx.x * kGemvRows + hw;
    if (row >= rows) return;  // whole half-warps leave together (the shuffles use 16-lane masks)
    const unsigned mask = 0xffffu << (threadIdx.x & 16);
    const float4 *w4 = reinterpret_cast<const float4 *>(W.p + (long long)row * cols) + u;
    const float4 *x4 = reinterpret_cast<const float4 *>(X.p) + u;
    const int R = cols / 64;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int k = 0;
    for (; k + 8 <= R; k += 8) {
        float4 wv[8], xv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            wv[i] = __ldcs(w4 + 16 * (k + i));  // streamed once: no reuse in the caches
            xv[i] = __ldg(x4 + 16 * (k + i));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            a0 = __fadd_rn(a0, __fmul_rn(wv[i].x, xv[i].x));
            a1 = __fadd_rn(a1, __fmul_rn(wv[i].y, xv[i].y));
            a2 = __fadd_rn(a2, __fmul_rn(wv[i].z, xv[i].z));
            a3 = __fadd_rn(a3, __fmul_rn(wv[i].w, xv[i].w));
        }
    }
    for (; k < R; ++k) {
        const float4 wv = __ldcs(w4 + 16 * k), xv = __ldg(x4 + 16 * k);
        a0 = __fadd_rn(a0, __fmul_rn(wv.x, xv.x));
        a1 = __fadd_rn(a1, __fmul_rn(wv.y, xv.y));
        a2 = __fadd_rn(a2, __fmul_rn(wv.z, xv.z));
        a3 = __fadd_rn(a3, __fmul_rn(wv.w, xv.w));
    }
#pragma unroll
    for (int s = 8; s > 0; s >>= 1) {  // reference levels 32, 16, 8, 4
        a0 = __fadd_rn(a0, __shfl_down_sync(mask, a0, s, 16));
        a1 = __fadd_rn(a1, __shfl_down_sync(mask, a1, s, 16));
        a2 = __fadd_rn(a2, __shfl_down_sync(mask, a2, s, 16));
        a3 = __fadd_rn(a3, __shfl_down_sync(mask, a3, s, 16));
    }
    if (u == 0) {
        a0 = __fadd_rn(a0, a2);  // level 2
        a1 = __fadd_rn(a1, a3);
        Y.set((long long)outputOffset + row, __fadd_rn(a0, a1), err);  // level 1
    }
}

// The same one-token projection as a weight stream, for matrices of at least 512 rows. Block b
// owns the contiguous rows [b n, b n + n) and pulls them, one bulk copy (cp.async.bulk) per row,
// through row slots in shared memory: up to about 200 KB in flight per SM, independent of
// registers. The first copies are requested before dep_enter() (kernels never write weights), so
// they stream while the previous kernel finishes. Each of the first `halves` half-warps owns
// `depth` slots and the block rows h, h + halves, ... (its k-th row in slot h depth + k % depth);
// it forms each row exactly as k_project_gemv does (thread u holds the reference's lanes
// 4u .. 4u + 3, the same chains and tree), reading the row from its slot and the input from a
// copy staged once per block, then refills the slot with its row k + depth. A slot is only ever
// waited on and refilled by its own half-warp, in order, so the full barrier's parity is never
// ambiguous. Every wait is bounded: past the limit the block records kErrWaitTimeout, stops, and
// thread 0 waits (bounded) for the copies that were issued before the block exits.
constexpr int kStreamThreads = 256, kStreamHalves = kStreamThreads / 16, kStreamMaxSlots = 64, kStreamMaxDepth = 4;
constexpr size_t kStreamSmem = 200 * 1024;
constexpr unsigned long long kStreamSpin = 1ull << 20;
__global__ void __launch_bounds__(kStreamThreads, 1) k_project_stream(FB X, FB W, FB Y, int cols, int rows, int rows_per_block, int halves,
                                                                      int depth, int outputOffset, unsigned *err) {
    extern __shared__ __align__(128) float stream_smem[];  // [cols] input, then [halves * depth][cols] weight rows
    __shared__ __align__(8) unsigned long long full[kStreamMaxSlots];
    __shared__ int issued[kStreamMaxSlots];  // copies issued into each slot
    __shared__ int failed;
    const int r0 = blockIdx.x * rows_per_block, n = max(0, min(rows_per_block, rows - r0));
    const int slots = halves * depth, stride = halves * depth;  // a half-warp's row k + depth is block row i + stride
    const unsigned row_bytes = (unsigned)cols * 4;
    float *xs = stream_smem, *ring = stream_smem + cols;
    const float *wrow0 = W.p + (long long)r0 * cols;
    if (threadIdx.x == 0) {
        failed = 0;
        for (int sl = 0; sl < slots; ++sl) {
            q2::mbar_init(&full[sl], 1);
            issued[sl] = 0;
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int h = 0; h < halves; ++h)  // weights only: before the dependency wait
            for (int k = 0; k < depth && h + k * halves < n; ++k) {
                const int sl = h * depth + k;
                q2::mbar_expect(&full[sl], row_bytes);
                q2::bulk_copy(ring + (size_t)sl * cols, wrow0 + (long long)(h + k * halves) * cols, row_bytes, &full[sl]);
                issued[sl] = 1;
            }
    }
    dep_enter();
    {
        const float4 *x4 = reinterpret_cast<const float4 *>(X.p);
        float4 *xs4 = reinterpret_cast<float4 *>(xs);
        for (int k = threadIdx.x; k < cols / 4; k += kStreamThreads) xs4[k] = x4[k];
    }
    __syncthreads();
    auto wait_bar = [&](unsigned long long *bar, unsigned parity) -> bool {
        for (unsigned long long i = 0;; ++i) {
            if (q2::mbar_try(bar, parity)) return true;
            if (i > kStreamSpin || *(volatile int *)&failed) return false;
        }
    };
    const int hw = threadIdx.x >> 4, u = threadIdx.x & 15;
    const unsigned mask = 0xffffu << (threadIdx.x & 16);
    const int R = cols / 64;
    if (hw < halves)
        for (int k = 0, i = hw; i < n; ++k, i += halves) {
            const int sl = hw * depth + k % depth;
            if (__any_sync(mask, !wait_bar(&full[sl], (k / depth) & 1))) {
                if (u == 0) {
                    failed = 1;
                    raise_error(err, kErrWaitTimeout);
                }
                break;
            }
            const float4 *w4 = reinterpret_cast<const float4 *>(ring + (size_t)sl * cols) + u;
            const float4 *x4 = reinterpret_cast<const float4 *>(xs) + u;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 8
            for (int r = 0; r < R; ++r) {
                const float4 wv = w4[16 * r], xv = x4[16 * r];
                a0 = __fadd_rn(a0, __fmul_rn(wv.x, xv.x));
                a1 = __fadd_rn(a1, __fmul_rn(wv.y, xv.y));
                a2 = __fadd_rn(a2, __fmul_rn(wv.z, xv.z));
                a3 = __fadd_rn(a3, __fmul_rn(wv.w, xv.w));
            }
            __syncwarp(mask);  // the slot has been read by all 16 threads
            if (u == 0 && i + stride < n) {  // refill it (it was read through the generic proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                q2::mbar_expect(&full[sl], row_bytes);
                q2::bulk_copy(ring + (size_t)sl * cols, wrow0 + (long long)(i + stride) * cols, row_bytes, &full[sl]);
                issued[sl] = k / depth + 2;
            }
#pragma unroll
            for (int sh = 8; sh > 0; sh >>= 1) {  // reference levels 32, 16, 8, 4
                a0 = __fadd_rn(a0, __shfl_down_sync(mask, a0, sh, 16));
                a1 = __fadd_rn(a1, __shfl_down_sync(mask, a1, sh, 16));
                a2 = __fadd_rn(a2, __shfl_down_sync(mask, a2, sh, 16));
                a3 = __fadd_rn(a3, __shfl_down_sync(mask, a3, sh, 16));
            }
            if (u == 0) {
                a0 = __fadd_rn(a0, a2);  // level 2
                a1 = __fadd_rn(a1, a3);
                Y.p[(long long)outputOffset + r0 + i] = __fadd_rn(a0, a1);  // level 1
            }
        }
    __syncthreads();
    if (threadIdx.x == 0 && failed)  // copies still in flight must land before the block exits
        for (int sl = 0; sl < slots; ++sl)
            for (unsigned long long k = 0; issued[sl] > 0 && !q2::mbar_try(&full[sl], (issued[sl] - 1) & 1) && k <= kStreamSpin; ++k) {
            }
}

// The same projection for dispatches with few (row, token) pairs: one block per pair stages the
// weight row and the input row in shared memory with all its threads (every load in flight at
// once), then one warp forms the reference's strided sums and tree from shared memory. The host
// launches it only when the buffers cover every row it reads.
constexpr int kStagedThreads = 256;
__global__ void __launch_bounds__(kStagedThreads) k_project_staged(FB X, FB W, FB Y, int cols, int outputStride, int outputOffset,
                                                                   unsigned *err) {
    if (threadIdx.x == 0 && blockIdx.y == 0) prefetch_l2(W.p + (long long)blockIdx.x * cols, (unsigned long long)cols * 4);
    dep_enter();
    extern __shared__ float staged[];  // [cols] weights, then [cols] inputs
    const long long row = blockIdx.x, token = blockIdx.y;
    stage_row(staged, W.p + row * cols, cols);
    stage_row(staged + cols, X.p + token * cols, cols);
    __syncthreads();
    if (threadIdx.x < 32) {
        const float r = lane_dot(staged, staged + cols, cols, threadIdx.x);
        if (threadIdx.x == 0) Y.set(token * outputStride + outputOffset + row, r, err);
    }
}

// The same projection for prompt chunks and decode batches (8 or more tokens), register-tiled
// with four reference lanes per thread. A half-warp computes 4 rows x 4 tokens; its thread u
// holds lanes 4u .. 4u + 3 of each of those 16 sums (elements 4u + 64k .. 4u + 64k + 3, k
// ascending) as two register pairs that advance with the paired rounded product (an FMA whose
// addend is a run-time -0) and the paired rounded add, each element rounded exactly as the scalar
// __fmul_rn / __fadd_rn would: the 16 bytes a thread needs of a staged weight or input row per
// step come in one shared load, already paired. Each output then takes the
// reference's tree over its 64 lanes: the levels 32, 16, 8 and 4 are exchanges between
// half-warp threads 8, 4, 2 and 1 apart, in which each thread keeps (and adds) half of the
// outputs it holds, so that thread u ends with output u; levels 2 and 1 are in the thread. A
// block (16 half-warps: 2 row groups x 8 token groups) stages 256-column chunks of its 8 weight
// rows and 32 input rows in shared memory with 16-byte asynchronous copies, two chunks in flight.
// Used when cols is a multiple of 256, the rows are 16-byte aligned, and the host has checked
// that W and X cover every row and token named.
constexpr int kTileRows = 4, kTileTokens = 8, kTileWarps = 8, kTileK = 256;  // minimum rows and tokens; warps; chunk columns
constexpr int kBlockRows = 2 * kTileRows, kBlockTokens = 8 * 4;
constexpr size_t kTileSmem = 2 * (size_t)(kBlockRows + kBlockTokens) * kTileK * 4;  // 80 KB
__global__ void __launch_bounds__(kTileWarps * 32) k_project_quad(FB X, FB W, FB Y, int cols, int rows, int tokens, int outputStride,
                                                                  int outputOffset, unsigned long long neg0, unsigned *err) {
    dep_enter();
    extern __shared__ __align__(16) float tile_smem[];  // [2 stages][8 weight rows + 32 input rows][256]
    const int hw = threadIdx.x / 16, u = threadIdx.x & 15;
    const int rb = blockIdx.x * kBlockRows, tb = blockIdx.y * kBlockTokens;
    const int rg = (hw / 8) * 4, tg = (hw % 8) * 4;  // this half-warp's rows / tokens within the block
    const int chunks = cols / kTileK;
    auto stage = [&](int c, int st) {  // chunk c of every block row into stage st (rows past the end repeat the last)
        float *base = tile_smem + (size_t)st * (kBlockRows + kBlockTokens) * kTileK;
        for (int k = threadIdx.x; k < (kBlockRows + kBlockTokens) * (kTileK / 4); k += kTileWarps * 32) {
            const int line = k / (kTileK / 4), q = k % (kTileK / 4);
            const float *src = line < kBlockRows ? W.p + (long long)min(rb + line, rows - 1) * cols
                                                 : X.p + (long long)min(tb + line - kBlockRows, tokens - 1) * cols;
            copy16_async(base + (size_t)line * kTileK + q * 4, src + (long long)c * kTileK + q * 4);
        }
        copy_commit();
    };
    unsigned long long acc[4][4][2];  // [row][token][lanes (4u, 4u + 1) | (4u + 2, 4u + 3)]
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][j][0] = acc[r][j][1] = 0ull;
    stage(0, 0);
    for (int c = 0; c < chunks; ++c) {
        if (c + 1 < chunks) {
            stage(c + 1, (c + 1) & 1);
            copy_wait<1>();
        } else {
            copy_wait<0>();
        }
        __syncthreads();
        const float *sbase = tile_smem + (size_t)(c & 1) * (kBlockRows + kBlockTokens) * kTileK;
        const unsigned ws = (unsigned)__cvta_generic_to_shared(sbase + (size_t)rg * kTileK + 4 * u);
        const unsigned xs = (unsigned)__cvta_generic_to_shared(sbase + (size_t)(kBlockRows + tg) * kTileK + 4 * u);
#pragma unroll
        for (int k = 0; k < kTileK / STRATA_LANES; ++k) {
            unsigned long long w[4][2], x[4][2];
#pragma unroll
            for (int r = 0; r < 4; ++r)
                asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(w[r][0]), "=l"(w[r][1]) : "r"(ws + (unsigned)(r * kTileK + 64 * k) * 4));
#pragma unroll
            for (int j = 0; j < 4; ++j)
                asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(x[j][0]), "=l"(x[j][1]) : "r"(xs + (unsigned)(j * kTileK + 64 * k) * 4));
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h) acc[r][j][h] = add2_rn(acc[r][j][h], mul_rn2(w[r][h], x[j][h], neg0));
        }
        __syncthreads();
    }
    // the tree: v[o][i] = lane 4u + i of output o = 4 r + j
    float v[16][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            unpack2(acc[r][j][0], v[4 * r + j][0], v[4 * r + j][1]);
            unpack2(acc[r][j][1], v[4 * r + j][2], v[4 * r + j][3]);
        }
#pragma unroll
    for (int m = 8, n = 16; m >= 1; m >>= 1, n >>= 1) {  // levels 32, 16, 8, 4: partner u ^ m; keep half of n outputs
        const bool upper = (u & m) != 0;
#pragma unroll
        for (int o = 0; o < n / 2; ++o)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float give = upper ? v[o][i] : v[o + n / 2][i], keep = upper ? v[o + n / 2][i] : v[o][i];
                v[o][i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, give, m));
            }
    }
    const float sum = __fadd_rn(__fadd_rn(v[0][0], v[0][2]), __fadd_rn(v[0][1], v[0][3]));  // levels 2 and 1
    const int row = rb + rg + u / 4, token = tb + tg + u % 4;
    if (row < rows && token < tokens) Y.set((long long)token * outputStride + outputOffset + row, sum, err);
}

// kernels/strata.cu:168-176
__global__ void k_bf16_project(Grid g, FB X, UB Codes, FB Y, int cols, int rows, int tokens, int outputStride, int outputOffset,
                               unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z)) return;
    if (!((int)row < rows && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    float acc[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < cols; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int i = i0 + 32 * h;
            if (i >= cols) continue;
            long long ix = (long long)row * cols + i;
            unsigned bits = (Codes.get(ix / 2, err) >> ((ix % 2) * 16)) & 65535u;
            acc[h] = __fadd_rn(acc[h], __fmul_rn(__uint_as_float(bits << 16), X.get((long long)token * cols + i, err)));
        }
    float r = tree64(acc[0], acc[1]);
    if (t == 0) Y.set((long long)token * outputStride + outputOffset + row, r, err);
}

// kernels/strata.cu:179-192
__global__ void k_q2_project(Grid g, FB X, UB Blob, FB Y, int cols, int rows, int tokens, int outputStride, int outputOffset,
                             int codeOffset, int scaleOffset, int weightRow, int rowStride, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z)) return;
    if (!((int)row < rows && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    float acc[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < cols; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int i = i0 + 32 * h;
            if (i >= cols) continue;
            long long ix = ((long long)weightRow + (long long)row * rowStride) * cols + i;
            float weight = __fmul_rn((float)code_of(Blob, codeOffset, ix, err), half_of(Blob, scaleOffset + ix / 64, err));
            acc[h] = __fadd_rn(acc[h], __fmul_rn(weight, X.get((long long)token * cols + i, err)));
        }
    float r = tree64(acc[0], acc[1]);
    if (t == 0) Y.set((long long)token * outputStride + outputOffset + row, r, err);
}

// kernels/strata.cu:81-87 — IQ4_NL blocks of 32 values in 18 bytes: an FP16 scale, then 16 code
// bytes (value i of a block: low nibble of byte i for i < 16, else high nibble of byte i - 16).
// The scale starts at an even byte (18 per block), so it never straddles two words.
__device__ __forceinline__ float ple_value(const UB &Packed, long long byte0, int i, unsigned *err) {
    const long long scale_byte = byte0 + (long long)(i / 32) * 18, code_byte = scale_byte + 2 + i % 16;
    const unsigned half = (Packed.get(scale_byte / 4, err) >> ((scale_byte % 4) * 8)) & 65535u;
    const int code = (int)((Packed.get(code_byte / 4, err) >> ((code_byte % 4) * 8 + (i % 32 < 16 ? 0 : 4))) & 15u);
    return __fmul_rn(half_bits(half), iq4(code));
}
__global__ void k_ple_decode(Grid g, UB Packed, FB Values, int count, unsigned *err) {
    dep_enter();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (long long)g.x * STRATA_LANES && i < count) Values.set(i, ple_value(Packed, 0, (int)i, err), err);
}
// Rows Ids[h] of a device-resident IQ4_NL table (rows of head_dim values, head_dim / 32 * 18
// bytes each) decoded into Values[h * head_dim + j]: the values strata_ple_decode gives for the
// same rows packed one after another (src/model.js:230-242 gathers them on the host). A row
// outside the table reads zeros and sets kErrIndex; a non-finite scale sets kErrPleScale
// (src/model.js:241 rejects those rows).
__global__ void k_ple_gather_decode(UB Table, IB Ids, FB Values, int rows, int head_dim, unsigned *err) {
    dep_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * head_dim) return;
    const int h = (int)(i / head_dim), j = (int)(i % head_dim);
    const long long byte0 = (long long)Ids.get(h, err) * (head_dim / 32 * 18);
    const long long scale_byte = byte0 + (long long)(j / 32) * 18;
    if (j % 32 == 0 && ((Table.get(scale_byte / 4, err) >> ((scale_byte % 4) * 8)) & 0x7c00u) == 0x7c00u) raise_error(err, kErrPleScale);
    Values.set(i, ple_value(Table, byte0, j, err), err);
}

__device__ __forceinline__ long long group_of(long long index, int size) {
    if (size == 16) return index >> 4;
    if (size == 32) return index >> 5;
    if (size == 64) return index >> 6;
    return index / size;
}

// kernels/strata.cu:193-211
__global__ void k_quant_project(Grid g, FB X, UB Codes, FB Scales, FB Offsets, FB Y, int cols, int rows, int tokens, int outputStride,
                                int outputOffset, int bits, int groupSize, int bias, int codebook, int hasOffset, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z)) return;
    if (!((int)row < rows && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    float acc[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < cols; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int i = i0 + 32 * h;
            if (i >= cols) continue;
            long long index = (long long)row * cols + i, bit = index * bits;
            int code = (int)((Codes.get(bit / 32, err) >> (bit % 32)) & ((1u << bits) - 1u));
            float value = codebook == 1 ? iq4(code) : (float)(code + bias);
            long long grp = group_of(index, groupSize);
            float weight = __fmul_rn(value, Scales.get(grp, err));
            if (hasOffset != 0) weight = __fadd_rn(weight, Offsets.get(grp, err));
            acc[h] = __fadd_rn(acc[h], __fmul_rn(weight, X.get((long long)token * cols + i, err)));
        }
    float r = tree64(acc[0], acc[1]);
    if (t == 0) Y.set((long long)token * outputStride + outputOffset + row, r, err);
}

// kernels/strata.cu:38-55
__global__ void k_q2_gate_up(Grid g, FB X, UB Blob, FB Scales, IB Mapping, FB Hidden, int width, int ff, int tokens, int mapped,
                             int expanded, int codeOffset, int scaleOffset, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z)) return;
    if (!((int)row < ff && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    long long inputRow = mapped != 0 ? Mapping.get(2LL * token, err) : (long long)token;
    float ga[2] = {0.0f, 0.0f}, ua[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < width; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int i = i0 + 32 * h;
            if (i >= width) continue;
            long long gi = (long long)row * 2 * width + i, ui = gi + width;
            int gc = code_of(Blob, codeOffset, gi, err), uc = code_of(Blob, codeOffset, ui, err);
            long long gs = scaleOffset + gi / 64, us = scaleOffset + ui / 64;
            float gw = __fmul_rn((float)gc, expanded != 0 ? Scales.get(gs, err) : half_of(Blob, gs, err));
            float uw = __fmul_rn((float)uc, expanded != 0 ? Scales.get(us, err) : half_of(Blob, us, err));
            float x = X.get(inputRow * width + i, err);
            ga[h] = __fadd_rn(ga[h], __fmul_rn(gw, x));
            ua[h] = __fadd_rn(ua[h], __fmul_rn(uw, x));
        }
    float gsum = tree64(ga[0], ga[1]);
    float usum = tree64(ua[0], ua[1]);
    if (t == 0) Hidden.set((long long)token * ff + row, __fmul_rn(ref_silu(gsum), usum), err);
}

// kernels/strata.cu:56-69
__global__ void k_q2_down(Grid g, FB Hidden, UB Blob, FB Scales, IB Mapping, FB Y, int width, int ff, int tokens, int mapped,
                          int expanded, int outputOffset, int codeOffset, int scaleOffset, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z)) return;
    if (!((int)row < width && (int)token < tokens)) return;
    int t = threadIdx.x & 31;
    float acc[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < ff; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int i = i0 + 32 * h;
            if (i >= ff) continue;
            long long index = (long long)row * ff + i;
            int code = code_of(Blob, codeOffset, index, err);
            long long si = scaleOffset + index / 64;
            float w = __fmul_rn((float)code, expanded != 0 ? Scales.get(si, err) : half_of(Blob, si, err));
            acc[h] = __fadd_rn(acc[h], __fmul_rn(w, Hidden.get((long long)token * ff + i, err)));
        }
    float r = tree64(acc[0], acc[1]);
    long long destination = mapped != 0 ? Mapping.get(2LL * token + 1, err) : (long long)token;
    if (t == 0) Y.set(outputOffset + destination * width + row, r, err);
}

}  // namespace

namespace {
// kernels/strata.cu:238-270 and :478-509. Logits are staged in shared memory per warp.
__global__ void k_router_batch(Grid g, FB Logits, IB Ids, FB Weights, int experts, int topK, int batch, unsigned *err) {
    dep_enter();
    __shared__ float lg[kWarpsPerBlock][512];
    __shared__ float sel[kWarpsPerBlock][32];
    __shared__ int ids[kWarpsPerBlock][32];
    __shared__ float wts[kWarpsPerBlock][32];
    unsigned token, y, z;
    if (!my_group(g, token, y, z)) return;
    if (!batch && (token | y | z)) return;  // strata_router: every workgroup computes token 0 (one is enough)
    if (batch && (y | z)) return;           // strata_router_batch: blockIdx.x is the token
    int w = (threadIdx.x / 32) % kWarpsPerBlock, t = threadIdx.x & 31;
    for (int e = t; e < experts; e += 32) lg[w][e] = Logits.get((long long)token * experts + e, err);
    __syncwarp();
    route_warp(lg[w], experts, topK, ids[w], wts[w], sel[w]);
    for (int k = t; k < topK; k += 32) {
        Ids.set((long long)token * topK + k, ids[w][k], err);
        Weights.set((long long)token * topK + k, wts[w][k], err);
    }
}

// ---------------------------------------------------------------- launchers


cudaError_t L_unpack_half(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_unpack_half, LANESL, grid_of(g), U(0), F(1), a[2].i, err);
    return cudaGetLastError();
}
cudaError_t L_ple_decode(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_ple_decode, LANESL, grid_of(g), U(0), F(1), a[2].i, err);
    return cudaGetLastError();
}
cudaError_t L_expert_scales(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_expert_scales, LANESL, grid_of(g), U(0), F(1), a[2].i, a[3].i, err);
    return cudaGetLastError();
}
cudaError_t L_q2_gate_up(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_q2_gate_up, GROUPS, grid_of(g), F(0), U(1), F(2), I(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i, err);
    return cudaGetLastError();
}
cudaError_t L_q2_down(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_q2_down, GROUPS, grid_of(g), F(0), U(1), F(2), I(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i, a[12].i,
                          err);
    return cudaGetLastError();
}
cudaError_t L_project(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    // few (row, token) pairs of long rows: one staging block per pair (the pairs the dispatch
    // names, rows < g[0] and tokens < g[1]; z repeats them)
    const long long cols = a[3].i, rows = std::min<long long>(a[4].i, g[0]), tokens = std::min<long long>(a[5].i, g[1]);
    const bool aligned16 = ((reinterpret_cast<uintptr_t>(a[0].ptr) | reinterpret_cast<uintptr_t>(a[1].ptr)) & 15) == 0;
    // one token, at least 512 rows: the weight stream (one block per SM, rows through a ring of
    // bulk-copied slots)
    if (tokens == 1 && rows >= 512 && cols >= 64 && cols % 64 == 0 && (size_t)cols * 8 <= kStreamSmem && aligned16 &&
        a[1].len >= rows * cols && a[0].len >= cols && (long long)a[7].i + rows <= a[2].len && a[7].i >= 0 && rows <= INT32_MAX) {
        static int sms = 0;
        if (!sms) {
            int dev = 0;
            cudaError_t e = cudaGetDevice(&dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess || sms <= 0) return e != cudaSuccess ? e : cudaErrorInvalidValue;
        }
        const long long blocks = std::min<long long>(rows, sms), per = (rows + blocks - 1) / blocks;
        // slots that fit beside the input row; half-warps that own them, and slots per half-warp
        const long long fit = std::min<long long>(kStreamMaxSlots, (long long)(kStreamSmem / ((size_t)cols * 4)) - 1);
        const long long halves = std::min<long long>({(long long)kStreamHalves, fit, per});
        const long long depth = std::max<long long>(
            1, std::min<long long>({(long long)kStreamMaxDepth, fit / halves, (per + halves - 1) / halves}));
        const size_t bytes = (size_t)(halves * depth + 1) * cols * 4;
        cudaError_t e = cudaFuncSetAttribute(k_project_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        launch_k(true, k_project_stream, (unsigned)((rows + per - 1) / per), kStreamThreads, bytes, s, F(0), F(1), F(2), (int)cols, (int)rows,
                 (int)per, (int)halves, (int)depth, a[7].i, err);
        return cudaGetLastError();
    }
    // one token, many rows: a half-warp per row, 16-byte streaming loads (fewer rows: the
    // staging blocks below have every load of a row in flight at once)
    if (tokens == 1 && rows > 2048 && cols >= 64 && cols % 64 == 0 && aligned16 && a[1].len >= rows * cols && a[0].len >= cols &&
        (long long)a[7].i + rows <= a[2].len && a[7].i >= 0) {
        launch_k(true, k_project_gemv, (unsigned)((rows + kGemvRows - 1) / kGemvRows), kGemvThreads, 0, s, F(0), F(1), F(2), (int)cols, (int)rows,
                                                                                                 a[7].i, err);
        return cudaGetLastError();
    }
    const size_t bytes = (size_t)cols * 8;
    if (rows * tokens <= 2048 && cols >= 512 && bytes <= 200 * 1024 && a[1].len >= rows * cols && a[0].len >= tokens * cols &&
        rows > 0 && tokens > 0) {
        cudaError_t e = cudaFuncSetAttribute(k_project_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        launch_k(tokens == 1, k_project_staged, dim3((unsigned)rows, (unsigned)tokens), kStagedThreads, bytes, s, F(0), F(1), F(2), a[3].i, a[6].i, a[7].i,
                                                                                                err);
        return cudaGetLastError();
    }
    const bool aligned = ((reinterpret_cast<uintptr_t>(a[0].ptr) | reinterpret_cast<uintptr_t>(a[1].ptr)) & 15) == 0;
    if (tokens >= kTileTokens && rows >= kTileRows && cols % kTileK == 0 && aligned && a[1].len >= rows * cols &&
        a[0].len >= tokens * cols && g[2] >= 1) {
        cudaError_t e = cudaFuncSetAttribute(k_project_quad, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTileSmem);
        if (e != cudaSuccess) return e;
        const dim3 blocks((unsigned)((rows + kBlockRows - 1) / kBlockRows), (unsigned)((tokens + kBlockTokens - 1) / kBlockTokens));
        launch_k(false, k_project_quad, blocks, kTileWarps * 32, kTileSmem, s, F(0), F(1), F(2), a[3].i, (int)rows, (int)tokens, a[6].i, a[7].i,
                                                                   kNegZero2, err);
        return cudaGetLastError();
    }
    launch_k(tokens == 1, k_project, GROUPS, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, a[6].i, a[7].i, err);
    return cudaGetLastError();
}
cudaError_t L_bf16_project(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_bf16_project, GROUPS, grid_of(g), F(0), U(1), F(2), a[3].i, a[4].i, a[5].i, a[6].i, a[7].i, err);
    return cudaGetLastError();
}
cudaError_t L_q2_project(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_q2_project, GROUPS, grid_of(g), F(0), U(1), F(2), a[3].i, a[4].i, a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i,
                             err);
    return cudaGetLastError();
}
cudaError_t L_quant_project(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_quant_project, GROUPS, grid_of(g), F(0), U(1), F(2), F(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i,
                                a[12].i, a[13].i, a[14].i, err);
    return cudaGetLastError();
}
cudaError_t L_elementwise(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(a[3].i <= 16384, k_elementwise, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].f, err);
    return cudaGetLastError();
}
cudaError_t L_router(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_router_batch, 1, kWarpsPerBlock * 32, 0, s, Grid{1, 1, 1}, F(0), I(1), F(2), a[3].i, a[4].i, 0, err);
    return cudaGetLastError();
}
cudaError_t L_router_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_router_batch, GROUPS, grid_of(g), F(0), I(1), F(2), a[3].i, a[4].i, 1, err);
    return cudaGetLastError();
}
cudaError_t L_moe_combine(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_moe_combine, LANESL, grid_of(g), F(0), F(1), F(2), F(3), F(4), a[5].i, a[6].i, err);
    return cudaGetLastError();
}
cudaError_t L_moe_combine_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_moe_combine_batch, LANESL, grid_of(g), F(0), F(1), F(2), F(3), F(4), a[5].i, a[6].i, a[7].i, err);
    return cudaGetLastError();
}
cudaError_t L_gather_rows(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_gather_rows, LANESL, grid_of(g), F(0), I(1), F(2), a[3].i, a[4].i, err);
    return cudaGetLastError();
}
cudaError_t L_scatter_rows(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_scatter_rows, LANESL, grid_of(g), F(0), I(1), F(2), a[3].i, a[4].i, err);
    return cudaGetLastError();
}
}  // namespace

cudaError_t ple_gather_decode(const unsigned *table, long long table_words, const int *ids, long long ids_len, int rows, int head_dim,
                              float *values, long long values_len, cudaStream_t s, unsigned *err) {
    const long long n = (long long)rows * head_dim;
    launch_k(true, k_ple_gather_decode, (unsigned)((n + 255) / 256), 256, 0, s, UB{const_cast<unsigned *>(table), table_words},
                                                                      IB{const_cast<int *>(ids), ids_len}, FB{values, values_len}, rows,
                                                                      head_dim, err);
    return cudaGetLastError();
}

// Parameter lists in kernels/strata.cu order and spelling. Kinds: 'f' float buffer, 'u' u32
// buffer, 'i' i32 buffer, 'I' i32 scalar, 'F' f32 scalar.
const KernelSpec kKernels[] = {
    {"strata_unpack_half", "Packed:u Values:f count:I", L_unpack_half},
    {"strata_expert_scales", "Blob:u Scales:f offset:I count:I", L_expert_scales},
    {"strata_ple_decode", "Packed:u Values:f count:I", L_ple_decode},
    {"strata_q2_gate_up",
     "X:f Blob:u Scales:f Mapping:i Hidden:f width:I ff:I tokens:I mapped:I expanded:I codeOffset:I scaleOffset:I", L_q2_gate_up},
    {"strata_q2_down",
     "Hidden:f Blob:u Scales:f Mapping:i Y:f width:I ff:I tokens:I mapped:I expanded:I outputOffset:I codeOffset:I scaleOffset:I",
     L_q2_down},
    {"strata_project", "X:f W:f Y:f cols:I rows:I tokens:I outputStride:I outputOffset:I", L_project},
    {"strata_bf16_project", "X:f Codes:u Y:f cols:I rows:I tokens:I outputStride:I outputOffset:I", L_bf16_project},
    {"strata_q2_project",
     "X:f Blob:u Y:f cols:I rows:I tokens:I outputStride:I outputOffset:I codeOffset:I scaleOffset:I weightRow:I rowStride:I",
     L_q2_project},
    {"strata_quant_project",
     "X:f Codes:u Scales:f Offsets:f Y:f cols:I rows:I tokens:I outputStride:I outputOffset:I bits:I groupSize:I bias:I codebook:I "
     "hasOffset:I",
     L_quant_project},
    {"strata_elementwise", "A:f B:f Y:f n:I mode:I scale:F", L_elementwise},
    {"strata_router", "Logits:f Ids:i Weights:f experts:I topK:I", L_router},
    {"strata_router_batch", "Logits:f Ids:i Weights:f experts:I topK:I", L_router_batch},
    {"strata_moe_combine", "Parts:f Weights:f Shared:f SharedGate:f Y:f width:I count:I", L_moe_combine},
    {"strata_moe_combine_batch", "Parts:f Weights:f Shared:f SharedGate:f Y:f width:I count:I tokens:I", L_moe_combine_batch},
    {"strata_gather_rows", "X:f Indices:i Y:f width:I rows:I", L_gather_rows},
    {"strata_scatter_rows", "X:f Indices:i Y:f width:I rows:I", L_scatter_rows},
};
const int kNumKernels = sizeof(kKernels) / sizeof(kKernels[0]);

}  // namespace strata
