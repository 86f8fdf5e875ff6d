// The rest of the reference's kernels (kernels/strata.cu:72-534 apart from the mixture-of-experts
// entries in compat.cu): embeddings, RoPE, norms, hyper-connection mixing, the gated delta-net
// recurrence, causal convolution, attention, per-layer-embedding gating and greedy argmax. With
// them strata_run() serves every entry that src/engine.js, src/ops.js and src/prefill.js
// dispatch, so the reference host runs a whole model on this library.
//
// Numerics: every F32 product, sum and quotient is rounded separately in the reference's order
// (__fmul_rn / __fadd_rn / __fdiv_rn / __fsqrt_rn, no contraction), reductions keep the
// 64-lane stride and the shared-memory tree, and expf is the reference's own (ref_expf), so
// results are bit-identical to the reference's CPU build. The three other transcendentals
// (logf in the softplus, cosf / sinf of the RoPE table) are evaluated in double precision and
// rounded once to float: the reference leaves them to its C library, whose float versions are
// not correctly rounded in every case, so these agree with it to within an ulp.
//
// Layout: as in compat.cu, a reference workgroup is one warp (thread t owns lanes t and t+32)
// and element entries run one reference lane per thread. Every access is bounds-checked
// against its buffer; an out-of-range index sets the device error word instead of faulting.
#include "compat.cuh"

#include <algorithm>
#include <cstdint>
#include <cstdlib>

namespace strata {
namespace {

constexpr int kMaxCells = 2048;  // kernels/strata.cu:333, the shared score array

// Index of this thread's reference lane for an element entry, or -1 past the dispatch grid or n.
// Workgroups beyond the first along y and z repeat the same lanes in the reference; each lane
// runs once here (for the in-place entries the repeats would race with one another).
__device__ __forceinline__ long long lane_index(const Grid g, long long n) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    return (i < (long long)g.x * STRATA_LANES && i < n) ? i : -1;
}

__device__ __forceinline__ float max_tree64(float lo, float hi) {
    float a = fmaxf(lo, hi);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) a = fmaxf(a, __shfl_down_sync(0xffffffffu, a, s));
    return a;
}

// log(x) and cos / sin rounded once from double precision.
__device__ __forceinline__ float log_f(float x) { return __double2float_rn(log((double)x)); }
__device__ __forceinline__ float cos_f(float x) { return __double2float_rn(cos((double)x)); }
__device__ __forceinline__ float sin_f(float x) { return __double2float_rn(sin((double)x)); }

// Rotated value of element d of one head row (NeoX half split): a = x[pair], b = x[pair + half].
__device__ __forceinline__ float rotate(float a, float b, float c, float s, bool first) {
    return first ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)) : __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

// ---------------------------------------------------------------- embeddings

// kernels/strata.cu:72-80: one token row (F32, BF16 or canonical packed codes) copied to every
// stream of the residual.
__global__ void k_embedding(Grid g, FB Values, UB Codes, FB Scales, FB Offsets, FB Residual, int width, int streams, int outputOffset,
                            int format, int bits, int groupSize, int bias, int codebook, int hasOffset, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, width);
    if (i < 0) return;
    float value = 0.0f;
    if (format == 0) {
        value = Values.get(i, err);
    } else if (format == 1) {
        value = __uint_as_float(((Codes.get(i / 2, err) >> ((i % 2) * 16)) & 65535u) << 16);
    } else {
        long long bit = i * bits;
        int code = (int)((Codes.get(bit / 32, err) >> (bit % 32)) & ((1u << bits) - 1u));
        long long group = i / groupSize;
        value = __fmul_rn(codebook == 1 ? iq4(code) : (float)(code + bias), Scales.get(group, err));
        if (hasOffset != 0) value = __fadd_rn(value, Offsets.get(group, err));
    }
    for (int stream = 0; stream < streams; ++stream) Residual.set((long long)outputOffset + (long long)stream * width + i, value, err);
}

// kernels/strata.cu:282-284 and :399-402
__global__ void k_embed(Grid g, FB Row, FB Residual, int width, int streams, int tokens, unsigned *err) {
    dep_enter();
    const long long hc = (long long)width * streams;
    long long i = lane_index(g, hc * tokens);
    if (i >= 0) Residual.set(i, Row.get((i / hc) * width + i % width, err), err);
}

// ---------------------------------------------------------------- RoPE

// kernels/strata.cu:90-104: inverse frequencies base^(-2i/rotary) from a range-reduced log
// series and an exp series, in double arithmetic with every operation rounded on its own (the
// reference's CPU target has no fused multiply-add), split into a float and its remainder.
__global__ void k_rope_frequencies(Grid g, FB High, FB Low, int rotary, float base, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, rotary / 2);
    if (i < 0) return;
    double value = (double)base;
    int exponent = 0;
    while (value >= 2.0) {  // at most 128 halvings for a finite float base
        value = __dmul_rn(value, 0.5);
        exponent += 1;
    }
    const double y = __ddiv_rn(__dsub_rn(value, 1.0), __dadd_rn(value, 1.0));
    double term = y, logarithm = 0.0;
    for (int n = 1; n <= 49; n += 2) {
        logarithm = __dadd_rn(logarithm, __ddiv_rn(term, (double)n));
        term = __dmul_rn(__dmul_rn(term, y), y);
    }
    const double ln2 = 0.693147180559945309417232121458176568;
    logarithm = __dadd_rn(__dmul_rn(2.0, logarithm), __dmul_rn((double)exponent, ln2));
    const double power = __ddiv_rn(__dmul_rn(-logarithm, (double)(2 * i)), (double)rotary);
    int whole = (int)__double2float_rn(__ddiv_rn(power, ln2));
    const double remainder = __dsub_rn(power, __dmul_rn((double)whole, ln2));
    double result = 1.0;
    term = 1.0;
    for (int n = 1; n <= 20; ++n) {
        term = __ddiv_rn(__dmul_rn(term, remainder), (double)n);
        result = __dadd_rn(result, term);
    }
    for (; whole < 0; ++whole) result = __dmul_rn(result, 0.5);
    const float high = __double2float_rn(result);
    High.set(i, high, err);
    Low.set(i, __double2float_rn(__dsub_rn(result, (double)high)), err);
}

// kernels/strata.cu:105-111: cos / sin of position * frequency, reduced by whole turns in double.
__global__ void k_rope_table(Grid g, FB High, FB Low, FB Cos, FB Sin, int rotary, int context, unsigned *err) {
    dep_enter();
    const int half = rotary / 2;
    long long i = lane_index(g, (long long)context * half);
    if (i < 0) return;
    const long long pair = i % half;
    const double angle = __dmul_rn((double)(i / half), __dadd_rn((double)High.get(pair, err), (double)Low.get(pair, err)));
    const double turn = 6.283185307179586476925286766559005768;
    const int wraps = (int)__double2float_rn(__dadd_rn(__ddiv_rn(angle, turn), 0.5));
    const float reduced = __double2float_rn(__dsub_rn(angle, __dmul_rn((double)wraps, turn)));
    Cos.set(i, cos_f(reduced), err);
    Sin.set(i, sin_f(reduced), err);
}

// kernels/strata.cu:113-120 (rope_position: table row position + token), :319-327 (rope: one
// row of Cos / Sin) and :445-452 (rope_batch: table row = token). `mode` 0 / 1 / 2 picks which;
// mode 3 (strata_rope_seqs, no reference counterpart) rotates token t's rows at Pos[t], the
// position of the sequence that token t belongs to.
__global__ void k_rope(Grid g, FB X, FB Cos, FB Sin, FB Y, int dim, int heads, int rotary, int position, int tokens, int mode, IB Pos,
                       unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)dim * heads * tokens);
    if (i < 0) return;
    const long long d = i % dim, token = i / ((long long)dim * heads);
    if (Pos.n > 0) position = Pos.get(mode == 3 ? token : 0, err);  // strata_rope_at / _seqs: positions live on the device
    if (d >= rotary) {
        Y.set(i, X.get(i, err), err);
        return;
    }
    const int half = rotary / 2;
    const long long pair = d % half, row = i - d;
    const long long angle = mode == 1 ? pair : (mode == 0 ? (position + token) : mode == 3 ? position : token) * half + pair;
    const float a = X.get(row + pair, err), b = X.get(row + pair + half, err);
    Y.set(i, rotate(a, b, Cos.get(angle, err), Sin.get(angle, err), d < half), err);
}

// ---------------------------------------------------------------- reductions over a row

// kernels/strata.cu:121-131: Y[token, row] = W[row] . X[token], 64-lane stride then the tree.
__global__ void k_gemv(Grid g, FB X, FB W, FB Y, int cols, int rows, int tokens, unsigned *err) {
    dep_enter();
    unsigned row, token, z;
    if (!my_group(g, row, token, z) || (int)row >= rows || (int)token >= tokens) return;
    const int t = threadIdx.x & 31;
    const long long wb = (long long)row * cols, xb = (long long)token * cols;
    float r;
    if (covers(W, wb, cols) && covers(X, xb, cols)) {
        r = lane_dot(W.p + wb, X.p + xb, cols, t);
    } else {
        float lo = 0.0f, hi = 0.0f;
        for (int i = t; i < cols; i += STRATA_LANES) {
            lo = __fadd_rn(lo, __fmul_rn(W.get(wb + i, err), X.get(xb + i, err)));
            if (i + 32 < cols) hi = __fadd_rn(hi, __fmul_rn(W.get(wb + i + 32, err), X.get(xb + i + 32, err)));
        }
        r = tree64(lo, hi);
    }
    if (t == 0) Y.set((long long)token * rows + row, r, err);
}

// kernels/strata.cu:134-153: one row of canonical packed codes (2, 4 or 8 bits, affine or IQ4_NL,
// scale and optional offset per group) against one input vector.
__global__ void k_quant_gemv(Grid g, FB X, UB Codes, FB Scales, FB Offsets, FB Y, int cols, int rows, int bits, int groupSize, int bias,
                             int codebook, int hasOffset, unsigned *err) {
    dep_enter();
    unsigned row, y, z;
    if (!my_group(g, row, y, z) || (int)row >= rows) return;
    const int t = threadIdx.x & 31;
    const unsigned mask = (1u << bits) - 1u;
    float acc[2] = {0.0f, 0.0f};
    for (int i0 = t; i0 < cols; i0 += STRATA_LANES)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = i0 + 32 * h;
            if (i >= cols) continue;
            const long long index = (long long)row * cols + i, bit = index * bits;
            const int code = (int)((Codes.get(bit / 32, err) >> (bit % 32)) & mask);
            const long long group = index / groupSize;
            float weight = __fmul_rn(codebook == 1 ? iq4(code) : (float)(code + bias), Scales.get(group, err));
            if (hasOffset != 0) weight = __fadd_rn(weight, Offsets.get(group, err));
            acc[h] = __fadd_rn(acc[h], __fmul_rn(weight, X.get(i, err)));
        }
    const float r = tree64(acc[0], acc[1]);
    if (t == 0) Y.set(row, r, err);
}

// kernels/strata.cu:214-227: mode 0 weighted RMSNorm (gamma row `row % weightRows`), mode 1 L2 norm.
__global__ void k_norm(Grid g, FB X, FB W, FB Y, int cols, int rows, int weightRows, int mode, float epsilon, float scale, unsigned *err) {
    dep_enter();
    unsigned row, y, z;
    if (!my_group(g, row, y, z) || (int)row >= rows) return;
    const int t = threadIdx.x & 31;
    const long long base = (long long)row * cols, wbase = (long long)(row % weightRows) * cols;
    const bool fast = covers(X, base, cols) && covers(Y, base, cols) && (mode != 0 || covers(W, wbase, cols));
    float ss;
    if (fast) {
        ss = lane_dot(X.p + base, X.p + base, cols, t);
    } else {
        float lo = 0.0f, hi = 0.0f;
        for (int i = t; i < cols; i += STRATA_LANES) {
            const float a = X.get(base + i, err);
            lo = __fadd_rn(lo, __fmul_rn(a, a));
            if (i + 32 < cols) {
                const float b = X.get(base + i + 32, err);
                hi = __fadd_rn(hi, __fmul_rn(b, b));
            }
        }
        ss = tree64(lo, hi);
    }
    ss = __shfl_sync(0xffffffffu, ss, 0);
    const float inv = __fdiv_rn(scale, __fsqrt_rn(__fadd_rn(mode == 0 ? __fdiv_rn(ss, (float)cols) : ss, epsilon)));
    if (fast) {
        const float *x = X.p + base, *w = W.p + wbase;
        float *y = Y.p + base;
        int i = t;
        for (; i + 7 * 32 < cols; i += 8 * 32) {  // eight loads of each row in flight, then the stores
            float xv[8], wv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                xv[u] = x[i + 32 * u];
                wv[u] = mode == 0 ? w[i + 32 * u] : 1.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) y[i + 32 * u] = __fmul_rn(__fmul_rn(xv[u], inv), wv[u]);
        }
        for (; i < cols; i += 32) y[i] = __fmul_rn(__fmul_rn(x[i], inv), mode == 0 ? w[i] : 1.0f);
        return;
    }
    for (int i = t; i < cols; i += 32) {
        const float w = mode == 0 ? W.get(wbase + i, err) : 1.0f;
        Y.set(base + i, __fmul_rn(__fmul_rn(X.get(base + i, err), inv), w), err);
    }
}

// The same norm with one block per row for long rows: the block stages the row (and its gamma
// row) in shared memory, one warp forms the sum of squares in the reference's order, and every
// thread writes its share of the outputs. Launched only when the buffers cover every row.
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) k_norm_staged(FB X, FB W, FB Y, int cols, int weightRows, int mode, float epsilon,
                                                              float scale) {
    dep_enter();
    extern __shared__ float staged[];  // [cols] row, then [cols] gamma (mode 0)
    __shared__ float inv_s;
    const long long row = blockIdx.x, base = row * cols;
    stage_row(staged, X.p + base, cols);
    if (mode == 0) stage_row(staged + cols, W.p + (row % weightRows) * cols, cols);
    __syncthreads();
    if (threadIdx.x < 32) {
        const float ss = lane_dot(staged, staged, cols, threadIdx.x);
        if (threadIdx.x == 0) inv_s = __fdiv_rn(scale, __fsqrt_rn(__fadd_rn(mode == 0 ? __fdiv_rn(ss, (float)cols) : ss, epsilon)));
    }
    __syncthreads();
    const float inv = inv_s;
    for (int i = threadIdx.x; i < cols; i += kNormThreads)
        Y.p[base + i] = __fmul_rn(__fmul_rn(staged[i], inv), mode == 0 ? staged[cols + i] : 1.0f);
}

// kernels/strata.cu:367-377: per stream, gate = sigmoid(sign(v) sqrt(max(|v|, 1e-6))) with
// v = key . query / sqrt(width).
__global__ void k_ple_gate(Grid g, FB Key, FB Query, FB Gate, int width, int streams, unsigned *err) {
    dep_enter();
    unsigned c, y, z;
    if (!my_group(g, c, y, z) || (int)c >= streams) return;
    const int t = threadIdx.x & 31;
    const long long base = (long long)c * width;
    float dot;
    if (covers(Key, base, width) && covers(Query, base, width)) {
        dot = lane_dot(Key.p + base, Query.p + base, width, t);
    } else {
        float lo = 0.0f, hi = 0.0f;
        for (int d = t; d < width; d += STRATA_LANES) {
            lo = __fadd_rn(lo, __fmul_rn(Key.get(base + d, err), Query.get(base + d, err)));
            if (d + 32 < width) hi = __fadd_rn(hi, __fmul_rn(Key.get(base + d + 32, err), Query.get(base + d + 32, err)));
        }
        dot = tree64(lo, hi);
    }
    if (t == 0) {
        const float v = __fdiv_rn(dot, __fsqrt_rn((float)width));
        const float sign = v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f);
        Gate.set(c, ref_sigmoid(__fmul_rn(sign, __fsqrt_rn(fmaxf(fabsf(v), 0.000001f)))), err);
    }
}

// kernels/strata.cu:386-397: greedy token, the lowest index wins a tie. The reference's answer is
// the element that is largest under (value, then lower index), among values that are not NaN and
// not below -3.402823e38 (else `count`): a maximum under a total order, which any reduction order
// reaches. One block of 1024 threads takes it with the reference's comparison (loads eight ahead),
// then warp shuffles and a shared-memory round combine the threads' bests.
constexpr int kArgmaxThreads = 1024;
__device__ __forceinline__ bool takes(float v, int i, float best, int id) { return v > best || (v == best && i < id); }
// Block r takes row r of Logits (strata_argmax_rows, no reference counterpart: one greedy token per
// sequence of a decode batch); strata_argmax is the one-block case.
__global__ void __launch_bounds__(kArgmaxThreads) k_argmax(FB Logits, IB Token, int count, unsigned *err) {
    dep_enter();
    __shared__ float wbest[kArgmaxThreads / 32];
    __shared__ int wid[kArgmaxThreads / 32];
    const int tid = threadIdx.x, t = tid & 31, w = tid / 32;
    const long long base = (long long)blockIdx.x * count;
    float best = -3.402823e38f;
    int id = count;
    const bool fast = covers(Logits, base, count);
    int i = tid;
    if (fast) {
        for (; i + 7 * kArgmaxThreads < count; i += 8 * kArgmaxThreads) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = Logits.p[base + i + u * kArgmaxThreads];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (takes(v[u], i + u * kArgmaxThreads, best, id)) {
                    best = v[u];
                    id = i + u * kArgmaxThreads;
                }
        }
    }
    for (; i < count; i += kArgmaxThreads) {
        const float v = Logits.get(base + i, err);
        if (takes(v, i, best, id)) {
            best = v;
            id = i;
        }
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const float ob = __shfl_down_sync(0xffffffffu, best, s);
        const int oi = __shfl_down_sync(0xffffffffu, id, s);
        if (takes(ob, oi, best, id)) {
            best = ob;
            id = oi;
        }
    }
    if (t == 0) {
        wbest[w] = best;
        wid[w] = id;
    }
    __syncthreads();
    if (w == 0) {
        best = wbest[t];
        id = wid[t];
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            const float ob = __shfl_down_sync(0xffffffffu, best, s);
            const int oi = __shfl_down_sync(0xffffffffu, id, s);
            if (takes(ob, oi, best, id)) {
                best = ob;
                id = oi;
            }
        }
        if (t == 0) Token.set(blockIdx.x, id, err);
    }
}

// ---------------------------------------------------------------- attention

// Sixteen 16-byte loads (p[0 .. 15]) issued back to back, one statement: all in flight at once.
__device__ __forceinline__ void ld16_v4(const float4 *p, float4 (&v)[16]) {
#pragma unroll
    for (int g = 0; g < 4; ++g)
        asm volatile(
            "ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%16];\n\t"
            "ld.global.nc.v4.f32 {%4, %5, %6, %7}, [%16 + 16];\n\t"
            "ld.global.nc.v4.f32 {%8, %9, %10, %11}, [%16 + 32];\n\t"
            "ld.global.nc.v4.f32 {%12, %13, %14, %15}, [%16 + 48];"
            : "=f"(v[4 * g].x), "=f"(v[4 * g].y), "=f"(v[4 * g].z), "=f"(v[4 * g].w), "=f"(v[4 * g + 1].x), "=f"(v[4 * g + 1].y),
              "=f"(v[4 * g + 1].z), "=f"(v[4 * g + 1].w), "=f"(v[4 * g + 2].x), "=f"(v[4 * g + 2].y), "=f"(v[4 * g + 2].z),
              "=f"(v[4 * g + 2].w), "=f"(v[4 * g + 3].x), "=f"(v[4 * g + 3].y), "=f"(v[4 * g + 3].z), "=f"(v[4 * g + 3].w)
            : "l"(p + 4 * g)
            : "memory");
}
// Sixteen 4-byte loads at p[i] (p[i] null: 0), issued back to back.
__device__ __forceinline__ void ld16_f(const float *const (&p)[16], float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        if (p[i]) asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v[i]) : "l"(p[i]) : "memory");
        else v[i] = 0.0f;
    }
}

// kernels/strata.cu:334-356 (decode: the Cells list, count cells) and :512-534 (prompt: query
// token = y, its causal prefix of position + token + 1 cells). One CTA per (head, query token)
// computes what the reference's (head, 64-wide tile) workgroups compute, each value by the same
// operations in the same order, without their redundancy:
//   A. the CTA's threads share out the cells; each score is one thread's in-order sum over the
//      head dimension (16-byte loads, four in flight), times `scale`, into shared memory;
//   B. one warp takes the maximum and the exponential sum in the reference's lane order and tree;
//   C. each output dimension d is one thread's in-order sum over the cells, divided by the sum.
// A key or value row outside its buffer reads as zeros and is reported.
constexpr int kAttnThreads = 512;
__global__ void __launch_bounds__(kAttnThreads) k_attention(Grid g, FB Q, FB Keys, FB Values, IB Cells, FB Y, int dim, int heads,
                                                            int kvHeads, int count, int position, float scale, int batch, IB Pos,
                                                            int seqCells, unsigned *err) {
    dep_enter();
    __shared__ float scores[kMaxCells];
    __shared__ long long value_row[kMaxCells];  // element offset of each cell's value row, or -1
    __shared__ float total_s;
    const unsigned h = blockIdx.x, token = blockIdx.y;
    const int tid = threadIdx.x;
    if ((int)h >= heads) return;
    // strata_attention_at: the prefix of one query; strata_attention_seqs (seqCells > 0): query
    // token t is sequence t's, over cells 0 .. Pos[t] of its own cache of seqCells cells
    if (Pos.n > 0) position = Pos.get(seqCells > 0 ? (long long)token : 0, err);
    const long long n = seqCells > 0 ? (long long)position + 1 : batch ? (long long)position + token + 1 : count;
    const long long cell0 = seqCells > 0 ? (long long)token * seqCells : 0;
    if (n < 1 || n > kMaxCells || (seqCells > 0 && n > seqCells)) {
        if (tid == 0) raise_error(err, kErrIndex);
        return;
    }
    const int kh = (int)h / (heads / kvHeads);
    const long long qbase = batch ? ((long long)token * heads + h) * dim : (long long)h * dim;
    const bool q_ok = covers(Q, qbase, dim);
    const bool vec = q_ok && dim % 4 == 0 && ((reinterpret_cast<uintptr_t>(Q.p) | reinterpret_cast<uintptr_t>(Keys.p)) & 15) == 0;
    for (int c = tid; c < n; c += kAttnThreads) {  // A
        const long long cell = batch ? c : (long long)Cells.get(c, err);
        const long long kb = ((cell0 + cell) * kvHeads + kh) * dim;
        const bool key_ok = cell >= 0 && covers(Keys, kb, dim), value_ok = cell >= 0 && covers(Values, kb, dim);
        if (!key_ok || !value_ok) raise_error(err, kErrIndex);
        float score = 0.0f;
        if (key_ok && vec) {
            const float4 *k4 = reinterpret_cast<const float4 *>(Keys.p + kb), *q4 = reinterpret_cast<const float4 *>(Q.p + qbase);
            const int d4 = dim / 4;
            int j = 0;
            for (; j + 16 <= d4; j += 16) {  // sixteen key loads in flight (one round trip for a 256-wide head)
                float4 kv[16];
                ld16_v4(k4 + j, kv);
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const float4 qv = q4[j + u];
                    score = __fadd_rn(score, __fmul_rn(qv.x, kv[u].x));
                    score = __fadd_rn(score, __fmul_rn(qv.y, kv[u].y));
                    score = __fadd_rn(score, __fmul_rn(qv.z, kv[u].z));
                    score = __fadd_rn(score, __fmul_rn(qv.w, kv[u].w));
                }
            }
            for (; j + 4 <= d4; j += 4) {
                float4 kv[4], qv[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    kv[u] = k4[j + u];
                    qv[u] = q4[j + u];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    score = __fadd_rn(score, __fmul_rn(qv[u].x, kv[u].x));
                    score = __fadd_rn(score, __fmul_rn(qv[u].y, kv[u].y));
                    score = __fadd_rn(score, __fmul_rn(qv[u].z, kv[u].z));
                    score = __fadd_rn(score, __fmul_rn(qv[u].w, kv[u].w));
                }
            }
            for (; j < d4; ++j) {
                const float4 kv = k4[j], qv = q4[j];
                score = __fadd_rn(score, __fmul_rn(qv.x, kv.x));
                score = __fadd_rn(score, __fmul_rn(qv.y, kv.y));
                score = __fadd_rn(score, __fmul_rn(qv.z, kv.z));
                score = __fadd_rn(score, __fmul_rn(qv.w, kv.w));
            }
        } else if (key_ok) {
            for (int j = 0; j < dim; ++j) score = __fadd_rn(score, __fmul_rn(Q.get(qbase + j, err), Keys.p[kb + j]));
        }
        scores[c] = __fmul_rn(score, scale);
        value_row[c] = value_ok ? kb : -1;
    }
    __syncthreads();
    if (tid < 32) {  // B
        float mlo = -3.402823e38f, mhi = -3.402823e38f;
        for (int c = tid; c < n; c += STRATA_LANES) mlo = fmaxf(mlo, scores[c]);
        for (int c = tid + 32; c < n; c += STRATA_LANES) mhi = fmaxf(mhi, scores[c]);
        const float m = __shfl_sync(0xffffffffu, max_tree64(mlo, mhi), 0);
        float slo = 0.0f, shi = 0.0f;
        for (int c = tid; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(scores[c], m));
            scores[c] = p;
            slo = __fadd_rn(slo, p);
        }
        for (int c = tid + 32; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(scores[c], m));
            scores[c] = p;
            shi = __fadd_rn(shi, p);
        }
        const float total = tree64(slo, shi);
        if (tid == 0) total_s = total;
    }
    __syncthreads();
    const float total = total_s;
    const int dmax = (int)min((long long)dim, (long long)g.y * STRATA_LANES);  // the dispatched 64-wide tiles
    for (int d = tid; d < dmax; d += kAttnThreads) {  // C
        float value = 0.0f;
        int c = 0;
        for (; c + 64 <= n; c += 64) {  // 64 value loads in flight ahead of the ordered sum
            float vv[4][16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float *ptr[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const long long r = value_row[c + 16 * q4 + u];
                    ptr[u] = r >= 0 ? Values.p + r + d : nullptr;
                }
                ld16_f(ptr, vv[q4]);
            }
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
                for (int u = 0; u < 16; ++u) value = __fadd_rn(value, __fmul_rn(scores[c + 16 * q4 + u], vv[q4][u]));
        }
        for (; c + 16 <= n; c += 16) {  // sixteen value loads in flight ahead of the ordered sum
            float vv[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const long long r = value_row[c + u];
                vv[u] = r >= 0 ? Values.p[r + d] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) value = __fadd_rn(value, __fmul_rn(scores[c + u], vv[u]));
        }
        for (; c < n; ++c) {
            const long long r = value_row[c];
            value = __fadd_rn(value, __fmul_rn(scores[c], r >= 0 ? Values.p[r + d] : 0.0f));
        }
        Y.set(qbase + d, __fdiv_rn(value, total), err);
    }
}

// The same attention for a few query tokens, split over an 8-CTA cluster per (head, query
// token) so that every SM streams a share of the keys and values (one CTA per head left 16 SMs
// reading the whole cache). Same values, same order:
//   A. CTA r scores cells [r m, r m + m) (m = n / 8 rounded up), each one thread's in-order sum
//      over the head dimension, times `scale`;
//   the cluster's CTAs then copy each other's scores from distributed shared memory;
//   B. one warp per CTA takes the maximum and the exponential sum in the reference's lane order
//      and tree (every CTA the same values);
//   C. CTA r forms output dimensions [r dim / 8, (r + 1) dim / 8): each one thread's in-order sum
//      over all cells, from value rows staged in shared memory by the whole CTA (64 cells at a
//      time, double-buffered), divided by the sum.
// Requires dim a multiple of 64 and at most 256, 16-byte aligned keys and values. A key or value
// row outside its buffer reads as zeros and is reported.
constexpr int kAcThreads = 256, kAcCluster = 8, kAcChunk = 64;
__device__ __forceinline__ unsigned ac_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void ac_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ac_ld_peer(const float *local, unsigned rank) {
    unsigned remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"((unsigned)__cvta_generic_to_shared(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}
__global__ void __cluster_dims__(kAcCluster, 1, 1) __launch_bounds__(kAcThreads)
    k_attention_cl(Grid g, FB Q, FB Keys, FB Values, IB Cells, FB Y, int dim, int heads, int kvHeads, int count, int position, float scale,
                   int batch, IB Pos, int seqCells, unsigned *err) {
    dep_enter();
    __shared__ float scores[kMaxCells];
    __shared__ long long value_row[kMaxCells];
    __shared__ __align__(16) float vst[2][kAcChunk][32];  // value rows' slices of this CTA's dimensions
    __shared__ float total_s;
    const unsigned rank = ac_rank(), h = blockIdx.x / kAcCluster, token = blockIdx.y;
    const int tid = threadIdx.x;
    if (Pos.n > 0) position = Pos.get(seqCells > 0 ? (long long)token : 0, err);  // as in k_attention
    const long long n = seqCells > 0 ? (long long)position + 1 : batch ? (long long)position + token + 1 : count;
    const long long cell0 = seqCells > 0 ? (long long)token * seqCells : 0;
    // every CTA of the cluster takes the same branch: the cluster barriers below are reached by all
    const bool run = (int)h < heads && n >= 1 && n <= kMaxCells && (seqCells <= 0 || n <= seqCells);
    if (!run && tid == 0 && (int)h < heads) raise_error(err, kErrIndex);
    const int kh = run ? (int)h / (heads / kvHeads) : 0;
    const long long qbase = batch ? ((long long)token * heads + h) * dim : (long long)h * dim;
    const bool q_ok = covers(Q, qbase, dim);
    const int m = run ? (int)((n + kAcCluster - 1) / kAcCluster) : 0;
    const int c0 = (int)rank * m, c1 = run ? (int)min(n, (long long)c0 + m) : 0;
    if (run) {
        for (int c = tid; c < n; c += kAcThreads) {  // every cell's value row (and its checks, once: by its scorer)
            const long long cell = batch ? c : (long long)Cells.get(c, err);
            const long long kb = ((cell0 + cell) * kvHeads + kh) * dim;
            const bool key_ok = cell >= 0 && covers(Keys, kb, dim), value_ok = cell >= 0 && covers(Values, kb, dim);
            value_row[c] = value_ok ? kb : -1;
            if (c >= c0 && c < c1) {  // A
                if (!key_ok || !value_ok || !q_ok) raise_error(err, kErrIndex);
                float score = 0.0f;
                if (key_ok && q_ok) {
                    const float4 *k4 = reinterpret_cast<const float4 *>(Keys.p + kb), *q4 = reinterpret_cast<const float4 *>(Q.p + qbase);
                    for (int j = 0; j < dim / 4; j += 16) {
                        float4 kv[16];
                        ld16_v4(k4 + j, kv);
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            const float4 qv = q4[j + u];
                            score = __fadd_rn(score, __fmul_rn(qv.x, kv[u].x));
                            score = __fadd_rn(score, __fmul_rn(qv.y, kv[u].y));
                            score = __fadd_rn(score, __fmul_rn(qv.z, kv[u].z));
                            score = __fadd_rn(score, __fmul_rn(qv.w, kv[u].w));
                        }
                    }
                }
                scores[c] = __fmul_rn(score, scale);
            }
        }
    }
    ac_cluster_sync();  // every CTA's scores are in its shared memory
    if (run)
        for (int c = tid; c < n; c += kAcThreads)
            if (c < c0 || c >= c1) scores[c] = ac_ld_peer(&scores[c], (unsigned)(c / m));
    ac_cluster_sync();  // every peer read done: the scores may be overwritten
    if (!run) return;
    if (tid < 32) {  // B
        float mlo = -3.402823e38f, mhi = -3.402823e38f;
        for (int c = tid; c < n; c += STRATA_LANES) mlo = fmaxf(mlo, scores[c]);
        for (int c = tid + 32; c < n; c += STRATA_LANES) mhi = fmaxf(mhi, scores[c]);
        const float mx = __shfl_sync(0xffffffffu, max_tree64(mlo, mhi), 0);
        float slo = 0.0f, shi = 0.0f;
        for (int c = tid; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(scores[c], mx));
            scores[c] = p;
            slo = __fadd_rn(slo, p);
        }
        for (int c = tid + 32; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(scores[c], mx));
            scores[c] = p;
            shi = __fadd_rn(shi, p);
        }
        const float total = tree64(slo, shi);
        if (tid == 0) total_s = total;
    }
    __syncthreads();
    // C: dimensions [d0, d0 + dp) of this CTA, 64 cells' slices staged per step
    const int dp = dim / kAcCluster, d0 = (int)rank * dp;
    const int dmax = (int)min((long long)dim, (long long)g.y * STRATA_LANES);  // the dispatched 64-wide tiles
    const int nv = dp / 4;  // 16-byte pieces of a row's slice
    auto stage = [&](int step, int buf) {
        for (int i = tid; i < kAcChunk * nv; i += kAcThreads) {
            const int cc = i / nv, piece = i % nv, c = step * kAcChunk + cc;
            float *dst = &vst[buf][cc][4 * piece];
            const long long r = c < n ? value_row[c] : -1;
            if (r >= 0) copy16_async(dst, Values.p + r + d0 + 4 * piece);
            else *reinterpret_cast<float4 *>(dst) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        copy_commit();
    };
    const int steps = (int)((n + kAcChunk - 1) / kAcChunk);
    const float total = total_s;
    float value = 0.0f;
    stage(0, 0);
    for (int st = 0; st < steps; ++st) {
        if (st + 1 < steps) {
            stage(st + 1, (st + 1) & 1);
            copy_wait<1>();
        } else {
            copy_wait<0>();
        }
        __syncthreads();
        if (tid < dp) {
            const int cend = (int)min((long long)kAcChunk, n - (long long)st * kAcChunk);
            const float *sc = scores + st * kAcChunk;
            for (int cc = 0; cc < cend; ++cc) value = __fadd_rn(value, __fmul_rn(sc[cc], vst[st & 1][cc][tid]));
        }
        __syncthreads();  // the buffer is refilled two steps on
    }
    if (tid < dp && d0 + tid < dmax) Y.set(qbase + d0 + tid, __fdiv_rn(value, total), err);
}

// The prompt form for a group of query heads that share one KV head (GQA): one block per (KV
// head, query token). Each key row is loaded once for the group's G scores (G independent
// in-order sums), one warp per head takes the maximum and the exponential sum in the reference's
// lane order, and each value is loaded once for four heads' in-order sums. Every value is formed
// by the same operations in the same order as in k_attention. Cells are 0 .. position + token; a
// key or value row outside its buffer reads as zeros and is reported. With seqCells > 0
// (strata_attention_seqs) query token t is sequence t's, over cells 0 .. Pos[t] of its own cache.
constexpr int kGroupThreads = 512, kMaxGroup = 8;
__global__ void __launch_bounds__(kGroupThreads) k_attention_group(Grid g, FB Q, FB Keys, FB Values, FB Y, int dim, int heads, int kvHeads,
                                                                   int position, float scale, IB Pos, int seqCells, unsigned *err) {
    dep_enter();
    extern __shared__ __align__(16) float group_smem[];  // [G][dim] queries, then [G][kMaxCells] scores
    __shared__ float totals[kMaxGroup];
    const int G = heads / kvHeads, kh = blockIdx.x, token = blockIdx.y, tid = threadIdx.x;
    if (Pos.n > 0) position = Pos.get(seqCells > 0 ? token : 0, err);
    const long long n = seqCells > 0 ? (long long)position + 1 : (long long)position + token + 1;
    const long long cell0 = seqCells > 0 ? (long long)token * seqCells : 0;
    if (n < 1 || n > kMaxCells || (seqCells > 0 && n > seqCells)) {
        if (tid == 0) raise_error(err, kErrIndex);
        return;
    }
    float *qs = group_smem, *scores = group_smem + (size_t)G * dim;
    const long long qbase = ((long long)token * heads + (long long)kh * G) * dim;  // the group's G query rows are consecutive
    for (int k = tid; k < G * dim; k += kGroupThreads) qs[k] = Q.get(qbase + k, err);
    __syncthreads();
    for (int c = tid; c < n; c += kGroupThreads) {  // A
        const long long kb = ((cell0 + c) * kvHeads + kh) * dim;
        float sc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) sc[h] = 0.0f;
        if (covers(Keys, kb, dim)) {
            const float4 *k4 = reinterpret_cast<const float4 *>(Keys.p + kb);
            auto step = [&](const float4 kv, int j4) {
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h) {
                    if (h >= G) break;
                    const float *q = qs + h * dim + 4 * j4;
                    sc[h] = __fadd_rn(sc[h], __fmul_rn(q[0], kv.x));
                    sc[h] = __fadd_rn(sc[h], __fmul_rn(q[1], kv.y));
                    sc[h] = __fadd_rn(sc[h], __fmul_rn(q[2], kv.z));
                    sc[h] = __fadd_rn(sc[h], __fmul_rn(q[3], kv.w));
                }
            };
            int j4 = 0;
            for (; j4 + 8 <= dim / 4; j4 += 8) {  // eight 16-byte key loads in flight ahead of the ordered sums
                float4 kv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) kv[u] = k4[j4 + u];
#pragma unroll
                for (int u = 0; u < 8; ++u) step(kv[u], j4 + u);
            }
            for (; j4 < dim / 4; ++j4) step(k4[j4], j4);
        } else {
            raise_error(err, kErrIndex);
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) scores[(size_t)h * kMaxCells + c] = __fmul_rn(sc[h], scale);
    }
    __syncthreads();
    const int warp = tid / 32, t = tid & 31;
    if (warp < G) {  // B: head `warp`
        float *sh = scores + (size_t)warp * kMaxCells;
        float mlo = -3.402823e38f, mhi = -3.402823e38f;
        for (int c = t; c < n; c += STRATA_LANES) mlo = fmaxf(mlo, sh[c]);
        for (int c = t + 32; c < n; c += STRATA_LANES) mhi = fmaxf(mhi, sh[c]);
        const float m = __shfl_sync(0xffffffffu, max_tree64(mlo, mhi), 0);
        float slo = 0.0f, shi = 0.0f;
        for (int c = t; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(sh[c], m));
            sh[c] = p;
            slo = __fadd_rn(slo, p);
        }
        for (int c = t + 32; c < n; c += STRATA_LANES) {
            const float p = ref_expf(__fsub_rn(sh[c], m));
            sh[c] = p;
            shi = __fadd_rn(shi, p);
        }
        const float total = tree64(slo, shi);
        if (t == 0) totals[warp] = total;
    }
    __syncthreads();
    const int dmax = (int)min((long long)dim, (long long)g.y * STRATA_LANES);
    constexpr int kHeadsPerThread = 4;
    const int quads = (G + kHeadsPerThread - 1) / kHeadsPerThread;
    for (int w = tid; w < dmax * quads; w += kGroupThreads) {  // C: dimension d of heads h0 .. h0 + 3
        const int d = w % dmax, h0 = (w / dmax) * kHeadsPerThread;
        float value[kHeadsPerThread] = {0.0f, 0.0f, 0.0f, 0.0f};
        int c = 0;
        for (; c + 32 <= n; c += 32) {  // 32 value loads in flight ahead of the ordered sums
            float v[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) {
                const long long vb = ((cell0 + c + u) * kvHeads + kh) * dim;
                v[u] = covers(Values, vb, dim) ? Values.p[vb + d] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 32; ++u)
#pragma unroll
                for (int q = 0; q < kHeadsPerThread; ++q)
                    if (h0 + q < G) value[q] = __fadd_rn(value[q], __fmul_rn(scores[(size_t)(h0 + q) * kMaxCells + c + u], v[u]));
        }
        for (; c < n; ++c) {
            const long long vb = ((cell0 + c) * kvHeads + kh) * dim;
            const float v = covers(Values, vb, dim) ? Values.p[vb + d] : 0.0f;
#pragma unroll
            for (int q = 0; q < kHeadsPerThread; ++q)
                if (h0 + q < G) value[q] = __fadd_rn(value[q], __fmul_rn(scores[(size_t)(h0 + q) * kMaxCells + c], v));
        }
#pragma unroll
        for (int u = 0; u < kHeadsPerThread; ++u)
            if (h0 + u < G) Y.set(((long long)token * heads + (long long)kh * G + h0 + u) * dim + d, __fdiv_rn(value[u], totals[h0 + u]), err);
    }
}

// The cluster form's conditions: a head dimension of whole 64-element key loads, at most 256 (eight
// slices of at most 32), 16-byte aligned key and value buffers, whole KV groups.
static bool attention_cl_ok(const KArg &k, const KArg &v, int dim, int heads, int kvHeads, const unsigned g[3]) {
    return dim >= 64 && dim <= 256 && dim % 64 == 0 && kvHeads >= 1 && heads % kvHeads == 0 && g[0] >= 1 &&
           ((reinterpret_cast<uintptr_t>(k.ptr) | reinterpret_cast<uintptr_t>(v.ptr)) & 15) == 0;
}
cudaError_t launch_attention_prompt(const KArg *a, int qi, int ki, int vi, int yi, int dim, int heads, int kvHeads, int position, float scale,
                                    IB pos, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int G = kvHeads > 0 ? heads / kvHeads : 0;
    const size_t bytes = ((size_t)G * dim + (size_t)G * kMaxCells) * 4;
    const bool aligned = ((reinterpret_cast<uintptr_t>(a[ki].ptr)) & 15) == 0;
    if (g[2] >= 8 && G >= 1 && G <= kMaxGroup && heads % kvHeads == 0 && dim % 4 == 0 && aligned && bytes <= 200 * 1024 &&
        g[0] >= (unsigned)heads) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_group, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        launch_k(false, k_attention_group, dim3(kvHeads, g[2]), kGroupThreads, bytes, s, grid_of(g), F(qi), F(ki), F(vi), F(yi), dim, heads, kvHeads,
                                                                           position, scale, pos, 0, err);
        return cudaGetLastError();
    }
    if (attention_cl_ok(a[ki], a[vi], dim, heads, kvHeads, g)) {
        launch_k(g[2] == 1, k_attention_cl, dim3(g[0] * kAcCluster, g[2]), kAcThreads, 0, s, grid_of(g), F(qi), F(ki), F(vi), IB{nullptr, 0}, F(yi), dim,
                                                                            heads, kvHeads, 0, position, scale, 1, pos, 0, err);
        return cudaGetLastError();
    }
    launch_k(g[2] == 1, k_attention, dim3(g[0], g[2]), kAttnThreads, 0, s, grid_of(g), F(qi), F(ki), F(vi), IB{nullptr, 0}, F(yi), dim, heads, kvHeads, 0,
                                                          position, scale, 1, pos, 0, err);
    return cudaGetLastError();
}

// kernels/strata.cu:328-330 and :453-456
// With seqCells > 0 (strata_kv_append_seqs, no reference counterpart) token t's row goes to cell
// Pos[t] of sequence t's own cache, cells [t seqCells, (t + 1) seqCells) of Keys and Values.
__global__ void k_kv_append(Grid g, FB K, FB V, FB Keys, FB Values, int width, int position, int tokens, IB Pos, int seqCells,
                            unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)width * tokens);
    if (i < 0) return;
    const long long token = i / width;
    if (Pos.n > 0) position = Pos.get(seqCells > 0 ? token : 0, err);
    if (seqCells > 0 && (position < 0 || position >= seqCells)) {
        raise_error(err, kErrIndex);
        return;
    }
    const long long at = seqCells > 0 ? (token * seqCells + position) * width + i % width : (long long)position * width + i;
    Keys.set(at, K.get(i, err), err);
    Values.set(at, V.get(i, err), err);
}

// kernels/strata.cu:357-359 and :457-459: attention output times sigmoid of the gate half of
// each head's [query | gate] row.
__global__ void k_attention_gate(Grid g, FB Attention, FB FullQ, FB Y, int dim, int heads, int tokens, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)dim * heads * tokens);
    if (i >= 0) Y.set(i, __fmul_rn(Attention.get(i, err), ref_sigmoid(FullQ.get((i / dim) * dim * 2 + dim + i % dim, err))), err);
}

// kernels/strata.cu:314-316
__global__ void k_slice(Grid g, FB X, FB Y, int width, int rows, int stride, int offset, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)width * rows);
    if (i >= 0) Y.set(i, X.get((i / width) * stride + offset + i % width, err), err);
}

// ---------------------------------------------------------------- hyper-connections

// kernels/strata.cu:273-277 and :403-408: mean over streams of norm * sigmoid(gate).
__global__ void k_hc_mix(Grid g, FB Norm, FB Gate, FB Mixed, int width, int streams, int tokens, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)width * tokens);
    if (i < 0) return;
    const long long token = i / width, d = i % width;
    float v = 0.0f;
    for (int c = 0; c < streams; ++c) {
        const long long p = (token * streams + c) * width + d;
        v = __fadd_rn(v, __fmul_rn(Norm.get(p, err), ref_sigmoid(Gate.get(p, err))));
    }
    Mixed.set(i, __fdiv_rn(v, (float)streams), err);
}

// kernels/strata.cu:278-281 and :409-412: residual += output * 2 sigmoid(inject / streams).
__global__ void k_hc_write(Grid g, FB Residual, FB Output, FB Inject, int width, int streams, int tokens, unsigned *err) {
    dep_enter();
    const long long hc = (long long)width * streams;
    long long i = lane_index(g, hc * tokens);
    if (i < 0) return;
    const float gain = __fmul_rn(2.0f, ref_sigmoid(__fdiv_rn(Inject.get(i / width, err), (float)streams)));
    Residual.set(i, __fadd_rn(Residual.get(i, err), __fmul_rn(Output.get((i / hc) * width + i % width, err), gain)), err);
}

// ---------------------------------------------------------------- per-layer embeddings

// kernels/strata.cu:378-380 and :460-463
__global__ void k_ple_broadcast(Grid g, FB Value, FB Gate, FB Y, int width, int streams, int tokens, unsigned *err) {
    dep_enter();
    const long long hc = (long long)width * streams;
    long long i = lane_index(g, hc * tokens);
    if (i >= 0) Y.set(i, __fmul_rn(Value.get((i / hc) * width + i % width, err), Gate.get(i / width, err)), err);
}

// kernels/strata.cu:381-383
__global__ void k_ple_add(Grid g, FB Residual, FB Gated, FB Conv, int n, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, n);
    if (i >= 0) Residual.set(i, __fadd_rn(Residual.get(i, err), __fadd_rn(Gated.get(i, err), Conv.get(i, err))), err);
}

// ---------------------------------------------------------------- recurrences

// kernels/strata.cu:287-295 and :413-424: causal convolution over a channel-major history
// (tap 0 oldest), optional SiLU, then the history shifts by one. One thread per channel walks
// the tokens in order; neighbouring channels are neighbouring threads.
__global__ void k_conv(Grid g, FB History, FB X, FB W, FB Y, int channels, int taps, int dilation, int activation, int tokens, int batch,
                       unsigned *err) {
    dep_enter();
    long long c = lane_index(g, channels);
    if (c < 0) return;
    const long long history = (long long)(taps - 1) * dilation, hbase = c * history;
    for (int token = 0; token < tokens; ++token) {
        const long long at = (long long)token * channels + c;
        float sum = 0.0f;
        for (int t = 0; t < taps - 1; ++t)
            sum = __fadd_rn(sum, __fmul_rn(History.get(hbase + (long long)t * dilation, err), W.get(c * taps + t, err)));
        const float x = X.get(at, err);
        sum = __fadd_rn(sum, __fmul_rn(x, W.get(c * taps + taps - 1, err)));
        Y.set(at, activation == 1 ? ref_silu(sum) : sum, err);
        for (long long t = 0; t < history - 1; ++t) History.set(hbase + t, History.get(hbase + t + 1, err), err);
        if (batch || history > 0) History.set(hbase + history - 1, x, err);
    }
}

// The same convolution with the channel's history in registers across the tokens, for the tap
// counts and dilations known at compile time (the model's 4 taps at dilations 1 and 3); loaded
// and stored once per dispatch. Launched only when the host's layout checks cover every index.
template <int TAPS, int DIL>
__global__ void k_conv_reg(Grid g, FB History, FB X, FB W, FB Y, int channels, int activation, int tokens) {
    dep_enter();
    constexpr int H = (TAPS - 1) * DIL;
    const long long c = lane_index(g, channels);
    if (c < 0) return;
    float hist[H], w[TAPS];
#pragma unroll
    for (int k = 0; k < H; ++k) hist[k] = History.p[c * H + k];
#pragma unroll
    for (int k = 0; k < TAPS; ++k) w[k] = W.p[c * TAPS + k];
    for (int token = 0; token < tokens; ++token) {
        const long long at = (long long)token * channels + c;
        const float x = X.p[at];
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < TAPS - 1; ++k) sum = __fadd_rn(sum, __fmul_rn(hist[k * DIL], w[k]));
        sum = __fadd_rn(sum, __fmul_rn(x, w[TAPS - 1]));
        Y.p[at] = activation == 1 ? ref_silu(sum) : sum;
#pragma unroll
        for (int k = 0; k + 1 < H; ++k) hist[k] = hist[k + 1];
        hist[H - 1] = x;
    }
#pragma unroll
    for (int k = 0; k < H; ++k) History.p[c * H + k] = hist[k];
}

cudaError_t launch_conv(const KArg *a, const unsigned g[3], int tokens, int batch, cudaStream_t s, unsigned *err) {
    const int channels = a[4].i, taps = a[5].i, dil = a[6].i, act = a[7].i;
    const long long c = channels;
    const bool covered = c >= 1 && a[0].len >= c * (taps - 1) * dil && a[2].len >= c * taps && a[1].len >= tokens * c &&
                         a[3].len >= tokens * c;
    if (covered && taps == 4 && dil == 1) {
        launch_k(tokens == 1, k_conv_reg<4, 1>, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, act, tokens);
    } else if (covered && taps == 4 && dil == 3) {
        launch_k(tokens == 1, k_conv_reg<4, 3>, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, act, tokens);
    } else {
        launch_k(tokens == 1, k_conv, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, taps, dil, act, tokens, batch, err);
    }
    return cudaGetLastError();
}

// strata_conv_seqs (no counterpart in the reference): one token of each of `tokens` independent
// sequences, token t with its own history [t channels (taps - 1) dilation, ...), each channel's
// value by strata_conv's operations in its order. One thread per (token, channel).
__global__ void k_conv_seqs(Grid g, FB History, FB X, FB W, FB Y, int channels, int taps, int dilation, int activation, int tokens,
                            unsigned *err) {
    dep_enter();
    const long long i = lane_index(g, (long long)channels * tokens);
    if (i < 0) return;
    const long long c = i % channels, history = (long long)(taps - 1) * dilation, hbase = i * history;
    float sum = 0.0f;
    for (int t = 0; t < taps - 1; ++t)
        sum = __fadd_rn(sum, __fmul_rn(History.get(hbase + (long long)t * dilation, err), W.get(c * taps + t, err)));
    const float x = X.get(i, err);
    sum = __fadd_rn(sum, __fmul_rn(x, W.get(c * taps + taps - 1, err)));
    Y.set(i, activation == 1 ? ref_silu(sum) : sum, err);
    for (long long t = 0; t < history - 1; ++t) History.set(hbase + t, History.get(hbase + t + 1, err), err);
    if (history > 0) History.set(hbase + history - 1, x, err);
}

// The same with the tap count and dilation known at compile time (the model's 4 taps at dilations
// 1 and 3): the thread's history and weights in registers, loaded and stored once. Launched only
// when the host's layout checks cover every index.
template <int TAPS, int DIL>
__global__ void k_conv_seqs_reg(Grid g, FB History, FB X, FB W, FB Y, int channels, int activation, int tokens) {
    dep_enter();
    constexpr int H = (TAPS - 1) * DIL;
    const long long i = lane_index(g, (long long)channels * tokens);
    if (i < 0) return;
    const long long c = i % channels;
    float hist[H], w[TAPS];
#pragma unroll
    for (int k = 0; k < H; ++k) hist[k] = History.p[i * H + k];
#pragma unroll
    for (int k = 0; k < TAPS; ++k) w[k] = W.p[c * TAPS + k];
    const float x = X.p[i];
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < TAPS - 1; ++k) sum = __fadd_rn(sum, __fmul_rn(hist[k * DIL], w[k]));
    sum = __fadd_rn(sum, __fmul_rn(x, w[TAPS - 1]));
    Y.p[i] = activation == 1 ? ref_silu(sum) : sum;
#pragma unroll
    for (int k = 0; k + 1 < H; ++k) History.p[i * H + k] = hist[k + 1];
    History.p[i * H + H - 1] = x;
}

// strata_gdn_prep (no counterpart in the reference): the delta-rule layer's input sequence of one
// token (src/engine.js's strata_conv (4 taps, dilation 1, SiLU) over the [q | k | v] projection,
// three strata_slice, then the L2 norms of the q heads (times qScale) and of the k heads,
// strata_norm mode 1) in one launch, each value by the same operations in the same order. Block
// b takes channels [2 hd b, 2 hd b + 2 hd): two heads' worth of q, k or v channels (keyDim and
// valueDim are multiples of 2 hd): the conv per channel, as k_conv_reg, into shared memory and
// the history; then two warps norm the block's two q or k heads as k_norm does (lane_dot, tree),
// or the v channels are copied out.
constexpr int kPrepThreads = 256;
__global__ void __launch_bounds__(kPrepThreads) k_gdn_prep(FB History, FB X, FB W, FB Q, FB K, FB V, int keyDim, int valueDim, int hd,
                                                           float qScale, float epsilon) {
    dep_enter();
    extern __shared__ float prep[];  // [2 hd] the block's convolved channels
    const int tid = threadIdx.x, warp = tid >> 5, t = tid & 31, span = 2 * hd;
    const long long c0 = (long long)blockIdx.x * span;
    for (int i = tid; i < span; i += kPrepThreads) {  // k_conv_reg<4, 1>, one token
        const long long c = c0 + i;
        float hist[3], w[4];
#pragma unroll
        for (int k = 0; k < 3; ++k) hist[k] = History.p[c * 3 + k];
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = W.p[c * 4 + k];
        const float x = X.p[c];
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 3; ++k) sum = __fadd_rn(sum, __fmul_rn(hist[k], w[k]));
        sum = __fadd_rn(sum, __fmul_rn(x, w[3]));
        prep[i] = ref_silu(sum);
        History.p[c * 3 + 0] = hist[1];
        History.p[c * 3 + 1] = hist[2];
        History.p[c * 3 + 2] = x;
    }
    __syncthreads();
    if (c0 >= 2LL * keyDim) {  // v channels: the slice
        for (int i = tid; i < span; i += kPrepThreads) V.p[c0 - 2LL * keyDim + i] = prep[i];
        return;
    }
    if (warp >= 2) return;
    const bool is_q = c0 < keyDim;
    const float scale = is_q ? qScale : 1.0f;
    const float *x = prep + warp * hd;
    float *y = (is_q ? Q.p + c0 : K.p + (c0 - keyDim)) + warp * hd;
    const float ss = __shfl_sync(0xffffffffu, lane_dot(x, x, hd, t), 0);
    const float inv = __fdiv_rn(scale, __fsqrt_rn(__fadd_rn(ss, epsilon)));  // k_norm, mode 1
    for (int i = t; i < hd; i += 32) y[i] = __fmul_rn(__fmul_rn(x[i], inv), 1.0f);
}
cudaError_t L_gdn_prep(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const long long kd = a[6].i, vd = a[7].i, hd = a[8].i, c = 2 * kd + vd;
    if (hd < 32 || hd > 1024 || kd < 2 * hd || kd % (2 * hd) != 0 || vd % (2 * hd) != 0 || a[0].len < 3 * c || a[1].len < c ||
        a[2].len < 4 * c || a[3].len < kd || a[4].len < kd || a[5].len < vd)
        return cudaErrorInvalidValue;
    launch_k(true, k_gdn_prep, (unsigned)(c / (2 * hd)), kPrepThreads, (size_t)(2 * hd) * 4, s, F(0), F(1), F(2), F(3), F(4), F(5), (int)kd, (int)vd,
                                                                                   (int)hd, a[9].f, a[10].f);
    return cudaGetLastError();
}

// kernels/strata.cu:296-301 and :425-431: decay = exp(A softplus(alpha + dt)), strength = sigmoid(beta).
__global__ void k_gdn_gates(Grid g, FB Alpha, FB Beta, FB A, FB Dt, FB Decay, FB Strength, int heads, int tokens, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)heads * tokens);
    if (i < 0) return;
    const float x = __fadd_rn(Alpha.get(i, err), Dt.get(i % heads, err));
    const float sp = x > 20.0f ? x : log_f(__fadd_rn(1.0f, ref_expf(x)));
    Decay.set(i, ref_expf(__fmul_rn(A.get(i % heads, err), sp)), err);
    Strength.set(i, ref_sigmoid(Beta.get(i, err)), err);
}

// strata_gdn_gates_fused (no counterpart in the reference): the delta-rule layer's alpha and beta
// projections of each token (strata_project: rows h of AlphaW and BetaW dotted with the token's
// row of X, the reference's 64-lane order and tree) and then strata_gdn_gates, in one launch, each
// value by the same operations in the same order. Block (h, t) stages the two weight rows (L2
// prefetch before the wait on the previous kernel) and the token's input row in shared memory
// with 16-byte loads; warp 0 forms alpha, warp 1 beta, thread 0 the gates. The host checks that
// every row read lies inside its buffer.
constexpr int kGatesThreads = 128;
__global__ void __launch_bounds__(kGatesThreads) k_gdn_gates_fused(FB X, FB AlphaW, FB BetaW, FB A, FB Dt, FB Decay, FB Strength, int width,
                                                                   int heads) {
    const int h = blockIdx.x, t = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *aw = AlphaW.p + (long long)h * width, *bw = BetaW.p + (long long)h * width;
    if (threadIdx.x == 0) {  // weights: no kernel writes them
        prefetch_l2(aw, (unsigned long long)width * 4);
        prefetch_l2(bw, (unsigned long long)width * 4);
    }
    dep_enter();
    extern __shared__ __align__(16) float gates_smem[];  // [3][width]: alpha row, beta row, input row
    __shared__ float ab[2];
    stage_row(gates_smem, aw, width);
    stage_row(gates_smem + width, bw, width);
    stage_row(gates_smem + 2 * width, X.p + (long long)t * width, width);
    __syncthreads();
    if (warp < 2) {
        const float r = lane_dot(gates_smem + warp * width, gates_smem + 2 * width, width, lane);
        if (lane == 0) ab[warp] = r;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const long long i = (long long)t * heads + h;
        const float x = __fadd_rn(ab[0], Dt.p[h]);
        const float sp = x > 20.0f ? x : log_f(__fadd_rn(1.0f, ref_expf(x)));
        Decay.p[i] = ref_expf(__fmul_rn(A.p[h], sp));
        Strength.p[i] = ref_sigmoid(ab[1]);
    }
}

// kernels/strata.cu:304-313 and :432-444: the gated delta rule. State is [dim_k][valueHeads][dim_v];
// thread jh owns column jh of every key row, so each of its dim loads is one coalesced row.
// Value head h reads key head h % keyHeads.
__global__ void k_gdn(Grid g, FB State, FB Q, FB K, FB V, FB Decay, FB Beta, FB Y, int dim, int keyHeads, int valueHeads, int tokens,
                      unsigned *err) {
    dep_enter();
    const long long stride = (long long)valueHeads * dim;
    long long jh = lane_index(g, stride);
    if (jh < 0) return;
    const long long h = jh / dim, kh = h % keyHeads;
    for (int token = 0; token < tokens; ++token) {
        const long long kbase = ((long long)token * keyHeads + kh) * dim, gh = (long long)token * valueHeads + h;
        const float decay = Decay.get(gh, err);
        float prediction = 0.0f;
        for (int i = 0; i < dim; ++i) {
            const long long ix = i * stride + jh;
            const float s = __fmul_rn(State.get(ix, err), decay);
            State.set(ix, s, err);
            prediction = __fadd_rn(prediction, __fmul_rn(s, K.get(kbase + i, err)));
        }
        const float delta = __fmul_rn(__fsub_rn(V.get(token * stride + jh, err), prediction), Beta.get(gh, err));
        float result = 0.0f;
        for (int i = 0; i < dim; ++i) {
            const long long ix = i * stride + jh;
            const float s = __fadd_rn(State.get(ix, err), __fmul_rn(K.get(kbase + i, err), delta));
            State.set(ix, s, err);
            result = __fadd_rn(result, __fmul_rn(s, Q.get(kbase + i, err)));
        }
        Y.set(token * stride + jh, result, err);
    }
}

// The same rule with the thread's state column in registers (DIM known at compile time), one
// block of DIM threads per value head: the head's key and query rows of each token are staged in
// shared memory and read through a volatile view, so the compiler issues them in order beside
// the accumulation chains instead of holding all 2 x DIM of them in registers.
// SEQS (strata_gdn_seqs, no reference counterpart): block (h, t) runs token t alone on sequence
// t's own state, [t DIM stride, (t + 1) DIM stride) of State.
template <int DIM, bool SEQS>
__global__ void __launch_bounds__(DIM) k_gdn_regs(FB State, FB Q, FB K, FB V, FB Decay, FB Beta, FB Y, int keyHeads, int valueHeads,
                                                  int tokens, long long columns) {
    dep_enter();
    __shared__ float ks[DIM], qs[DIM];
    const volatile float *kv = ks, *qv = qs;
    const long long stride = (long long)valueHeads * DIM;
    const long long h = blockIdx.x, jh = h * DIM + threadIdx.x, kh = h % keyHeads;
    const int x = threadIdx.x;
    const bool active = jh < columns;
    if (SEQS) State.p += (long long)blockIdx.y * DIM * stride;
    const int first = SEQS ? (int)blockIdx.y : 0, end = SEQS ? first + 1 : tokens;
    float st[DIM];
#pragma unroll
    for (int i = 0; i < DIM; ++i) st[i] = active ? State.p[i * stride + jh] : 0.0f;
    for (int token = first; token < end; ++token) {
        const long long kbase = ((long long)token * keyHeads + kh) * DIM, gh = (long long)token * valueHeads + h;
        ks[x] = K.p[kbase + x];
        qs[x] = Q.p[kbase + x];
        __syncthreads();
        const float decay = Decay.p[gh];
        float prediction = 0.0f;
#pragma unroll
        for (int i = 0; i < DIM; ++i) {
            st[i] = __fmul_rn(st[i], decay);
            prediction = __fadd_rn(prediction, __fmul_rn(st[i], kv[i]));
        }
        const float delta = __fmul_rn(__fsub_rn(active ? V.p[token * stride + jh] : 0.0f, prediction), Beta.p[gh]);
        float result = 0.0f;
#pragma unroll
        for (int i = 0; i < DIM; ++i) {
            st[i] = __fadd_rn(st[i], __fmul_rn(kv[i], delta));
            result = __fadd_rn(result, __fmul_rn(st[i], qv[i]));
        }
        if (active) Y.p[token * stride + jh] = result;
        __syncthreads();
    }
    if (active) {
#pragma unroll
        for (int i = 0; i < DIM; ++i) State.p[i * stride + jh] = st[i];
    }
}

// The register form when dim is 128 and the buffers cover every index, else the checked kernel.
cudaError_t launch_gdn(const Grid g, const KArg *a, int tokens, cudaStream_t s, unsigned *err) {
    const int dim = a[7].i, kh = a[8].i, vh = a[9].i;
    const long long stride = (long long)vh * dim, columns = std::min(stride, (long long)g.x * STRATA_LANES);
    const bool covered = a[0].len >= (long long)dim * stride && a[1].len >= (long long)tokens * kh * dim &&
                         a[2].len >= (long long)tokens * kh * dim && a[3].len >= tokens * stride && a[4].len >= (long long)tokens * vh &&
                         a[5].len >= (long long)tokens * vh && a[6].len >= tokens * stride && kh >= 1 && vh >= 1;
    if (dim == 128 && covered) {
        launch_k(tokens == 1, k_gdn_regs<128, false>, (unsigned)((columns + 127) / 128), 128, 0, s, F(0), F(1), F(2), F(3), F(4), F(5), F(6), kh, vh, tokens,
                                                                          columns);
    } else {
        launch_k(tokens == 1, k_gdn, (unsigned)(((unsigned long long)g.x * STRATA_LANES + 255) / 256), 256, 0, s, g, F(0), F(1), F(2), F(3), F(4), F(5), F(6),
                                                                                             dim, kh, vh, tokens, err);
    }
    return cudaGetLastError();
}

// strata_gdn_seqs (no counterpart in the reference), the checked form: one token of each of
// `tokens` independent sequences, token t on its own state [t dim stride, (t + 1) dim stride),
// each value by strata_gdn_step's operations in its order. One thread per (token, column).
__global__ void k_gdn_seqs(Grid g, FB State, FB Q, FB K, FB V, FB Decay, FB Beta, FB Y, int dim, int keyHeads, int valueHeads, int tokens,
                           unsigned *err) {
    dep_enter();
    const long long stride = (long long)valueHeads * dim;
    const long long i = lane_index(g, stride * tokens);
    if (i < 0) return;
    const long long token = i / stride, jh = i % stride, h = jh / dim, kh = h % keyHeads;
    const long long sbase = token * dim * stride, kbase = (token * keyHeads + kh) * dim, gh = token * valueHeads + h;
    const float decay = Decay.get(gh, err);
    float prediction = 0.0f;
    for (int k = 0; k < dim; ++k) {
        const long long ix = sbase + k * stride + jh;
        const float s = __fmul_rn(State.get(ix, err), decay);
        State.set(ix, s, err);
        prediction = __fadd_rn(prediction, __fmul_rn(s, K.get(kbase + k, err)));
    }
    const float delta = __fmul_rn(__fsub_rn(V.get(i, err), prediction), Beta.get(gh, err));
    float result = 0.0f;
    for (int k = 0; k < dim; ++k) {
        const long long ix = sbase + k * stride + jh;
        const float s = __fadd_rn(State.get(ix, err), __fmul_rn(K.get(kbase + k, err), delta));
        State.set(ix, s, err);
        result = __fadd_rn(result, __fmul_rn(s, Q.get(kbase + k, err)));
    }
    Y.set(i, result, err);
}

// ---------------------------------------------------------------- hyper-connection blocks
// No counterpart in the reference: the decode step's hyper-connection sequence (src/engine.js:
// 78-84: norm -> down projection -> SiLU(x / streams) -> up projection -> mix, and the inject
// projection of the same norm) in two launches instead of six, each value formed by the same
// operations in the same order as the reference entries (k_norm, k_project, k_elementwise,
// k_hc_mix). Neither needs a grid-wide wait: each block recomputes the small shared inputs.
constexpr int kHcThreads = 128;

// strata_hc_in: Norm = RMSNorm of the `streams` residual rows (gamma row = stream), then
// Down = down . Norm (rank rows of width*streams) and Inject = inject . Norm (streams rows). One
// block per output row copies the residual, its weight row and the gammas into shared memory
// with asynchronous 16-byte copies (all in flight at once), forms the norm there (one warp per
// stream row, as k_norm does) and one warp takes the row's ordered dot. Block 0 also writes the
// norm.
constexpr int kHcInThreads = 256;
__global__ void __launch_bounds__(kHcInThreads) k_hc_in(FB Residual, FB NormW, FB DownW, FB InjectW, FB Norm, FB Down, FB Inject, int width,
                                                        int streams, int rank, float epsilon) {
    extern __shared__ __align__(16) float hc_in[];  // [hc] residual -> norm, [hc] the weight row, [hc] the gammas
    __shared__ float inv_s[64];
    const int warp = threadIdx.x / 32, t = threadIdx.x & 31, hc = width * streams, j = blockIdx.x;
    float *x = hc_in, *w = hc_in + hc, *gam = hc_in + 2 * (size_t)hc;
    const float *wsrc = j < rank ? DownW.p + (long long)j * hc : InjectW.p + (long long)(j - rank) * hc;
    if (threadIdx.x == 0) prefetch_l2(wsrc, (unsigned long long)hc * 4);  // weights: before the previous kernel ends
    dep_enter();
    if (((reinterpret_cast<uintptr_t>(Residual.p) | reinterpret_cast<uintptr_t>(wsrc) | reinterpret_cast<uintptr_t>(NormW.p)) & 15) == 0 &&
        hc % 4 == 0) {
        for (int k = 4 * threadIdx.x; k < hc; k += 4 * kHcInThreads) {
            copy16_async(x + k, Residual.p + k);
            copy16_async(w + k, wsrc + k);
            copy16_async(gam + k, NormW.p + k);
        }
        copy_commit();
        copy_wait<0>();
    } else {
        stage_row(x, Residual.p, hc);
        stage_row(w, wsrc, hc);
        stage_row(gam, NormW.p, hc);
    }
    __syncthreads();
    for (int c = warp; c < streams; c += kHcInThreads / 32) {
        const float ss = lane_dot(x + (size_t)c * width, x + (size_t)c * width, width, t);
        if (t == 0) inv_s[c] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)width), epsilon)));
    }
    __syncthreads();
    for (int k = threadIdx.x; k < hc; k += kHcInThreads) x[k] = __fmul_rn(__fmul_rn(x[k], inv_s[k / width]), gam[k]);
    __syncthreads();
    if (j == 0)
        for (int k = threadIdx.x; k < hc; k += kHcInThreads) Norm.p[k] = x[k];
    if (warp == 0) {
        const float r = lane_dot(w, x, hc, t);
        if (t == 0) {
            if (j < rank) Down.p[j] = r;
            else Inject.p[j - rank] = r;
        }
    }
}

// strata_hc_out: Mixed[d] = sum_c Norm[c, d] * sigmoid(up[c, d] . lo) / streams with
// lo = SiLU(Down / streams) (elementwise mode 1, scale = 1/streams). Every block forms lo in shared
// memory; one warp per output column d computes its `streams` gate rows and the mix. With rank
// 256 and at most 4 streams a lane loads its elements of every gate row first (one round trip),
// then each row's two reference-lane sums run in order, as lane_dot's.
__global__ void __launch_bounds__(kHcThreads) k_hc_out(FB Norm, FB Down, FB UpW, FB Mixed, int width, int streams, int rank, float scale) {
    extern __shared__ __align__(16) float hc_lo[];  // [rank]
    const int warp = threadIdx.x / 32, t = threadIdx.x & 31;
    if (t < streams && blockIdx.x * (kHcThreads / 32) + warp < width)  // this warp's gate rows, before the previous kernel ends
        prefetch_l2(UpW.p + ((long long)t * width + blockIdx.x * (kHcThreads / 32) + warp) * rank, (unsigned long long)rank * 4);
    dep_enter();
    for (int k = threadIdx.x; k < rank; k += kHcThreads) hc_lo[k] = ref_silu(__fmul_rn(Down.p[k], scale));
    __syncthreads();
    const int d = blockIdx.x * (kHcThreads / 32) + warp;
    if (d >= width) return;
    float v = 0.0f;
    if (rank == 256 && streams <= 4) {
        float wv[4][8], nv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (c >= streams) break;
            const long long row = (long long)c * width + d;
            const float *wr = UpW.p + row * rank;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                wv[c][2 * k] = __ldg(wr + t + 64 * k);
                wv[c][2 * k + 1] = __ldg(wr + t + 32 + 64 * k);
            }
            nv[c] = __ldg(Norm.p + row);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (c >= streams) break;
            float lo = 0.0f, hi = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                lo = __fadd_rn(lo, __fmul_rn(wv[c][2 * k], hc_lo[t + 64 * k]));
                hi = __fadd_rn(hi, __fmul_rn(wv[c][2 * k + 1], hc_lo[t + 32 + 64 * k]));
            }
            const float gate = __shfl_sync(0xffffffffu, tree64(lo, hi), 0);
            v = __fadd_rn(v, __fmul_rn(nv[c], ref_sigmoid(gate)));
        }
    } else {
        for (int c = 0; c < streams; ++c) {
            const long long row = (long long)c * width + d;
            const float gate = __shfl_sync(0xffffffffu, lane_dot(UpW.p + row * rank, hc_lo, rank, t), 0);
            v = __fadd_rn(v, __fmul_rn(Norm.p[row], ref_sigmoid(gate)));
        }
    }
    if (t == 0) Mixed.p[d] = __fdiv_rn(v, (float)streams);
}

// ---------------------------------------------------------------- device-position entries
// No counterpart in the reference: the four token- or position-dependent dispatches of a decode
// step or prompt chunk with those values read from device memory instead of kernel arguments,
// so one captured CUDA graph replays every decode step (or every full prompt chunk).
// strata_attention_at takes its query tokens as the dispatch's z extent, like strata_attention_batch. Each computes exactly what its reference entry
// computes for the same value.

// strata_embed_token: for each of `tokens` ids in Token, that row of the table into every stream
// of the token's residual (token k at k * width * streams): strata_embedding format 0 per token.
__global__ void k_embed_token(Grid g, FB Table, IB Token, FB Residual, int width, int streams, int vocab, int tokens, unsigned *err) {
    dep_enter();
    long long i = lane_index(g, (long long)width * tokens);
    if (i < 0) return;
    const long long k = i / width, d = i % width;
    const int t = Token.get(k, err);
    if (t < 0 || t >= vocab) {
        raise_error(err, kErrIndex);
        return;
    }
    const float v = Table.get((long long)t * width + d, err);
    for (int stream = 0; stream < streams; ++stream) Residual.set((k * streams + stream) * width + d, v, err);
}

// ---------------------------------------------------------------- launchers
}  // namespace

bool engine_pdl() {
    static const bool on = [] {
        const char *v = std::getenv("STRATA_ENGINE_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

namespace {

constexpr int kOneToken = 1;  // the decode entries: one token
cudaError_t L_embedding(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_embedding, LANESL, grid_of(g), F(0), U(1), F(2), F(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i, a[12].i,
                            a[13].i, err);
    return cudaGetLastError();
}
cudaError_t L_embed(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_embed, LANESL, grid_of(g), F(0), F(1), a[2].i, a[3].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_embed_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_embed, LANESL, grid_of(g), F(0), F(1), a[2].i, a[3].i, a[4].i, err);
    return cudaGetLastError();
}
cudaError_t L_rope_frequencies(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_rope_frequencies, LANESL, grid_of(g), F(0), F(1), a[2].i, a[3].f, err);
    return cudaGetLastError();
}
cudaError_t L_rope_table(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_rope_table, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_rope_position(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_rope, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, a[6].i, a[7].i, a[8].i, 0, IB{nullptr, 0}, err);
    return cudaGetLastError();
}
cudaError_t L_rope(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_rope, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, a[6].i, 0, kOneToken, 1, IB{nullptr, 0}, err);
    return cudaGetLastError();
}
cudaError_t L_rope_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_rope, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, a[6].i, 0, a[7].i, 2, IB{nullptr, 0}, err);
    return cudaGetLastError();
}
cudaError_t L_embed_token(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(a[6].i == 1, k_embed_token, LANESL, grid_of(g), F(0), I(1), F(2), a[3].i, a[4].i, a[5].i, a[6].i, err);
    return cudaGetLastError();
}
cudaError_t L_rope_at(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(a[8].i == 1, k_rope, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[5].i, a[6].i, a[7].i, 0, a[8].i, 0, I(4), err);
    return cudaGetLastError();
}
cudaError_t L_kv_append_at(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(a[6].i == 1, k_kv_append, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[5].i, 0, a[6].i, I(4), 0, err);
    return cudaGetLastError();
}
cudaError_t L_attention_at(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_attention_prompt(a, 0, 1, 2, 4, a[5].i, a[6].i, a[7].i, 0, a[8].f, I(3), g, s, err);
}
cudaError_t L_hc_in(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int width = a[7].i, streams = a[8].i, rank = a[9].i;
    const size_t bytes = (size_t)width * streams * 12;  // residual, weight row and gammas staged
    if (streams < 1 || streams > 64 || bytes > 227 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_hc_in, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    launch_k(true, k_hc_in, (unsigned)(rank + streams), kHcInThreads, bytes, s, F(0), F(1), F(2), F(3), F(4), F(5), F(6), width, streams, rank, a[10].f);
    return cudaGetLastError();
}
cudaError_t L_hc_out(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int width = a[4].i, streams = a[5].i, rank = a[6].i;
    launch_k(true, k_hc_out, (unsigned)((width + kHcThreads / 32 - 1) / (kHcThreads / 32)), kHcThreads, (size_t)rank * 4, s, 
        F(0), F(1), F(2), F(3), width, streams, rank, a[7].f);
    return cudaGetLastError();
}
cudaError_t L_gemv(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_gemv, GROUPS, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_quant_gemv(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_quant_gemv, GROUPS, grid_of(g), F(0), U(1), F(2), F(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, a[9].i, a[10].i, a[11].i, err);
    return cudaGetLastError();
}
cudaError_t L_norm(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const long long cols = a[3].i, rows = std::min<long long>(a[4].i, g[0]), wrows = a[5].i;
    const int mode = a[6].i;
    const size_t bytes = (size_t)cols * (mode == 0 ? 8 : 4);
    if (cols >= 512 && bytes <= 200 * 1024 && rows > 0 && wrows > 0 && a[0].len >= rows * cols && a[2].len >= rows * cols &&
        (mode != 0 || a[1].len >= std::min(rows, wrows) * cols)) {
        cudaError_t e = cudaFuncSetAttribute(k_norm_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        launch_k(rows <= 64, k_norm_staged, (unsigned)rows, kNormThreads, bytes, s, F(0), F(1), F(2), a[3].i, a[5].i, mode, a[7].f, a[8].f);
        return cudaGetLastError();
    }
    launch_k(a[4].i <= 64, k_norm, GROUPS, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, a[6].i, a[7].f, a[8].f, err);
    return cudaGetLastError();
}
cudaError_t L_ple_gate(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_ple_gate, GROUPS, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, err);
    return cudaGetLastError();
}
cudaError_t L_argmax(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_argmax, 1, kArgmaxThreads, 0, s, F(0), I(1), a[2].i, err);
    return cudaGetLastError();
}
cudaError_t L_attention(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    if (attention_cl_ok(a[1], a[2], a[5].i, a[6].i, a[7].i, g)) {
        launch_k(true, k_attention_cl, dim3(g[0] * kAcCluster, 1), kAcThreads, 0, s, grid_of(g), F(0), F(1), F(2), I(3), F(4), a[5].i, a[6].i, a[7].i,
                                                                         a[8].i, 0, a[9].f, 0, IB{nullptr, 0}, 0, err);
        return cudaGetLastError();
    }
    launch_k(true, k_attention, dim3(g[0], 1), kAttnThreads, 0, s, grid_of(g), F(0), F(1), F(2), I(3), F(4), a[5].i, a[6].i, a[7].i, a[8].i, 0, a[9].f, 0,
                                                       IB{nullptr, 0}, 0, err);
    return cudaGetLastError();
}
cudaError_t L_attention_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_attention_prompt(a, 0, 1, 2, 3, a[4].i, a[5].i, a[6].i, a[7].i, a[8].f, IB{nullptr, 0}, g, s, err);
}
cudaError_t L_kv_append(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_kv_append, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, kOneToken, IB{nullptr, 0}, 0, err);
    return cudaGetLastError();
}
cudaError_t L_kv_append_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_kv_append, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[4].i, a[5].i, a[6].i, IB{nullptr, 0}, 0, err);
    return cudaGetLastError();
}
cudaError_t L_attention_gate(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_attention_gate, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_attention_gate_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_attention_gate, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_slice(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k((long long)a[2].i * a[3].i <= 16384, k_slice, LANESL, grid_of(g), F(0), F(1), a[2].i, a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_hc_mix(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_hc_mix, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_hc_mix_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_hc_mix, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_hc_write(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_hc_write, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_hc_write_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_hc_write, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_ple_broadcast(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_ple_broadcast, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_ple_broadcast_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_ple_broadcast, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, a[4].i, a[5].i, err);
    return cudaGetLastError();
}
cudaError_t L_ple_add(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_ple_add, LANESL, grid_of(g), F(0), F(1), F(2), a[3].i, err);
    return cudaGetLastError();
}
cudaError_t L_conv(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_conv(a, g, kOneToken, 0, s, err);
}
cudaError_t L_conv_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_conv(a, g, a[8].i, 1, s, err);
}
cudaError_t L_gdn_gates(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_gdn_gates, LANESL, grid_of(g), F(0), F(1), F(2), F(3), F(4), F(5), a[6].i, kOneToken, err);
    return cudaGetLastError();
}
cudaError_t L_gdn_gates_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(false, k_gdn_gates, LANESL, grid_of(g), F(0), F(1), F(2), F(3), F(4), F(5), a[6].i, a[7].i, err);
    return cudaGetLastError();
}
cudaError_t L_gdn_step(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_gdn(grid_of(g), a, kOneToken, s, err);
}
cudaError_t L_gdn_batch(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    return launch_gdn(grid_of(g), a, a[10].i, s, err);
}

// ---- sequence-batch entries (no reference counterpart): one decode token for each of `tokens`
// independent sequences, each with its own position, cache, history or state. Each value is formed
// by the same operations in the same order as the one-sequence entry it batches.
cudaError_t L_rope_seqs(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_rope, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[5].i, a[6].i, a[7].i, 0, a[8].i, 3, I(4), err);
    return cudaGetLastError();
}
cudaError_t L_kv_append_seqs(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_kv_append, LANESL, grid_of(g), F(0), F(1), F(2), F(3), a[5].i, 0, a[7].i, I(4), a[6].i, err);
    return cudaGetLastError();
}
cudaError_t L_attention_seqs(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int dim = a[5].i, heads = a[6].i, kvHeads = a[7].i, cells = a[8].i;
    const float scale = a[9].f;
    // the grouped-query form (each key and value row loaded once for the group's heads) when there
    // are enough sequences to fill the SMs with (KV head, sequence) blocks
    const int G = kvHeads > 0 ? heads / kvHeads : 0;
    const size_t bytes = ((size_t)G * dim + (size_t)G * kMaxCells) * 4;
    const bool aligned = (reinterpret_cast<uintptr_t>(a[1].ptr) & 15) == 0;
    if ((long long)g[2] * kvHeads >= 64 && G >= 1 && G <= kMaxGroup && heads % kvHeads == 0 && dim % 4 == 0 && aligned &&
        bytes <= 200 * 1024 && g[0] >= (unsigned)heads) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_group, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        launch_k(false, k_attention_group, dim3(kvHeads, g[2]), kGroupThreads, bytes, s, grid_of(g), F(0), F(1), F(2), F(4), dim, heads, kvHeads, 0,
                 scale, I(3), cells, err);
        return cudaGetLastError();
    }
    if (attention_cl_ok(a[1], a[2], dim, heads, kvHeads, g)) {
        launch_k(false, k_attention_cl, dim3(g[0] * kAcCluster, g[2]), kAcThreads, 0, s, grid_of(g), F(0), F(1), F(2), IB{nullptr, 0}, F(4), dim,
                 heads, kvHeads, 0, 0, scale, 1, I(3), cells, err);
        return cudaGetLastError();
    }
    launch_k(false, k_attention, dim3(g[0], g[2]), kAttnThreads, 0, s, grid_of(g), F(0), F(1), F(2), IB{nullptr, 0}, F(4), dim, heads, kvHeads, 0, 0,
             scale, 1, I(3), cells, err);
    return cudaGetLastError();
}
cudaError_t L_conv_seqs(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int channels = a[4].i, taps = a[5].i, dil = a[6].i, act = a[7].i, tokens = a[8].i;
    const long long n = (long long)channels * tokens;
    const bool covered = channels >= 1 && tokens >= 1 && (long long)g[0] * STRATA_LANES >= n && a[0].len >= n * (taps - 1) * dil &&
                         a[2].len >= (long long)channels * taps && a[1].len >= n && a[3].len >= n;
    if (covered && taps == 4 && dil == 1) {
        launch_k(true, k_conv_seqs_reg<4, 1>, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, act, tokens);
    } else if (covered && taps == 4 && dil == 3) {
        launch_k(true, k_conv_seqs_reg<4, 3>, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, act, tokens);
    } else {
        launch_k(true, k_conv_seqs, LANESL, grid_of(g), F(0), F(1), F(2), F(3), channels, taps, dil, act, tokens, err);
    }
    return cudaGetLastError();
}
cudaError_t L_gdn_seqs(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const int dim = a[7].i, kh = a[8].i, vh = a[9].i, tokens = a[10].i;
    const long long stride = (long long)vh * dim;
    const bool covered = kh >= 1 && vh >= 1 && tokens >= 1 && (long long)g[0] * STRATA_LANES >= stride * tokens &&
                         a[0].len >= (long long)tokens * dim * stride && a[1].len >= (long long)tokens * kh * dim &&
                         a[2].len >= (long long)tokens * kh * dim && a[3].len >= tokens * stride && a[4].len >= (long long)tokens * vh &&
                         a[5].len >= (long long)tokens * vh && a[6].len >= tokens * stride;
    if (dim == 128 && covered && tokens <= 65535) {
        launch_k(false, k_gdn_regs<128, true>, dim3((unsigned)((stride + 127) / 128), (unsigned)tokens), 128, 0, s, F(0), F(1), F(2), F(3), F(4),
                 F(5), F(6), kh, vh, tokens, stride);
    } else {
        launch_k(false, k_gdn_seqs, lane_blocks(g), 256, 0, s, grid_of(g), F(0), F(1), F(2), F(3), F(4), F(5), F(6), dim, kh, vh, tokens, err);
    }
    return cudaGetLastError();
}
cudaError_t L_gdn_gates_fused(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    const long long width = a[7].i, heads = a[8].i, tokens = a[9].i;
    if (width < 1 || heads < 1 || tokens < 1 || tokens > 65535 || a[0].len < tokens * width || a[1].len < heads * width ||
        a[2].len < heads * width || a[3].len < heads || a[4].len < heads || a[5].len < tokens * heads || a[6].len < tokens * heads)
        return cudaErrorInvalidValue;
    const size_t bytes = (size_t)width * 12;  // the two weight rows and the input row
    if (bytes > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k_gdn_gates_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    launch_k(tokens == 1, k_gdn_gates_fused, dim3((unsigned)heads, (unsigned)tokens), kGatesThreads, bytes, s, F(0), F(1), F(2), F(3), F(4),
             F(5), F(6), (int)width, (int)heads);
    return cudaGetLastError();
}
cudaError_t L_argmax_rows(const KArg *a, const unsigned g[3], cudaStream_t s, unsigned *err) {
    launch_k(true, k_argmax, (unsigned)a[3].i, kArgmaxThreads, 0, s, F(0), I(1), a[2].i, err);
    return cudaGetLastError();
}

}  // namespace

// Parameter lists in kernels/strata.cu order and spelling (kinds as in compat.cu's table).
const KernelSpec kEngineKernels[] = {
    {"strata_embedding",
     "Values:f Codes:u Scales:f Offsets:f Residual:f width:I streams:I outputOffset:I format:I bits:I groupSize:I bias:I codebook:I "
     "hasOffset:I",
     L_embedding},
    {"strata_embed", "Row:f Residual:f width:I streams:I", L_embed},
    {"strata_embed_batch", "Rows:f Residual:f width:I streams:I tokens:I", L_embed_batch},
    {"strata_rope_frequencies", "High:f Low:f rotary:I base:F", L_rope_frequencies},
    {"strata_rope_table", "High:f Low:f Cos:f Sin:f rotary:I context:I", L_rope_table},
    {"strata_rope_position", "X:f Cos:f Sin:f Y:f dim:I heads:I rotary:I position:I tokens:I", L_rope_position},
    {"strata_rope", "X:f Cos:f Sin:f Y:f dim:I heads:I rotary:I", L_rope},
    {"strata_rope_batch", "X:f Cos:f Sin:f Y:f dim:I heads:I rotary:I tokens:I", L_rope_batch},
    {"strata_gemv", "X:f W:f Y:f cols:I rows:I tokens:I", L_gemv},
    {"strata_quant_gemv", "X:f Codes:u Scales:f Offsets:f Y:f cols:I rows:I bits:I groupSize:I bias:I codebook:I hasOffset:I",
     L_quant_gemv},
    {"strata_norm", "X:f W:f Y:f cols:I rows:I weightRows:I mode:I epsilon:F scale:F", L_norm},
    {"strata_ple_gate", "Key:f Query:f Gate:f width:I streams:I", L_ple_gate},
    {"strata_argmax", "Logits:f Token:i count:I", L_argmax},
    {"strata_attention", "Q:f Keys:f Values:f Cells:i Y:f dim:I heads:I kvHeads:I count:I scale:F", L_attention},
    {"strata_attention_batch", "Q:f Keys:f Values:f Y:f dim:I heads:I kvHeads:I position:I scale:F", L_attention_batch},
    {"strata_kv_append", "K:f V:f Keys:f Values:f width:I position:I", L_kv_append},
    {"strata_kv_append_batch", "K:f V:f Keys:f Values:f width:I position:I tokens:I", L_kv_append_batch},
    {"strata_attention_gate", "Attention:f FullQ:f Y:f dim:I heads:I", L_attention_gate},
    {"strata_attention_gate_batch", "Attention:f FullQ:f Y:f dim:I heads:I tokens:I", L_attention_gate_batch},
    {"strata_slice", "X:f Y:f width:I rows:I stride:I offset:I", L_slice},
    {"strata_hc_mix", "Norm:f Gate:f Mixed:f width:I streams:I", L_hc_mix},
    {"strata_hc_mix_batch", "Norm:f Gate:f Mixed:f width:I streams:I tokens:I", L_hc_mix_batch},
    {"strata_hc_write", "Residual:f Output:f Inject:f width:I streams:I", L_hc_write},
    {"strata_hc_write_batch", "Residual:f Output:f Inject:f width:I streams:I tokens:I", L_hc_write_batch},
    {"strata_ple_broadcast", "Value:f Gate:f Y:f width:I streams:I", L_ple_broadcast},
    {"strata_ple_broadcast_batch", "Value:f Gate:f Y:f width:I streams:I tokens:I", L_ple_broadcast_batch},
    {"strata_ple_add", "Residual:f Gated:f Conv:f n:I", L_ple_add},
    {"strata_conv", "History:f X:f W:f Y:f channels:I taps:I dilation:I activation:I", L_conv},
    {"strata_conv_batch", "History:f X:f W:f Y:f channels:I taps:I dilation:I activation:I tokens:I", L_conv_batch},
    {"strata_gdn_gates", "Alpha:f Beta:f A:f Dt:f Decay:f Strength:f heads:I", L_gdn_gates},
    {"strata_gdn_gates_batch", "Alpha:f Beta:f A:f Dt:f Decay:f Strength:f heads:I tokens:I", L_gdn_gates_batch},
    {"strata_gdn_step", "State:f Q:f K:f V:f Decay:f Beta:f Y:f dim:I keyHeads:I valueHeads:I", L_gdn_step},
    {"strata_gdn_batch", "State:f Q:f K:f V:f Decay:f Beta:f Y:f dim:I keyHeads:I valueHeads:I tokens:I", L_gdn_batch},
    // device-position entries (no reference counterpart)
    {"strata_embed_token", "Table:f Token:i Residual:f width:I streams:I vocab:I tokens:I", L_embed_token},
    {"strata_rope_at", "X:f Cos:f Sin:f Y:f Position:i dim:I heads:I rotary:I tokens:I", L_rope_at},
    {"strata_kv_append_at", "K:f V:f Keys:f Values:f Position:i width:I tokens:I", L_kv_append_at},
    {"strata_attention_at", "Q:f Keys:f Values:f Position:i Y:f dim:I heads:I kvHeads:I scale:F", L_attention_at},
    // hyper-connection blocks (no reference counterpart)
    {"strata_hc_in", "Residual:f NormW:f DownW:f InjectW:f Norm:f Down:f Inject:f width:I streams:I rank:I epsilon:F", L_hc_in},
    {"strata_hc_out", "Norm:f Down:f UpW:f Mixed:f width:I streams:I rank:I scale:F", L_hc_out},
    {"strata_gdn_prep", "History:f X:f W:f Q:f K:f V:f keyDim:I valueDim:I headDim:I qScale:F epsilon:F", L_gdn_prep},
    // sequence-batch decode entries (no reference counterpart)
    {"strata_rope_seqs", "X:f Cos:f Sin:f Y:f Positions:i dim:I heads:I rotary:I tokens:I", L_rope_seqs},
    {"strata_kv_append_seqs", "K:f V:f Keys:f Values:f Positions:i width:I cells:I tokens:I", L_kv_append_seqs},
    {"strata_attention_seqs", "Q:f Keys:f Values:f Positions:i Y:f dim:I heads:I kvHeads:I cells:I scale:F", L_attention_seqs},
    {"strata_conv_seqs", "History:f X:f W:f Y:f channels:I taps:I dilation:I activation:I tokens:I", L_conv_seqs},
    {"strata_gdn_seqs", "State:f Q:f K:f V:f Decay:f Beta:f Y:f dim:I keyHeads:I valueHeads:I tokens:I", L_gdn_seqs},
    {"strata_argmax_rows", "Logits:f Tokens:i count:I rows:I", L_argmax_rows},
    // the delta-rule gate inputs in one launch (no reference counterpart)
    {"strata_gdn_gates_fused", "X:f AlphaW:f BetaW:f A:f Dt:f Decay:f Strength:f width:I heads:I tokens:I", L_gdn_gates_fused},
};
const int kNumEngineKernels = sizeof(kEngineKernels) / sizeof(kEngineKernels[0]);

}  // namespace strata
