/*
 * TEST INFRASTRUCTURE (oracle). A CPU restatement of the reference's mixture-of-experts
 * kernels, used only by tests/, bench.py's cpu_baseline / --impl reference legs and
 * __graft_entry__.smoke() as the checker. The product never links or calls it.
 *
 * Every entry keeps the reference's workgroup semantics (kernels/strata.cu:3: 64 lanes per
 * workgroup, lane-strided F32 accumulation, then a shared-memory tree s = 32..1) and its
 * dispatch convention: a grid (gx, gy, gz) of workgroups followed by the kernel's own
 * parameters, exactly as vendor/webcuda/src/wasm/compile.mjs:39 wraps each entry as
 * cw_<entry>(gx, gy, gz, params...). Arithmetic is F32 with no contraction (build with
 * -ffp-contract=off), so results are bit-identical to the reference's CPU path whenever
 * the same expf is used (strata_expf.h).
 *
 * Return value: 0, like cw_parallel (thread-pool.hpp:61) when no barrier diverged.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#include "strata_expf.h"

#define LANES 64

/* kernels/strata.cu:7-8 */
static inline float o_sigmoid(float x) { return 1.0f / (1.0f + strata_oracle_expf(-x)); }
static inline float o_silu(float x) { return x * o_sigmoid(x); }

/* kernels/strata.cu:9-12 */
static inline int o_group(int index, int size) {
    if (size == 16) return index >> 4;
    if (size == 32) return index >> 5;
    if (size == 64) return index >> 6;
    return index / size;
}

/* kernels/strata.cu:13-18 — FP16 bits to float, subnormals by a multiply with 2^-24. */
float oracle_half_bits(unsigned int h) {
    unsigned int sign = (h & 32768u) << 16;
    unsigned int exponent = (h >> 10) & 31u;
    unsigned int fraction = h & 1023u;
    if (exponent == 0u) {
        if (fraction == 0u) return strata_o_u2f(sign);
        float v = (float)fraction * 0.000000059604644775390625f;
        return sign != 0u ? -v : v;
    }
    if (exponent == 31u) return strata_o_u2f(sign | 2139095040u | (fraction << 13));
    return strata_o_u2f(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

/* kernels/strata.cu:22-31 */
static float o_iq4(int c) {
    static const float t[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
    return (c >= 0 && c < 15) ? t[c] : 113.0f;
}

float oracle_expf(float x) { return strata_oracle_expf(x); }

/* The reference's reduction: partial[lane] += partial[lane + s] for s = 32..1. */
static float tree_sum(float *p) {
    for (int s = 32; s > 0; s >>= 1)
        for (int l = 0; l < s; ++l) p[l] += p[l + s];
    return p[0];
}

static inline float half_at(const unsigned int *words, int halfIndex) {
    return oracle_half_bits((words[halfIndex / 2] >> ((halfIndex % 2) * 16)) & 65535u);
}
static inline int code_at(const unsigned int *words, int codeOffset, int index) {
    return (int)((words[codeOffset + index / 16] >> ((index % 16) * 2)) & 3u) - 1;
}

/* kernels/strata.cu:19-21 */
int oracle_strata_unpack_half(unsigned gx, unsigned gy, unsigned gz, const unsigned int *Packed, float *Values, int count) {
    (void)gy; (void)gz; /* blockIdx.y/z do not enter i: extra workgroups rewrite the same values */
    for (long i = 0; i < (long)gx * LANES && i < count; ++i) Values[i] = half_at(Packed, (int)i);
    return 0;
}

/* kernels/strata.cu:81-87 — IQ4_NL rows of 32 values in 18 bytes: an FP16 scale, then 16 bytes
   of codes (value i of the block: low nibble of byte i for i < 16, high nibble of byte i - 16). */
int oracle_strata_ple_decode(unsigned gx, unsigned gy, unsigned gz, const unsigned int *Packed, float *Values, int count) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < count; ++i) {
        int block = (int)(i / 32), scale_byte = block * 18, code_byte = scale_byte + 2 + (int)(i % 16);
        unsigned int half = (Packed[scale_byte / 4] >> ((scale_byte % 4) * 8)) & 65535u;
        int code = (int)((Packed[code_byte / 4] >> ((code_byte % 4) * 8 + (i % 32 < 16 ? 0 : 4))) & 15u);
        Values[i] = oracle_half_bits(half) * o_iq4(code);
    }
    return 0;
}

/* kernels/strata.cu:35-37 */
int oracle_strata_expert_scales(unsigned gx, unsigned gy, unsigned gz, const unsigned int *Blob, float *Scales, int offset, int count) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES; ++i)
        if (i < count) { int at = offset + (int)i; Scales[i] = half_at(Blob, at); }
    return 0;
}

/* kernels/strata.cu:38-55 — fused gate/up/SiLU over interleaved rows 2r (gate), 2r+1 (up). */
int oracle_strata_q2_gate_up(unsigned gx, unsigned gy, unsigned gz, const float *X, const unsigned int *Blob, const float *Scales,
                             const int *Mapping, float *Hidden, int width, int ff, int tokens, int mapped, int expanded,
                             int codeOffset, int scaleOffset) {
    (void)gz;
    float gate[LANES], up[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < ff && (int)token < tokens)) continue;
            int inputRow = mapped != 0 ? Mapping[2 * token] : (int)token;
            for (int lane = 0; lane < LANES; ++lane) {
                float g = 0.0f, u = 0.0f;
                for (int i = lane; i < width; i += LANES) {
                    int gi = (int)row * 2 * width + i, ui = gi + width;
                    int gc = code_at(Blob, codeOffset, gi), uc = code_at(Blob, codeOffset, ui);
                    int gs = scaleOffset + gi / 64, us = scaleOffset + ui / 64;
                    float gw = (float)gc * (expanded != 0 ? Scales[gs] : half_at(Blob, gs));
                    float uw = (float)uc * (expanded != 0 ? Scales[us] : half_at(Blob, us));
                    float x = X[inputRow * width + i];
                    g += gw * x; u += uw * x;
                }
                gate[lane] = g; up[lane] = u;
            }
            for (int s = 32; s > 0; s >>= 1)
                for (int l = 0; l < s; ++l) { gate[l] += gate[l + s]; up[l] += up[l + s]; }
            Hidden[token * ff + row] = o_silu(gate[0]) * up[0];
        }
    return 0;
}

/* kernels/strata.cu:56-69 — down projection scattered to Y[outputOffset + Mapping[2t+1]*width + row]. */
int oracle_strata_q2_down(unsigned gx, unsigned gy, unsigned gz, const float *Hidden, const unsigned int *Blob, const float *Scales,
                          const int *Mapping, float *Y, int width, int ff, int tokens, int mapped, int expanded, int outputOffset,
                          int codeOffset, int scaleOffset) {
    (void)gz;
    float partial[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < width && (int)token < tokens)) continue;
            for (int lane = 0; lane < LANES; ++lane) {
                float sum = 0.0f;
                for (int i = lane; i < ff; i += LANES) {
                    int index = (int)row * ff + i;
                    int code = code_at(Blob, codeOffset, index);
                    int si = scaleOffset + index / 64;
                    float w = (float)code * (expanded != 0 ? Scales[si] : half_at(Blob, si));
                    sum += w * Hidden[token * ff + i];
                }
                partial[lane] = sum;
            }
            float r = tree_sum(partial);
            int destination = mapped != 0 ? Mapping[2 * token + 1] : (int)token;
            Y[outputOffset + destination * width + row] = r;
        }
    return 0;
}

/* kernels/strata.cu:156-165 — F32 projection (router logits, shared-expert gate logit). */
int oracle_strata_project(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *W, float *Y, int cols, int rows,
                          int tokens, int outputStride, int outputOffset) {
    (void)gz;
    float partial[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < rows && (int)token < tokens)) continue;
            for (int lane = 0; lane < LANES; ++lane) {
                float sum = 0.0f;
                for (int i = lane; i < cols; i += LANES) sum += W[(long)row * cols + i] * X[(long)token * cols + i];
                partial[lane] = sum;
            }
            Y[(long)token * outputStride + outputOffset + row] = tree_sum(partial);
        }
    return 0;
}

/* kernels/strata.cu:168-176 — BF16 weight words, F32 math. */
int oracle_strata_bf16_project(unsigned gx, unsigned gy, unsigned gz, const float *X, const unsigned int *Codes, float *Y, int cols,
                               int rows, int tokens, int outputStride, int outputOffset) {
    (void)gz;
    float partial[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < rows && (int)token < tokens)) continue;
            for (int lane = 0; lane < LANES; ++lane) {
                float sum = 0.0f;
                for (int i = lane; i < cols; i += LANES) {
                    int ix = (int)row * cols + i;
                    unsigned int bits = (Codes[ix / 2] >> ((ix % 2) * 16)) & 65535u;
                    sum += strata_o_u2f(bits << 16) * X[token * cols + i];
                }
                partial[lane] = sum;
            }
            Y[token * outputStride + outputOffset + row] = tree_sum(partial);
        }
    return 0;
}

/* kernels/strata.cu:179-192 — one role of a resident Q2 blob (weightRow, rowStride 1 or 2). */
int oracle_strata_q2_project(unsigned gx, unsigned gy, unsigned gz, const float *X, const unsigned int *Blob, float *Y, int cols, int rows,
                             int tokens, int outputStride, int outputOffset, int codeOffset, int scaleOffset, int weightRow,
                             int rowStride) {
    (void)gz;
    float partial[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < rows && (int)token < tokens)) continue;
            for (int lane = 0; lane < LANES; ++lane) {
                float sum = 0.0f;
                for (int i = lane; i < cols; i += LANES) {
                    int ix = (weightRow + (int)row * rowStride) * cols + i;
                    int code = code_at(Blob, codeOffset, ix);
                    int si = scaleOffset + ix / 64;
                    float weight = (float)code * half_at(Blob, si);
                    sum += weight * X[token * cols + i];
                }
                partial[lane] = sum;
            }
            Y[token * outputStride + outputOffset + row] = tree_sum(partial);
        }
    return 0;
}

/* kernels/strata.cu:193-211 — generic S2/S4/S8 projection; the WASM expert path (bits 2, group 64, bias -1). */
int oracle_strata_quant_project(unsigned gx, unsigned gy, unsigned gz, const float *X, const unsigned int *Codes, const float *Scales,
                                const float *Offsets, float *Y, int cols, int rows, int tokens, int outputStride, int outputOffset,
                                int bits, int groupSize, int bias, int codebook, int hasOffset) {
    (void)gz;
    float partial[LANES];
    for (unsigned token = 0; token < gy; ++token)
        for (unsigned row = 0; row < gx; ++row) {
            if (!((int)row < rows && (int)token < tokens)) continue;
            for (int lane = 0; lane < LANES; ++lane) {
                float sum = 0.0f;
                for (int i = lane; i < cols; i += LANES) {
                    int index = (int)row * cols + i, bit = index * bits;
                    int code = (int)((Codes[bit / 32] >> (bit % 32)) & ((1u << bits) - 1u));
                    float value = codebook == 1 ? o_iq4(code) : (float)(code + bias);
                    int group = o_group(index, groupSize);
                    float weight = value * Scales[group];
                    if (hasOffset != 0) weight += Offsets[group];
                    sum += weight * X[token * cols + i];
                }
                partial[lane] = sum;
            }
            Y[token * outputStride + outputOffset + row] = tree_sum(partial);
        }
    return 0;
}

/* kernels/strata.cu:229-236 — 0 copy/scale; 1 SiLU; 2 sigmoid; 3 SiLU(A)*B; 4 A*sigmoid(B); 5 add. */
int oracle_strata_elementwise(unsigned gx, unsigned gy, unsigned gz, const float *A, const float *B, float *Y, int n, int mode, float scale) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < n; ++i) {
        float a = A[i] * scale, v = a;
        if (mode == 1) v = o_silu(a);
        if (mode == 2) v = o_sigmoid(a);
        if (mode == 3) v = o_silu(a) * B[i];
        if (mode == 4) v = a * o_sigmoid(B[i]);
        if (mode == 5) v = a + B[i];
        Y[i] = v;
    }
    return 0;
}

/* kernels/strata.cu:238-270 (router) and :478-509 (router_batch): softmax over all experts,
 * k rounds of lane-strided argmax with lower-ID tie-break, weights sel/max(sum, 2^-14). */
static void router_token(const float *Logits, int *Ids, float *Weights, int experts, int topK) {
    float prob[512], reduce[LANES], selected[32];
    int winner[LANES];
    for (int lane = 0; lane < LANES; ++lane) {
        float mx = -3.402823e38f;
        for (int e = lane; e < experts; e += LANES) mx = fmaxf(mx, Logits[e]);
        reduce[lane] = mx;
    }
    for (int s = 32; s > 0; s >>= 1)
        for (int l = 0; l < s; ++l) reduce[l] = fmaxf(reduce[l], reduce[l + s]);
    float mx = reduce[0];
    for (int lane = 0; lane < LANES; ++lane) {
        float sum = 0.0f;
        for (int e = lane; e < experts; e += LANES) { prob[e] = strata_oracle_expf(Logits[e] - mx); sum += prob[e]; }
        reduce[lane] = sum;
    }
    float inv = 1.0f / tree_sum(reduce);
    for (int e = 0; e < experts; ++e) prob[e] *= inv;
    for (int k = 0; k < topK; ++k) {
        for (int lane = 0; lane < LANES; ++lane) {
            float best = -1.0f; int id = experts;
            for (int e = lane; e < experts; e += LANES)
                if (prob[e] > best || (prob[e] == best && e < id)) { best = prob[e]; id = e; }
            reduce[lane] = best; winner[lane] = id;
        }
        for (int s = 32; s > 0; s >>= 1)
            for (int l = 0; l < s; ++l) {
                float v = reduce[l + s]; int j = winner[l + s];
                if (v > reduce[l] || (v == reduce[l] && j < winner[l])) { reduce[l] = v; winner[l] = j; }
            }
        Ids[k] = winner[0]; selected[k] = reduce[0]; prob[winner[0]] = -1.0f;
    }
    float denom = 0.0f;
    for (int k = 0; k < topK; ++k) denom += selected[k];
    denom = fmaxf(denom, 0.00006103515625f);
    for (int k = 0; k < topK; ++k) Weights[k] = selected[k] / denom;
}

int oracle_strata_router(unsigned gx, unsigned gy, unsigned gz, const float *Logits, int *Ids, float *Weights, int experts, int topK) {
    (void)gx; (void)gy; (void)gz;
    router_token(Logits, Ids, Weights, experts, topK);
    return 0;
}

int oracle_strata_router_batch(unsigned gx, unsigned gy, unsigned gz, const float *Logits, int *Ids, float *Weights, int experts, int topK) {
    (void)gy; (void)gz;
    for (unsigned t = 0; t < gx; ++t)
        router_token(Logits + (long)t * experts, Ids + (long)t * topK, Weights + (long)t * topK, experts, topK);
    return 0;
}

/* kernels/strata.cu:360-365 — y = shared*sigmoid(sg) + sum_k parts[k]*w[k], in this order. */
int oracle_strata_moe_combine(unsigned gx, unsigned gy, unsigned gz, const float *Parts, const float *Weights, const float *Shared,
                              const float *SharedGate, float *Y, int width, int count) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < width; ++i) {
        float value = Shared[i] * o_sigmoid(SharedGate[0]);
        for (int k = 0; k < count; ++k) value += Parts[k * width + i] * Weights[k];
        Y[i] = value;
    }
    return 0;
}

/* kernels/strata.cu:470-476 */
int oracle_strata_moe_combine_batch(unsigned gx, unsigned gy, unsigned gz, const float *Parts, const float *Weights, const float *Shared,
                                    const float *SharedGate, float *Y, int width, int count, int tokens) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < (long)width * tokens; ++i) {
        int token = (int)(i / width), d = (int)(i % width);
        float value = Shared[i] * o_sigmoid(SharedGate[token]);
        for (int k = 0; k < count; ++k) value += Parts[(long)(token * count + k) * width + d] * Weights[token * count + k];
        Y[i] = value;
    }
    return 0;
}

/* kernels/strata.cu:464-469 */
int oracle_strata_gather_rows(unsigned gx, unsigned gy, unsigned gz, const float *X, const int *Indices, float *Y, int width, int rows) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < (long)width * rows; ++i) Y[i] = X[(long)Indices[i / width] * width + i % width];
    return 0;
}
int oracle_strata_scatter_rows(unsigned gx, unsigned gy, unsigned gz, const float *X, const int *Indices, float *Y, int width, int rows) {
    (void)gy; (void)gz;
    for (long i = 0; i < (long)gx * LANES && i < (long)width * rows; ++i) Y[(long)Indices[i / width] * width + i % width] = X[i];
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * One MoE layer for one token, in the order of src/engine.js:133-156 on the WASM backend:
 *   logits = mat(ffn_gate_inp, x)                     (strata_project, src/ops.js:105)
 *   [logits += bias]                                  (strata_elementwise mode 5; synthetic Zipf offset)
 *   ids, w = strata_router(logits)                    (src/engine.js:136)
 *   for k: gate = mat(expert.gate, x); up = mat(expert.up, x)   (strata_quant_project with scales
 *          act = elementwise(gate, up, 3); down = mat(expert.down, act)   expanded by strata_expert_scales,
 *          parts[k] = down                            src/engine.js:129-131,148; src/ops.js:32-35,108)
 *   shared = expert(shared); sg = mat(ffn_gate_inp_shexp, x)    (src/engine.js:154)
 *   y = strata_moe_combine(parts, w, shared, sg)      (src/engine.js:155)
 * The quant projection with pre-expanded scales computes the same floats, in the same order, as
 * the fused strata_q2_gate_up/strata_q2_down entries, so this routine uses the Q2 blob directly.
 * Blob layout (vendor/strata/tools/pack_layer.py:54-65): gate/up codes (rows interleaved
 * g0,u0,g1,...), down codes, gate/up FP16 scales, down FP16 scales.
 * ------------------------------------------------------------------------------------- */
static void expert_token(const float *x, const unsigned int *blob, int width, int ff, float *hidden, float *out) {
    const int gu_codes = 0, d_codes = 2 * ff * width / 16, gu_scales = 2 * (3 * ff * width / 16), d_scales = gu_scales + 2 * ff * width / 64;
    (void)gu_codes;
    oracle_strata_q2_gate_up((unsigned)ff, 1, 1, x, blob, NULL, NULL, hidden, width, ff, 1, 0, 0, 0, gu_scales);
    oracle_strata_q2_down((unsigned)width, 1, 1, hidden, blob, NULL, NULL, out, width, ff, 1, 0, 0, 0, d_codes, d_scales);
}

/* x: [width]; router: [experts x width]; sharedGate: [width]; blobs: experts blobs of blobWords words;
 * bias: optional [experts] logit offsets. Writes y [width], ids/weights [topK]. */
int oracle_moe_token(const float *x, const float *router, const float *bias, const float *sharedGate, const unsigned int *blobs,
                     const unsigned int *sharedBlob, long blobWords, int width, int ff, int experts, int topK, float *y, int *ids,
                     float *weights) {
    float *logits = (float *)malloc(sizeof(float) * experts);
    float *parts = (float *)malloc(sizeof(float) * (size_t)width * topK);
    float *shared = (float *)malloc(sizeof(float) * width);
    float *hidden = (float *)malloc(sizeof(float) * ff);
    float sg;
    if (!logits || !parts || !shared || !hidden) { free(logits); free(parts); free(shared); free(hidden); return 1; }
    oracle_strata_project((unsigned)experts, 1, 1, x, router, logits, width, experts, 1, experts, 0);
    if (bias) oracle_strata_elementwise((unsigned)((experts + 63) / 64), 1, 1, logits, bias, logits, experts, 5, 1.0f);
    router_token(logits, ids, weights, experts, topK);
    for (int k = 0; k < topK; ++k) expert_token(x, blobs + (long)ids[k] * blobWords, width, ff, hidden, parts + (long)k * width);
    expert_token(x, sharedBlob, width, ff, hidden, shared);
    oracle_strata_project(1, 1, 1, x, sharedGate, &sg, width, 1, 1, 1, 0);
    oracle_strata_moe_combine((unsigned)((width + 63) / 64), 1, 1, parts, weights, shared, &sg, y, width, topK);
    free(logits); free(parts); free(shared); free(hidden);
    return 0;
}

/* Router logits only (for the routing-exactness checks at full batch sizes). */
int oracle_route_token(const float *x, const float *router, const float *bias, int width, int experts, int topK, float *logits, int *ids,
                       float *weights) {
    oracle_strata_project((unsigned)experts, 1, 1, x, router, logits, width, experts, 1, experts, 0);
    if (bias) oracle_strata_elementwise((unsigned)((experts + 63) / 64), 1, 1, logits, bias, logits, experts, 5, 1.0f);
    router_token(logits, ids, weights, experts, topK);
    return 0;
}

/* ======================================================================================
 * The rest of the reference's entries (kernels/strata.cu:72-534): embeddings, RoPE, norms,
 * hyper-connections, gated delta-net, convolution, attention, PLE gating, argmax.
 *
 * Element entries compute lane i = 0 .. min(gx * 64, n) - 1 once: further workgroups along y
 * and z repeat the same lanes in the reference, which for the in-place entries would race.
 * logf, sqrtf, cosf and sinf are the host C library's (the reference's CPU build links its
 * own C library's, so those agree to within an ulp, not bit for bit); expf is the reference's.
 * ====================================================================================== */

static long lane_count(unsigned gx, long n) {
    long lanes = (long)gx * LANES;
    return lanes < n ? lanes : n;
}

/* 64 lane partials over a strided range, then the tree. */
static float lane_dot(const float *a, const float *b, long n) {
    float p[LANES];
    for (int l = 0; l < LANES; ++l) {
        float s = 0.0f;
        for (long i = l; i < n; i += LANES) s += a[i] * b[i];
        p[l] = s;
    }
    return tree_sum(p);
}

/* kernels/strata.cu:72-80 */
int oracle_strata_embedding(unsigned gx, unsigned gy, unsigned gz, const float *Values, const unsigned int *Codes, const float *Scales,
                            const float *Offsets, float *Residual, int width, int streams, int outputOffset, int format, int bits,
                            int groupSize, int bias, int codebook, int hasOffset) {
    (void)gy; (void)gz;
    long n = lane_count(gx, width);
    for (long i = 0; i < n; ++i) {
        float v;
        if (format == 0) v = Values[i];
        else if (format == 1) v = strata_o_u2f(((Codes[i / 2] >> ((i % 2) * 16)) & 65535u) << 16);
        else {
            long bit = i * bits;
            int code = (int)((Codes[bit / 32] >> (bit % 32)) & ((1u << bits) - 1u));
            int g = o_group((int)i, groupSize);
            v = (codebook == 1 ? o_iq4(code) : (float)(code + bias)) * Scales[g];
            if (hasOffset) v += Offsets[g];
        }
        for (int s = 0; s < streams; ++s) Residual[outputOffset + (long)s * width + i] = v;
    }
    return 0;
}

static void embed_rows(unsigned gx, const float *Rows, float *Residual, int width, int streams, int tokens) {
    long hc = (long)width * streams, n = lane_count(gx, hc * tokens);
    for (long i = 0; i < n; ++i) Residual[i] = Rows[(i / hc) * width + i % width];
}
/* kernels/strata.cu:282-285 */
int oracle_strata_embed(unsigned gx, unsigned gy, unsigned gz, const float *Row, float *Residual, int width, int streams) {
    (void)gy; (void)gz;
    embed_rows(gx, Row, Residual, width, streams, 1);
    return 0;
}
/* kernels/strata.cu:399-402 */
int oracle_strata_embed_batch(unsigned gx, unsigned gy, unsigned gz, const float *Rows, float *Residual, int width, int streams, int tokens) {
    (void)gy; (void)gz;
    embed_rows(gx, Rows, Residual, width, streams, tokens);
    return 0;
}

/* kernels/strata.cu:90-104: ln(base) by halving into [1, 2) and the atanh series, then
 * exp(power) by whole ln2 steps and a Taylor series of the remainder; double precision. */
int oracle_strata_rope_frequencies(unsigned gx, unsigned gy, unsigned gz, float *High, float *Low, int rotary, float base) {
    (void)gy; (void)gz;
    const double ln2 = 0.693147180559945309417232121458176568;
    long n = lane_count(gx, rotary / 2);
    for (long i = 0; i < n; ++i) {
        double m = (double)base;
        int e = 0;
        while (m >= 2.0) { m = m * 0.5; ++e; }
        double y = (m - 1.0) / (m + 1.0), y2term = y, ln = 0.0;
        for (int k = 1; k <= 49; k += 2) { ln += y2term / (double)k; y2term = y2term * y * y; }
        ln = 2.0 * ln + (double)e * ln2;
        double power = -ln * (double)(2 * i) / (double)rotary;
        int whole = (int)(float)(power / ln2);
        double r = power - (double)whole * ln2, sum = 1.0, term = 1.0;
        for (int k = 1; k <= 20; ++k) { term = term * r / (double)k; sum += term; }
        for (; whole < 0; ++whole) sum = sum * 0.5;
        High[i] = (float)sum;
        Low[i] = (float)(sum - (double)High[i]);
    }
    return 0;
}

/* kernels/strata.cu:105-111 */
int oracle_strata_rope_table(unsigned gx, unsigned gy, unsigned gz, const float *High, const float *Low, float *Cos, float *Sin, int rotary,
                             int context) {
    (void)gy; (void)gz;
    const double turn = 6.283185307179586476925286766559005768;
    int half = rotary / 2;
    long n = lane_count(gx, (long)context * half);
    for (long i = 0; i < n; ++i) {
        int pair = (int)(i % half);
        double angle = (double)(i / half) * ((double)High[pair] + (double)Low[pair]);
        int wraps = (int)(float)(angle / turn + 0.5);
        float reduced = (float)(angle - (double)wraps * turn);
        Cos[i] = cosf(reduced);
        Sin[i] = sinf(reduced);
    }
    return 0;
}

/* The NeoX half-split rotation shared by kernels/strata.cu:113-120, :319-327, :445-452;
 * table row of token t: rows_at + t * step (step 0: one row for all). */
static void rope_rows(unsigned gx, const float *X, const float *Cos, const float *Sin, float *Y, int dim, int heads, int rotary, int tokens,
                      long rows_at, long step) {
    int half = rotary / 2;
    long n = lane_count(gx, (long)dim * heads * tokens);
    for (long i = 0; i < n; ++i) {
        long d = i % dim;
        if (d >= rotary) { Y[i] = X[i]; continue; }
        long pair = d % half, row = i - d, t = i / ((long)dim * heads), at = (rows_at + t * step) * half + pair;
        float a = X[row + pair], b = X[row + pair + half];
        Y[i] = d < half ? a * Cos[at] - b * Sin[at] : b * Cos[at] + a * Sin[at];
    }
}
int oracle_strata_rope_position(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *Cos, const float *Sin, float *Y, int dim,
                                int heads, int rotary, int position, int tokens) {
    (void)gy; (void)gz;
    rope_rows(gx, X, Cos, Sin, Y, dim, heads, rotary, tokens, position, 1);
    return 0;
}
int oracle_strata_rope(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *Cos, const float *Sin, float *Y, int dim, int heads,
                       int rotary) {
    (void)gy; (void)gz;
    rope_rows(gx, X, Cos, Sin, Y, dim, heads, rotary, 1, 0, 0);
    return 0;
}
int oracle_strata_rope_batch(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *Cos, const float *Sin, float *Y, int dim,
                             int heads, int rotary, int tokens) {
    (void)gy; (void)gz;
    rope_rows(gx, X, Cos, Sin, Y, dim, heads, rotary, tokens, 0, 1);
    return 0;
}

/* kernels/strata.cu:121-131 */
int oracle_strata_gemv(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *W, float *Y, int cols, int rows, int tokens) {
    (void)gz;
    for (unsigned t = 0; t < gy && (int)t < tokens; ++t)
        for (unsigned r = 0; r < gx && (int)r < rows; ++r) Y[(long)t * rows + r] = lane_dot(W + (long)r * cols, X + (long)t * cols, cols);
    return 0;
}

/* kernels/strata.cu:134-153 */
int oracle_strata_quant_gemv(unsigned gx, unsigned gy, unsigned gz, const float *X, const unsigned int *Codes, const float *Scales,
                             const float *Offsets, float *Y, int cols, int rows, int bits, int groupSize, int bias, int codebook,
                             int hasOffset) {
    (void)gy; (void)gz;
    for (unsigned r = 0; r < gx && (int)r < rows; ++r) {
        float p[LANES];
        for (int l = 0; l < LANES; ++l) {
            float s = 0.0f;
            for (int i = l; i < cols; i += LANES) {
                int index = (int)r * cols + i, bit = index * bits;
                int code = (int)((Codes[bit / 32] >> (bit % 32)) & ((1u << bits) - 1u));
                int g = o_group(index, groupSize);
                float w = (codebook == 1 ? o_iq4(code) : (float)(code + bias)) * Scales[g];
                if (hasOffset) w += Offsets[g];
                s += w * X[i];
            }
            p[l] = s;
        }
        Y[r] = tree_sum(p);
    }
    return 0;
}

/* kernels/strata.cu:214-227 */
int oracle_strata_norm(unsigned gx, unsigned gy, unsigned gz, const float *X, const float *W, float *Y, int cols, int rows, int weightRows,
                       int mode, float epsilon, float scale) {
    (void)gy; (void)gz;
    for (unsigned r = 0; r < gx && (int)r < rows; ++r) {
        const float *x = X + (long)r * cols;
        float ss = lane_dot(x, x, cols);
        float inv = scale / sqrtf((mode == 0 ? ss / (float)cols : ss) + epsilon);
        for (int i = 0; i < cols; ++i) Y[(long)r * cols + i] = x[i] * inv * (mode == 0 ? W[(long)(r % weightRows) * cols + i] : 1.0f);
    }
    return 0;
}

/* kernels/strata.cu:367-377 */
int oracle_strata_ple_gate(unsigned gx, unsigned gy, unsigned gz, const float *Key, const float *Query, float *Gate, int width, int streams) {
    (void)gy; (void)gz;
    for (unsigned c = 0; c < gx && (int)c < streams; ++c) {
        float v = lane_dot(Key + (long)c * width, Query + (long)c * width, width) / sqrtf((float)width);
        float sign = v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f);
        Gate[c] = o_sigmoid(sign * sqrtf(fmaxf(fabsf(v), 0.000001f)));
    }
    return 0;
}

/* kernels/strata.cu:386-397: the greater value wins, the lower index on a tie. */
static int takes(float v, int id, float best, int best_id) { return v > best || (v == best && id < best_id); }
int oracle_strata_argmax(unsigned gx, unsigned gy, unsigned gz, const float *Logits, int *Token, int count) {
    (void)gx; (void)gy; (void)gz;
    float v[LANES];
    int id[LANES];
    for (int l = 0; l < LANES; ++l) {
        v[l] = -3.402823e38f;
        id[l] = count;
        for (int i = l; i < count; i += LANES)
            if (takes(Logits[i], i, v[l], id[l])) { v[l] = Logits[i]; id[l] = i; }
    }
    for (int s = 32; s > 0; s >>= 1)
        for (int l = 0; l < s; ++l)
            if (takes(v[l + s], id[l + s], v[l], id[l])) { v[l] = v[l + s]; id[l] = id[l + s]; }
    Token[0] = id[0];
    return 0;
}

/* Softmax-weighted values over `n` cells for one head; cell c is at row cells[c] (or c). */
static void attend(const float *q, const float *Keys, const float *Values, const int *cells, int n, float *y, int dim, int kvHeads, int kh,
                   float scale, long dmax) {
    static float scores[2048];
    float p[LANES];
    for (int l = 0; l < LANES; ++l) {
        float mx = -3.402823e38f;
        for (int c = l; c < n; c += LANES) {
            const float *k = Keys + ((long)(cells ? cells[c] : c) * kvHeads + kh) * dim;
            float s = 0.0f;
            for (int j = 0; j < dim; ++j) s += q[j] * k[j];
            s *= scale;
            scores[c] = s;
            mx = fmaxf(mx, s);
        }
        p[l] = mx;
    }
    for (int s = 32; s > 0; s >>= 1)
        for (int l = 0; l < s; ++l) p[l] = fmaxf(p[l], p[l + s]);
    float mx = p[0];
    for (int l = 0; l < LANES; ++l) {
        float s = 0.0f;
        for (int c = l; c < n; c += LANES) { scores[c] = strata_oracle_expf(scores[c] - mx); s += scores[c]; }
        p[l] = s;
    }
    float total = tree_sum(p);
    for (int d = 0; d < dim && d < dmax; ++d) {
        float v = 0.0f;
        for (int c = 0; c < n; ++c) v += scores[c] * Values[((long)(cells ? cells[c] : c) * kvHeads + kh) * dim + d];
        y[d] = v / total;
    }
}
/* kernels/strata.cu:334-356 */
int oracle_strata_attention(unsigned gx, unsigned gy, unsigned gz, const float *Q, const float *Keys, const float *Values, const int *Cells,
                            float *Y, int dim, int heads, int kvHeads, int count, float scale) {
    (void)gz;
    if (count < 1 || count > 2048) return 0;
    for (unsigned h = 0; h < gx && (int)h < heads; ++h)
        attend(Q + (long)h * dim, Keys, Values, Cells, count, Y + (long)h * dim, dim, kvHeads, (int)h / (heads / kvHeads), scale, (long)gy * LANES);
    return 0;
}
/* kernels/strata.cu:512-534 */
int oracle_strata_attention_batch(unsigned gx, unsigned gy, unsigned gz, const float *Q, const float *Keys, const float *Values, float *Y,
                                  int dim, int heads, int kvHeads, int position, float scale) {
    for (unsigned t = 0; t < gz; ++t) {
        int n = position + (int)t + 1;
        if (n > 2048) return 0;
        for (unsigned h = 0; h < gx && (int)h < heads; ++h) {
            long row = ((long)t * heads + h) * dim;
            attend(Q + row, Keys, Values, NULL, n, Y + row, dim, kvHeads, (int)h / (heads / kvHeads), scale, (long)gy * LANES);
        }
    }
    return 0;
}

static void kv_rows(unsigned gx, const float *K, const float *V, float *Keys, float *Values, int width, int position, int tokens) {
    long n = lane_count(gx, (long)width * tokens), at = (long)position * width;
    for (long i = 0; i < n; ++i) { Keys[at + i] = K[i]; Values[at + i] = V[i]; }
}
/* kernels/strata.cu:328-330 */
int oracle_strata_kv_append(unsigned gx, unsigned gy, unsigned gz, const float *K, const float *V, float *Keys, float *Values, int width,
                            int position) {
    (void)gy; (void)gz;
    kv_rows(gx, K, V, Keys, Values, width, position, 1);
    return 0;
}
/* kernels/strata.cu:453-456 */
int oracle_strata_kv_append_batch(unsigned gx, unsigned gy, unsigned gz, const float *K, const float *V, float *Keys, float *Values, int width,
                                  int position, int tokens) {
    (void)gy; (void)gz;
    kv_rows(gx, K, V, Keys, Values, width, position, tokens);
    return 0;
}

static void gate_heads(unsigned gx, const float *Attention, const float *FullQ, float *Y, int dim, int heads, int tokens) {
    long n = lane_count(gx, (long)dim * heads * tokens);
    for (long i = 0; i < n; ++i) Y[i] = Attention[i] * o_sigmoid(FullQ[(i / dim) * dim * 2 + dim + i % dim]);
}
/* kernels/strata.cu:357-359 */
int oracle_strata_attention_gate(unsigned gx, unsigned gy, unsigned gz, const float *Attention, const float *FullQ, float *Y, int dim,
                                 int heads) {
    (void)gy; (void)gz;
    gate_heads(gx, Attention, FullQ, Y, dim, heads, 1);
    return 0;
}
/* kernels/strata.cu:457-459 */
int oracle_strata_attention_gate_batch(unsigned gx, unsigned gy, unsigned gz, const float *Attention, const float *FullQ, float *Y, int dim,
                                       int heads, int tokens) {
    (void)gy; (void)gz;
    gate_heads(gx, Attention, FullQ, Y, dim, heads, tokens);
    return 0;
}

/* kernels/strata.cu:314-316 */
int oracle_strata_slice(unsigned gx, unsigned gy, unsigned gz, const float *X, float *Y, int width, int rows, int stride, int offset) {
    (void)gy; (void)gz;
    long n = lane_count(gx, (long)width * rows);
    for (long i = 0; i < n; ++i) Y[i] = X[(i / width) * stride + offset + i % width];
    return 0;
}

static void mix_streams(unsigned gx, const float *Norm, const float *Gate, float *Mixed, int width, int streams, int tokens) {
    long n = lane_count(gx, (long)width * tokens);
    for (long i = 0; i < n; ++i) {
        long t = i / width, d = i % width;
        float v = 0.0f;
        for (int c = 0; c < streams; ++c) v += Norm[(t * streams + c) * width + d] * o_sigmoid(Gate[(t * streams + c) * width + d]);
        Mixed[i] = v / (float)streams;
    }
}
/* kernels/strata.cu:273-277 */
int oracle_strata_hc_mix(unsigned gx, unsigned gy, unsigned gz, const float *Norm, const float *Gate, float *Mixed, int width, int streams) {
    (void)gy; (void)gz;
    mix_streams(gx, Norm, Gate, Mixed, width, streams, 1);
    return 0;
}
/* kernels/strata.cu:403-408 */
int oracle_strata_hc_mix_batch(unsigned gx, unsigned gy, unsigned gz, const float *Norm, const float *Gate, float *Mixed, int width,
                               int streams, int tokens) {
    (void)gy; (void)gz;
    mix_streams(gx, Norm, Gate, Mixed, width, streams, tokens);
    return 0;
}

static void write_streams(unsigned gx, float *Residual, const float *Output, const float *Inject, int width, int streams, int tokens) {
    long hc = (long)width * streams, n = lane_count(gx, hc * tokens);
    for (long i = 0; i < n; ++i) Residual[i] += Output[(i / hc) * width + i % width] * (2.0f * o_sigmoid(Inject[i / width] / (float)streams));
}
/* kernels/strata.cu:278-281 */
int oracle_strata_hc_write(unsigned gx, unsigned gy, unsigned gz, float *Residual, const float *Output, const float *Inject, int width,
                           int streams) {
    (void)gy; (void)gz;
    write_streams(gx, Residual, Output, Inject, width, streams, 1);
    return 0;
}
/* kernels/strata.cu:409-412 */
int oracle_strata_hc_write_batch(unsigned gx, unsigned gy, unsigned gz, float *Residual, const float *Output, const float *Inject, int width,
                                 int streams, int tokens) {
    (void)gy; (void)gz;
    write_streams(gx, Residual, Output, Inject, width, streams, tokens);
    return 0;
}

static void broadcast_gate(unsigned gx, const float *Value, const float *Gate, float *Y, int width, int streams, int tokens) {
    long hc = (long)width * streams, n = lane_count(gx, hc * tokens);
    for (long i = 0; i < n; ++i) Y[i] = Value[(i / hc) * width + i % width] * Gate[i / width];
}
/* kernels/strata.cu:378-380 */
int oracle_strata_ple_broadcast(unsigned gx, unsigned gy, unsigned gz, const float *Value, const float *Gate, float *Y, int width, int streams) {
    (void)gy; (void)gz;
    broadcast_gate(gx, Value, Gate, Y, width, streams, 1);
    return 0;
}
/* kernels/strata.cu:460-463 */
int oracle_strata_ple_broadcast_batch(unsigned gx, unsigned gy, unsigned gz, const float *Value, const float *Gate, float *Y, int width,
                                      int streams, int tokens) {
    (void)gy; (void)gz;
    broadcast_gate(gx, Value, Gate, Y, width, streams, tokens);
    return 0;
}
/* kernels/strata.cu:381-383 */
int oracle_strata_ple_add(unsigned gx, unsigned gy, unsigned gz, float *Residual, const float *Gated, const float *Conv, int n) {
    (void)gy; (void)gz;
    long m = lane_count(gx, n);
    for (long i = 0; i < m; ++i) Residual[i] += Gated[i] + Conv[i];
    return 0;
}

/* kernels/strata.cu:287-295 and :413-424. With no history (taps == 1) the prompt entry of the
 * reference stores the newest tap one element before the history buffer; nothing is stored here
 * (the CUDA entry reports that store as an index outside its buffer). */
static void causal_conv(unsigned gx, float *History, const float *X, const float *W, float *Y, int channels, int taps, int dilation,
                        int activation, int tokens) {
    long span = (long)(taps - 1) * dilation, n = lane_count(gx, channels);
    for (long c = 0; c < n; ++c) {
        float *h = History + c * span;
        for (int t = 0; t < tokens; ++t) {
            float x = X[(long)t * channels + c], s = 0.0f;
            for (int k = 0; k < taps - 1; ++k) s += h[(long)k * dilation] * W[c * taps + k];
            s += x * W[c * taps + taps - 1];
            Y[(long)t * channels + c] = activation == 1 ? o_silu(s) : s;
            for (long k = 0; k + 1 < span; ++k) h[k] = h[k + 1];
            if (span > 0) h[span - 1] = x;
        }
    }
}
int oracle_strata_conv(unsigned gx, unsigned gy, unsigned gz, float *History, const float *X, const float *W, float *Y, int channels, int taps,
                       int dilation, int activation) {
    (void)gy; (void)gz;
    causal_conv(gx, History, X, W, Y, channels, taps, dilation, activation, 1);
    return 0;
}
int oracle_strata_conv_batch(unsigned gx, unsigned gy, unsigned gz, float *History, const float *X, const float *W, float *Y, int channels,
                             int taps, int dilation, int activation, int tokens) {
    (void)gy; (void)gz;
    causal_conv(gx, History, X, W, Y, channels, taps, dilation, activation, tokens);
    return 0;
}

/* kernels/strata.cu:296-301 and :425-431: softplus through log(1 + e^x) below 20. */
static void delta_gates(unsigned gx, const float *Alpha, const float *Beta, const float *A, const float *Dt, float *Decay, float *Strength,
                        int heads, int tokens) {
    long n = lane_count(gx, (long)heads * tokens);
    for (long i = 0; i < n; ++i) {
        float x = Alpha[i] + Dt[i % heads];
        float sp = x > 20.0f ? x : logf(1.0f + strata_oracle_expf(x));
        Decay[i] = strata_oracle_expf(A[i % heads] * sp);
        Strength[i] = o_sigmoid(Beta[i]);
    }
}
int oracle_strata_gdn_gates(unsigned gx, unsigned gy, unsigned gz, const float *Alpha, const float *Beta, const float *A, const float *Dt,
                            float *Decay, float *Strength, int heads) {
    (void)gy; (void)gz;
    delta_gates(gx, Alpha, Beta, A, Dt, Decay, Strength, heads, 1);
    return 0;
}
int oracle_strata_gdn_gates_batch(unsigned gx, unsigned gy, unsigned gz, const float *Alpha, const float *Beta, const float *A,
                                  const float *Dt, float *Decay, float *Strength, int heads, int tokens) {
    (void)gy; (void)gz;
    delta_gates(gx, Alpha, Beta, A, Dt, Decay, Strength, heads, tokens);
    return 0;
}

/* kernels/strata.cu:304-313 and :432-444: the gated delta rule on State [dim][valueHeads][dim]. */
static void delta_rule(unsigned gx, float *State, const float *Q, const float *K, const float *V, const float *Decay, const float *Beta,
                       float *Y, int dim, int keyHeads, int valueHeads, int tokens) {
    long stride = (long)valueHeads * dim, n = lane_count(gx, stride);
    for (long col = 0; col < n; ++col) {
        long h = col / dim, kh = h % keyHeads;
        for (int t = 0; t < tokens; ++t) {
            const float *k = K + ((long)t * keyHeads + kh) * dim, *q = Q + ((long)t * keyHeads + kh) * dim;
            long gh = (long)t * valueHeads + h;
            float pred = 0.0f, out = 0.0f;
            for (int i = 0; i < dim; ++i) { float *s = State + i * stride + col; *s *= Decay[gh]; pred += *s * k[i]; }
            float delta = (V[t * stride + col] - pred) * Beta[gh];
            for (int i = 0; i < dim; ++i) { float *s = State + i * stride + col; *s += k[i] * delta; out += *s * q[i]; }
            Y[t * stride + col] = out;
        }
    }
}
int oracle_strata_gdn_step(unsigned gx, unsigned gy, unsigned gz, float *State, const float *Q, const float *K, const float *V,
                           const float *Decay, const float *Beta, float *Y, int dim, int keyHeads, int valueHeads) {
    (void)gy; (void)gz;
    delta_rule(gx, State, Q, K, V, Decay, Beta, Y, dim, keyHeads, valueHeads, 1);
    return 0;
}
int oracle_strata_gdn_batch(unsigned gx, unsigned gy, unsigned gz, float *State, const float *Q, const float *K, const float *V,
                            const float *Decay, const float *Beta, float *Y, int dim, int keyHeads, int valueHeads, int tokens) {
    (void)gy; (void)gz;
    delta_rule(gx, State, Q, K, V, Decay, Beta, Y, dim, keyHeads, valueHeads, tokens);
    return 0;
}
