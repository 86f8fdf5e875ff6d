// One-warp router shared by the strata_router entries and the fused layer.
#pragma once
#include "common.cuh"

namespace strata {

// kernels/strata.cu:238-270 for one token, by one warp: softmax over all experts (max, exp,
// 64-lane sum, multiply by 1/sum), then k rounds of lane-strided argmax with the lower ID
// winning ties, then weights = sel_k / max(sum_k sel_k, 2^-14). Thread t owns virtual lanes
// t (experts t + 64m) and t + 32 (experts t + 32 + 64m), m < 8. `sel` is 32 floats of
// scratch for this warp.
__device__ __forceinline__ void route_warp(const float *logits, int experts, int topK, int *ids, float *weights, float *sel) {
    // `logits` must hold 512 readable floats (entries past `experts` may be anything): every
    // lane evaluates all 16 of its slots without branches and masks the unused ones, which
    // lets the 16 exp evaluations interleave. Masked slots contribute exactly nothing:
    // fmaxf(m, -3.402823e38f) == m, s + 0.0f == s for the non-negative sums.
    const int t = threadIdx.x & 31;
    float pa[8], pb[8];
    float ma = -3.402823e38f, mb = -3.402823e38f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int ea = t + 64 * m, eb = ea + 32;
        ma = fmaxf(ma, ea < experts ? logits[ea] : -3.402823e38f);
        mb = fmaxf(mb, eb < experts ? logits[eb] : -3.402823e38f);
    }
    float mx = fmaxf(ma, mb);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_down_sync(0xffffffffu, mx, s));  // lane 0 holds the tree
    mx = __shfl_sync(0xffffffffu, mx, 0);
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int ea = t + 64 * m, eb = ea + 32;
        const float xa = ref_expf(__fsub_rn(logits[ea], mx)), xb = ref_expf(__fsub_rn(logits[eb], mx));
        pa[m] = ea < experts ? xa : 0.0f;
        pb[m] = eb < experts ? xb : 0.0f;
        sa = __fadd_rn(sa, pa[m]);
        sb = __fadd_rn(sb, pb[m]);
    }
    float sum = __shfl_sync(0xffffffffu, tree64(sa, sb), 0);
    float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int m = 0; m < 8; ++m) { pa[m] = __fmul_rn(pa[m], inv); pb[m] = __fmul_rn(pb[m], inv); }
    // The reference's rounds (lane-strided scan with strict >, ascending ids, then the tree)
    // always select the largest remaining probability and, among equal ones, the lowest id: a
    // total order. Encode it as a 64-bit key (probability bits + 1 above, inverted id below;
    // removed entries (-1) and NaN get 0), sort each lane's 16 keys descending once, then each
    // round is two warp reductions (largest high word, lowest id holding it) and a shift in the
    // winning lane.
    unsigned long long key[16];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int ea = t + 64 * m, eb = ea + 32;
        key[2 * m] = ea < experts && pa[m] >= 0.0f ? ((unsigned long long)(__float_as_uint(pa[m]) + 1u) << 32) | (0xffffffffu - (unsigned)ea) : 0ull;
        key[2 * m + 1] = eb < experts && pb[m] >= 0.0f ? ((unsigned long long)(__float_as_uint(pb[m]) + 1u) << 32) | (0xffffffffu - (unsigned)eb) : 0ull;
    }
#pragma unroll
    for (int size = 2; size <= 16; size <<= 1)
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;  // descending runs first: the final merge is descending
                    const unsigned long long a = key[i], b = key[j];
                    const bool swap = desc ? (a < b) : (a > b);
                    key[i] = swap ? b : a;
                    key[j] = swap ? a : b;
                }
            }
    for (int k = 0; k < topK; ++k) {
        const unsigned hi = (unsigned)(key[0] >> 32);
        const unsigned top = __reduce_max_sync(0xffffffffu, hi);
        const unsigned win = __reduce_min_sync(0xffffffffu, hi == top ? 0xffffffffu - (unsigned)key[0] : 0xffffffffu);
        if (t == 0) {
            ids[k] = (int)win;
            sel[k] = top ? __uint_as_float(top - 1u) : -1.0f;
        }
        const bool mine = hi == top && 0xffffffffu - (unsigned)key[0] == win;
#pragma unroll
        for (int i = 0; i < 15; ++i) key[i] = mine ? key[i + 1] : key[i];
        key[15] = mine ? 0ull : key[15];
    }
    __syncwarp();
    float denom = 0.0f;  // sequential, in selection order, as the reference
    for (int k = 0; k < topK; ++k) denom = __fadd_rn(denom, sel[k]);
    denom = fmaxf(denom, 0.00006103515625f);
    for (int k = t; k < topK; k += 32) weights[k] = __fdiv_rn(sel[k], denom);
    __syncwarp();
}

}  // namespace strata
