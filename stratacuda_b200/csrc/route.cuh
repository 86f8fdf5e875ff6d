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
    const int t = threadIdx.x & 31;
    float pa[8], pb[8];
    float ma = -3.402823e38f, mb = -3.402823e38f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        int ea = t + 64 * m, eb = ea + 32;
        if (ea < experts) ma = fmaxf(ma, logits[ea]);
        if (eb < experts) mb = fmaxf(mb, logits[eb]);
    }
    float mx = fmaxf(ma, mb);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        float o = __shfl_down_sync(0xffffffffu, mx, s);
        if (t < s) mx = fmaxf(mx, o);
    }
    mx = __shfl_sync(0xffffffffu, mx, 0);
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        int ea = t + 64 * m, eb = ea + 32;
        pa[m] = ea < experts ? ref_expf(__fsub_rn(logits[ea], mx)) : 0.0f;
        pb[m] = eb < experts ? ref_expf(__fsub_rn(logits[eb], mx)) : 0.0f;
        if (ea < experts) sa = __fadd_rn(sa, pa[m]);
        if (eb < experts) sb = __fadd_rn(sb, pb[m]);
    }
    float sum = __shfl_sync(0xffffffffu, tree64(sa, sb), 0);
    float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int m = 0; m < 8; ++m) { pa[m] = __fmul_rn(pa[m], inv); pb[m] = __fmul_rn(pb[m], inv); }
    for (int k = 0; k < topK; ++k) {
        float ba = -1.0f, bb = -1.0f;
        int ia = experts, ib = experts;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            int ea = t + 64 * m, eb = ea + 32;
            if (ea < experts && (pa[m] > ba || (pa[m] == ba && ea < ia))) { ba = pa[m]; ia = ea; }
            if (eb < experts && (pb[m] > bb || (pb[m] == bb && eb < ib))) { bb = pb[m]; ib = eb; }
        }
        if (bb > ba || (bb == ba && ib < ia)) { ba = bb; ia = ib; }  // s = 32 step, in-thread
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) {
            float v = __shfl_down_sync(0xffffffffu, ba, s);
            int j = __shfl_down_sync(0xffffffffu, ia, s);
            if (t < s && (v > ba || (v == ba && j < ia))) { ba = v; ia = j; }
        }
        int win = __shfl_sync(0xffffffffu, ia, 0);
        float best = __shfl_sync(0xffffffffu, ba, 0);
        if (t == 0) { ids[k] = win; sel[k] = best; }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (t + 64 * m == win) pa[m] = -1.0f;
            if (t + 32 + 64 * m == win) pb[m] = -1.0f;
        }
    }
    __syncwarp();
    if (t == 0) {
        float denom = 0.0f;
        for (int k = 0; k < topK; ++k) denom = __fadd_rn(denom, sel[k]);
        denom = fmaxf(denom, 0.00006103515625f);
        for (int k = 0; k < topK; ++k) weights[k] = __fdiv_rn(sel[k], denom);
    }
    __syncwarp();
}

}  // namespace strata
