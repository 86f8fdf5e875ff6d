// One-warp router shared by the strata_router entries and the fused layer.
#pragma once
#include "common.cuh"

namespace strata {

// kernels/strata.cu:238-270 for one token, by one warp: softmax over all experts (max, exp,
// 64-lane sum, multiply by 1/sum), then k rounds of lane-strided argmax with the lower ID
// winning ties, then weights = sel_k / max(sum_k sel_k, 2^-14). Thread t owns virtual lanes
// t (experts t + 64m) and t + 32 (experts t + 32 + 64m), m < 8. `sel` is 32 floats of
// scratch for this warp; `exp_tab` (optional) the expf table staged in shared memory.
__device__ __forceinline__ void route_warp(const float *logits, int experts, int topK, int *ids, float *weights, float *sel,
                                           const unsigned long long *exp_tab = nullptr) {
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
        const float xa = ref_expf(__fsub_rn(logits[ea], mx), exp_tab), xb = ref_expf(__fsub_rn(logits[eb], mx), exp_tab);
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


// ---------------------------------------------------------------------------------------
// The same routing for one token by a group of W consecutive warps (W in {1, 2, 4, 8}):
// thread i of the group owns experts i + 32W m. Steps, each exact:
//   max      order-free (fmaxf), so any partition gives the reference's value;
//   exp      one ref_expf per expert, written back over the logits;
//   sum      the reference's 64-lane order (lane l adds experts l, l+64, ... from 0, then the
//            tree), recomputed by every warp of the group from shared memory;
//   top-k    keys (probability bits + 1, inverted id) are a total order equal to the
//            reference's selection order. The 512 keys form 8 subgroups of 64 (two per
//            lane of one warp); each subgroup is bitonic-sorted and its first K keys become
//            candidates. The global top K lie among them (an element beaten by fewer than K
//            elements overall is beaten by fewer than K of its subgroup), and a candidate's
//            rank is the number of candidates above it.
//   weights  sel_k / max(sum_k sel_k, 2^-14), the sum in selection order.
// `lg` holds the token's logits (512 floats; entries past `experts` are ignored) and is
// overwritten. `red` holds W floats, `cand` 8*topK keys (16-byte aligned), `nzc` one int
// that the caller zeroes before the call; ids/sel/weights receive topK entries. Group
// synchronisation uses named barrier `bar_id` (W > 1). `exp_tab` (optional): the expf table
// staged in shared memory by the caller.
template <int W>
__device__ __forceinline__ void group_sync(int bar_id) {
    if (W == 1) __syncwarp();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(32 * W) : "memory");
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
    const unsigned lo = __shfl_xor_sync(0xffffffffu, (unsigned)v, m);
    const unsigned hi = __shfl_xor_sync(0xffffffffu, (unsigned)(v >> 32), m);
    return ((unsigned long long)hi << 32) | lo;
}

// Sorts 64 keys, element 2*lane + j in k.x (j = 0) / k.y (j = 1), into descending order
// (bitonic network, unrolled: measured 4% faster for 8-token decode than one rolled copy).
static __device__ __forceinline__ ulonglong2 warp_sort64_desc(ulonglong2 k, int lane) {
    unsigned long long k0 = k.x, k1 = k.y;
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
        const bool desc = ((2 * lane) & size) == 0;  // direction of this element's block
#pragma unroll
        for (int stride = size >> 1; stride > 1; stride >>= 1) {
            const unsigned long long o0 = shfl_xor_u64(k0, stride >> 1), o1 = shfl_xor_u64(k1, stride >> 1);
            const bool take_max = (((2 * lane) & stride) == 0) == desc;  // lower element of a descending pair
            k0 = take_max ? (k0 > o0 ? k0 : o0) : (k0 < o0 ? k0 : o0);
            k1 = take_max ? (k1 > o1 ? k1 : o1) : (k1 < o1 ? k1 : o1);
        }
        const unsigned long long hi = k0 > k1 ? k0 : k1, lo = k0 > k1 ? k1 : k0;
        k0 = desc ? hi : lo;
        k1 = desc ? lo : hi;
    }
    return make_ulonglong2(k0, k1);
}

// `after_ids` runs on every thread of the group once the ids are final, before the weights
// (the one-token decode layer requests its expert's tiles there).
template <int W, class AfterIds>
__device__ __forceinline__ void route_group(float *lg, int experts, int topK, float *red, unsigned long long *cand, int *nzc,
                                            int *ids, float *sel, float *weights, int bar_id, const unsigned long long *exp_tab,
                                            AfterIds &&after_ids) {
    constexpr int T = 32 * W, NPT = 512 / T;
    const int i = threadIdx.x % T, lane = threadIdx.x & 31, wg = i >> 5;
    float v[NPT];
    float mx = -3.402823e38f;
#pragma unroll
    for (int m = 0; m < NPT; ++m) {
        const int e = i + T * m;
        v[m] = lg[e];
        mx = fmaxf(mx, e < experts ? v[m] : -3.402823e38f);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    if (W > 1) {
        if (lane == 0) red[wg] = mx;
        group_sync<W>(bar_id);
        mx = red[0];
#pragma unroll
        for (int k = 1; k < W; ++k) mx = fmaxf(mx, red[k]);
    }
#pragma unroll
    for (int m = 0; m < NPT; ++m) {
        const int e = i + T * m;
        const float ex = ref_expf(__fsub_rn(v[m], mx), exp_tab);
        v[m] = e < experts ? ex : 0.0f;
        lg[e] = v[m];
    }
    group_sync<W>(bar_id);
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        sa = __fadd_rn(sa, lg[lane + 64 * m]);
        sb = __fadd_rn(sb, lg[lane + 32 + 64 * m]);
    }
    const float inv = __fdiv_rn(1.0f, __shfl_sync(0xffffffffu, tree64(sa, sb), 0));
#pragma unroll 1  // one sort network in the code: unrolled copies cost more in instruction fetch than they gain
    for (int a = 0; a < NPT / 2; ++a) {
        const int e0 = i + T * (2 * a), e1 = e0 + T;
        const float p0 = __fmul_rn(lg[e0], inv), p1 = __fmul_rn(lg[e1], inv);  // lg holds the masked exponentials
        const ulonglong2 k = warp_sort64_desc(
            make_ulonglong2(e0 < experts && p0 >= 0.0f ? ((unsigned long long)(__float_as_uint(p0) + 1u) << 32) | (0xffffffffu - (unsigned)e0) : 0ull,
                            e1 < experts && p1 >= 0.0f ? ((unsigned long long)(__float_as_uint(p1) + 1u) << 32) | (0xffffffffu - (unsigned)e1) : 0ull),
            lane);
        const unsigned long long k0 = k.x, k1 = k.y;
        unsigned long long *c = cand + (wg * (NPT / 2) + a) * topK;
        if (2 * lane < topK) c[2 * lane] = k0;
        if (2 * lane + 1 < topK) c[2 * lane + 1] = k1;
        const int nz = __popc(__ballot_sync(0xffffffffu, 2 * lane < topK && k0 != 0ull)) +
                       __popc(__ballot_sync(0xffffffffu, 2 * lane + 1 < topK && k1 != 0ull));
        if (lane == 0 && nz) atomicAdd(nzc, nz);
    }
    group_sync<W>(bar_id);
    const int N = 8 * topK;  // even
    const ulonglong2 *c2 = reinterpret_cast<const ulonglong2 *>(cand);
    for (int c = i; c < N; c += T) {
        const unsigned long long kc = cand[c];
        if (kc == 0ull) continue;
        int r0 = 0, r1 = 0;
#pragma unroll 8
        for (int x = 0; x < N / 2; ++x) {
            const ulonglong2 v = c2[x];
            r0 += v.x > kc;
            r1 += v.y > kc;
        }
        const int r = r0 + r1;
        if (r < topK) {
            ids[r] = (int)(0xffffffffu - (unsigned)kc);
            sel[r] = __uint_as_float((unsigned)(kc >> 32) - 1u);
        }
    }
    if (i < topK && i >= *nzc) {  // rounds past the last valid key find nothing: the reference records -1
        ids[i] = -1;
        sel[i] = -1.0f;
    }
    group_sync<W>(bar_id);
    after_ids();
    if (i < topK) {
        float denom = 0.0f;  // sequential, in selection order
        for (int k = 0; k < topK; ++k) denom = __fadd_rn(denom, sel[k]);
        denom = fmaxf(denom, 0.00006103515625f);
        weights[i] = __fdiv_rn(sel[i], denom);
    }
    group_sync<W>(bar_id);
}
template <int W>
__device__ __forceinline__ void route_group(float *lg, int experts, int topK, float *red, unsigned long long *cand, int *nzc,
                                            int *ids, float *sel, float *weights, int bar_id, const unsigned long long *exp_tab = nullptr) {
    route_group<W>(lg, experts, topK, red, cand, nzc, ids, sel, weights, bar_id, exp_tab, [] {});
}

}  // namespace strata
