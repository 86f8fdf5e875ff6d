// Fast fused mixture-of-experts layer for decode batches (tokens <= 8): ONE persistent
// cooperative launch, one CTA per SM, 8 warps, two grid-wide arrivals (three from 3 tokens).
//
// Work units. An expert's layer splits by hidden columns into F/64 units: unit (slot, j)
// owns hidden values [64j, 64j+64) of one expert slot (slot 0 = the shared expert, slots
// 1.. = distinct routed experts in first-appearance order, src/prefill.js:56-60). A unit
//   * multiplies the 128 interleaved gate/up rows of its hidden values (blob rows
//     128j .. 128j+127, full width) with the slot's tokens: warp w takes rows 16w .. 16w+15;
//   * forms hidden = silu(gate) * up for its 64 values and tokens;
//   * multiplies the down projection's column slice (all H rows, code bytes 16j .. 16j+15,
//     one scale group) with them: warp w takes rows H/8 w .. H/8 (w+1);
//   * stores weight * result, one partial row of y per (group j, token-expert pair), to a
//     global buffer with plain 16-byte stores.
// So the hidden values never leave the CTA. Units are dealt round-robin: unit u runs on
// CTA u % G. After a second grid arrival every CTA sums a slice of y from the partial rows
// in a fixed order (group j, then the shared expert and the routed pairs in selection
// order): y is the same bits run to run, within 1e-5 relative L2 of the reference (tested).
// (Adding the partials with atomics instead serialised in L2: every y element received
// one add per unit, up to ~90.)
//
// Phase 0 (from entry): x is staged in shared memory; router logits, row r of the 512 (+1
// shared-gate row) on CTA r % G, warp r / G, in the reference's exact order
// (kernels/strata.cu:156-165) so that the routing below is bit-identical. A CTA arrives as
// soon as its rows are written; the remaining warps turn x into integer tensor-core operands
// while the grid gathers. CTAs that own a shared-expert unit start its copies at entry and
// compute its gate/up part before waiting at the arrival. y is not touched before the final
// sum, so it needs no zeroing.
// Phase 1 (after the arrival: all logits written): with one or two tokens every CTA routes
// them redundantly (route.cuh route_group: 8 or 4 warps per token), so only the logits cross
// the grid; with more, CTA G-1-t routes token t with all 8 warps and a third arrival hands
// the ids and weights to every CTA (one warp per token on every CTA took 16 us at 8 tokens).
// Each CTA then builds the expert slots and runs its units.
//
// Memory pipeline, per warp: a ring of gate/up stages (one 16-row x 128-byte box of codes,
// 128-byte swizzle, by TMA tensor copy; the first chunk of a unit also brings the 16 rows'
// FP16 scales, 1 KB contiguous, by one bulk copy) and one down stage (H/8 rows x 16 bytes of
// codes plus each row's 4-byte scale word, by cp.async from all lanes: the rows are too short
// for the TMA engine, which spends one request per box row). The down stages share their
// memory with the phase-0 copy of x and the routing scratch, so they are first issued once
// routing is done.
//
// Tensor-core math (exact integer products): mma.sync m16n8k32 u8 x s8 -> s32.
//   A = weight codes c in {0..3} as u8: four codes per register by one shift and one mask.
//   B = activations as three signed 8-bit digits: v = round(x * 2^k) (k per vector, |v| <
//       2^22), v = d0 + 256 d1 + 65536 d2. Each token takes four MMA columns (d0, d1, d2,
//       zero), so one MMA serves two tokens; a unit with one or two tokens needs one MMA per
//       32-element step.
//   Per 64-group: sum((c-1) v) = (acc0 + 256 acc1 + 65536 acc2) - sum(v), exact in int32;
//   then total += scale * float(that) in F32, and the row is multiplied by 2^-k.
// The only rounding is v (2^-22 of the vector's largest |x|) and the F32 accumulation.
//
// All waits (the grid arrivals, mbarriers) are bounded: past the limit the kernel records
// kErrWaitTimeout, waits (bounded) for its own copies in flight and leaves.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "q2mma.cuh"
#include "route.cuh"

namespace strata {
namespace fast {

using namespace q2;

constexpr int kMaxPairs = kMaxTokens * 32;
constexpr int kMaxSlots = kMaxPairs + 1;
constexpr int kXBuildBarrier = 9;     // named barrier of the x-operand warps (route groups use 1..8)
constexpr int kRowsBarrier = 10;      // named barrier of the router-row warps
constexpr int kSplitRouteTokens = 3;  // from this many tokens on, routing is split over CTAs

struct Params {
    MoeLayerDev L;
    const float *x;
    int tokens;
    float *y;
    int *ids;
    float *weights;
    float *logits;   // [tokens][experts]
    float *sg;       // [tokens]
    float *part;     // [F/64][tokens*topK + tokens][H] partial rows of y
    unsigned *sync;  // [0] first arrival, [1] second arrival, [2] exits, [3] routed tokens (split routing)
    unsigned *err;
    unsigned long long spin_limit;
    // TMA maps: [0] routed experts, [1] the shared expert
    CUtensorMap tm_gu[2];  // gate/up codes: {H/4 bytes, 2F rows, experts}, box {128, 16, 1}, 128B swizzle
    CUtensorMap tm_gu4[2]; // the same 16 rows in one request: box {128, 16, H/512 chunks, 1} (units of one box per warp)
};


template <int H, int F>
struct Smem {
    using G = Geo<H, F>;
    unsigned char gu_codes[kWarps][G::SGU][2048];  // 1024-aligned (128-byte swizzle)
    alignas(16) unsigned short gu_scales[kWarps][2][G::GS_BYTES / 2];  // by unit parity
    union Region {
        unsigned char down[kWarps][G::DN_STAGE];  // after routing
        float x[kMaxTokens * H];                  // phase 0
        struct Route {
            float lg[kMaxTokens][512];
            alignas(16) unsigned long long cand[kMaxTokens][8 * 32];
            float red[kMaxTokens][kWarps];
            float sel[kMaxTokens][32];
            int nzc[kMaxTokens];
            int owner[512];  // lowest pair index per expert
            int cnt[512];    // pairs per expert
            short slot_of[512];
            int wcount[kWarps];
        } r;  // routing and slot building
    } u;
    uint2 xf[G::NG * 2 * kMaxTokens * 4 * 3];  // x digits [group][h][token][q][digit]
    int xsum[kMaxTokens][G::NG];
    float xscale[kMaxTokens];
    unsigned xmax[kMaxTokens];
    float sgw[kMaxTokens];                    // shared-expert weights sigmoid(shared-gate logit)
    float hid[2][kMaxTokens][64];             // hidden values of the current unit (double-buffered by unit parity)
    float hmaxw[2][kWarps][kMaxTokens];       // per-warp max |hidden| of each token slot
    int ids[kMaxPairs];
    float wts[kMaxPairs];
    short slot_expert[kMaxSlots];
    short slot_pair[kMaxSlots][kMaxTokens];
    unsigned char slot_n[kMaxSlots];
    unsigned long long bar_gu[kWarps][G::SGU];
    int n_slots;
    int abort_flag;
};

// Bounded wait of thread 0 for *counter >= target, then a CTA barrier; sets abort on timeout.
__device__ __forceinline__ void cta_spin_until(const unsigned *counter, unsigned target, unsigned long long limit, int *abort_flag) {
    if (threadIdx.x == 0) {
        for (unsigned long long i = 0;; ++i) {
            if (ld_acquire(counter) >= target) break;
            if (i > limit) {
                *abort_flag = 1;
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
}

// Split routing (three or more tokens), out of line so that the one-token path keeps its
// code compact (instruction fetch is on that path's critical path). Token t on this CTA:
// wait for every logit, route with all eight warps, publish ids and weights, arrive.
template <int H, int F>
__device__ __forceinline__ void split_route_token(const Params &P, Smem<H, F> &S, int t) {
    const int tid = threadIdx.x, E = P.L.experts, K = P.L.topK;
    cta_spin_until(&P.sync[0], gridDim.x, P.spin_limit, &S.abort_flag);
    if (S.abort_flag) return;
    float *lg = S.u.r.lg[0];
    const float *src = P.logits + (long long)t * E;
    if ((E & 3) == 0) {
        for (int i = tid; i < E / 4; i += kThreads) reinterpret_cast<float4 *>(lg)[i] = __ldcg(reinterpret_cast<const float4 *>(src) + i);
    } else {
        for (int i = tid; i < E; i += kThreads) lg[i] = __ldcg(src + i);
    }
    if (tid == 0) S.u.r.nzc[0] = 0;
    __syncthreads();
    route_group<8>(lg, E, K, S.u.r.red[0], S.u.r.cand[0], &S.u.r.nzc[0], S.ids + t * K, S.u.r.sel[0], S.wts + t * K, 1);
    __syncthreads();
    for (int k = tid; k < K; k += kThreads) {
        P.ids[t * K + k] = S.ids[t * K + k];
        P.weights[t * K + k] = S.wts[t * K + k];
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&P.sync[3], 1u);
    }
}
// Every CTA, split routing: wait for all B tokens' routing, then take the ids and weights.
template <int H, int F>
__device__ __forceinline__ void split_route_receive(const Params &P, Smem<H, F> &S) {
    const int tid = threadIdx.x, B = P.tokens, K = P.L.topK;
    cta_spin_until(&P.sync[3], (unsigned)B, P.spin_limit, &S.abort_flag);  // every token routed (and so every logit written)
    if (S.abort_flag) return;
    for (int p = tid; p < B * K; p += kThreads) {
        S.ids[p] = __ldcg(P.ids + p);
        S.wts[p] = __ldcg(P.weights + p);
    }
    for (int e = tid; e < P.L.experts; e += kThreads) {
        S.u.r.owner[e] = 0x7fffffff;
        S.u.r.cnt[e] = 0;
    }
    if (tid < B) S.sgw[tid] = ref_sigmoid(__ldcg(P.sg + tid));
    __syncthreads();
}

// SPLIT: the instance for three or more tokens (split routing, router rows two tokens at a
// time, 16-byte x loads); the other one keeps the one-token code compact: the presence of
// the split code alone, even out of line, cost the one-token launch 0.8 us (instruction
// fetch is on its critical path).
template <int H, int F, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_moe_fast(const __grid_constant__ Params P) {
    using Gm = Geo<H, F>;
    constexpr int NG = Gm::NG, NJ = Gm::NJ, CPT = Gm::CPT, SGU = Gm::SGU, RW = Gm::RW;
    extern __shared__ unsigned char smem_raw[];
    auto &S = *reinterpret_cast<Smem<H, F> *>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
    const MoeLayerDev &L = P.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const int G = gridDim.x, cta = blockIdx.x;
    const int B = P.tokens, K = L.topK, E = L.experts;
    const long long d_codes_b = 2LL * F * H / 4, gu_scales_b = 3LL * F * H / 4, d_scales_b = gu_scales_b + 2LL * F * (H / 64) * 2;

    if (tid == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int s = 0; s < SGU; ++s) mbar_init(&S.bar_gu[w][s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
        S.n_slots = 1;
        for (int i = 0; i < 2; ++i) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.tm_gu[i])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.tm_gu4[i])) : "memory");
        }
    }
    if (tid < kMaxTokens) S.xmax[tid] = 0u;
    __syncthreads();

    // ------------------------------------------------------------------ copy pipeline (per warp)
    // Gate/up chunk k of this warp belongs to the CTA's unit k / CPT, column chunk k % CPT; down
    // stage i to unit i. Before routing only a shared-expert unit (u < NJ) is known.
    int gu_known = cta < NJ ? CPT : 0, dn_known = 0;
    int gu_issued = 0, gu_done = 0, dn_issued = 0, dn_done = 0;
    bool stalled = false;  // this warp saw a wait time out: issue nothing more
    // Unit index of the CTA's unit ui. One or two tokens: round-robin, unit u on CTA u % G.
    // Split instance: the CTAs of the shared-expert units (0 .. NJ-1, whose unit carries
    // every token) sit out the first round of routed units, and every later round starts at
    // CTA NJ, so a partial last round also misses them.
    auto unit_index = [&](int ui) -> int {
        if constexpr (SPLIT) {
            if (ui == 0) return cta;
            return cta < NJ ? (ui + 1) * G + cta - NJ : ui * G + cta - NJ;
        } else {
            return cta + ui * G;
        }
    };
    auto unit_of = [&](int ui, int &slot, int &j, int &m, int &e) {
        const int u = unit_index(ui);
        slot = u / NJ;
        j = u % NJ;
        m = slot == 0 ? 1 : 0;
        e = slot == 0 ? 0 : S.slot_expert[slot];
    };
    auto blob_of = [&](int slot, int e) {
        return reinterpret_cast<const unsigned char *>(slot == 0 ? L.shared_blob : L.blobs + (long long)e * L.blob_words);
    };
    // With as many stages as chunks per unit (H 2048) a warp's unit is one request of its 16 full
    // rows (8 KB, measured 2.5x faster per SM than four 2 KB boxes of the same rows), landing
    // chunk-major in stages 0..CPT-1 on stage 0's barrier; otherwise one box per chunk.
    constexpr bool UNIT_BOX = CPT == SGU;
    auto issue_gu = [&](int k) {
        const int ui = k / CPT, sub = k % CPT, st = k % SGU;
        int slot, j, m, e;
        unit_of(ui, slot, j, m, e);
        if (UNIT_BOX) {
            if (lane == 0 && sub == 0) {
                unsigned long long *bar = &S.bar_gu[warp][0];
                mbar_expect(bar, 2048 * CPT + Gm::GS_BYTES);
                tma_4d(S.gu_codes[warp][0], &P.tm_gu4[m], 0, 128 * j + 16 * warp, 0, e, bar);
                bulk_copy(S.gu_scales[warp][ui & 1], blob_of(slot, e) + gu_scales_b + (long long)(128 * j + 16 * warp) * 2 * NG,
                          Gm::GS_BYTES, bar);
            }
        } else if (lane == 0) {
            unsigned long long *bar = &S.bar_gu[warp][st];
            mbar_expect(bar, 2048 + (sub == 0 ? Gm::GS_BYTES : 0));
            tma_3d(S.gu_codes[warp][st], &P.tm_gu[m], 128 * sub, 128 * j + 16 * warp, e, bar);
            if (sub == 0)  // the unit's scales ride on its first chunk (chunks are consumed in order)
                bulk_copy(S.gu_scales[warp][ui & 1], blob_of(slot, e) + gu_scales_b + (long long)(128 * j + 16 * warp) * 2 * NG,
                          Gm::GS_BYTES, bar);
        }
    };
    auto issue_dn = [&](int ui) {  // all lanes: row r of this warp's slice by lane r % 32
        int slot, j, m, e;
        unit_of(ui, slot, j, m, e);
        const unsigned char *blob = blob_of(slot, e);
        unsigned char *dst = S.u.down[warp];
#pragma unroll 2
        for (int r = lane; r < RW; r += 32) {
            const long long row = (long long)RW * warp + r;
            cp_async16(dst + 16 * r, blob + d_codes_b + row * (F / 4) + 16 * j);
            cp_async4(dst + Gm::DN_CODES + 4 * r, blob + d_scales_b + (row * NJ + (j & ~1)) * 2);  // scales of groups j&~1, j|1
        }
        cp_async_commit();
    };
    auto pump = [&]() {  // stages being refilled were last accessed through the generic proxy: order before the copies
        if (stalled) return;
        const bool more_gu = gu_issued < gu_known && (UNIT_BOX ? gu_issued + CPT <= gu_done + SGU : gu_issued < gu_done + SGU);
        const bool more_dn = dn_issued < dn_known && dn_issued < dn_done + 1;
        if (more_gu || more_dn) {
            __syncwarp();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (UNIT_BOX) {  // whole units, once every stage is free
                for (; gu_issued < gu_known && gu_issued + CPT <= gu_done + SGU; gu_issued += CPT) issue_gu(gu_issued);
            } else {
                while (gu_issued < gu_known && gu_issued < gu_done + SGU) issue_gu(gu_issued++);
            }
            while (dn_issued < dn_known && dn_issued < dn_done + 1) issue_dn(dn_issued++);
            __syncwarp();
        }
    };
    auto wait_bar = [&](unsigned long long *bar, unsigned parity) -> bool {
        for (unsigned long long i = 0;; ++i) {
            if (mbar_try(bar, parity)) return true;
            if (i > P.spin_limit) return false;
        }
    };
    auto fail_wait = [&]() {  // warp-uniform: callers vote on the wait result
        stalled = true;
        atomicOr(&S.abort_flag, 1);
    };

    pump();  // the shared-expert unit's gate/up chunks: no routing needed

    // ------------------------------------------------------------------ phase 0
    // Router rows: row r on CTA r % G, warp r / G (warps [0, RWARPS)); their weights are
    // requested before x arrives. The other warps build the x operands meanwhile.
    const int RWARPS = min(kWarps, (E + 1 + G - 1) / G);
    const bool router_warp = warp < RWARPS;
    const int row0 = cta + G * warp;
    float wv[2 * NG];
    auto load_row = [&](int r) {
        const float *W = r < E ? L.router + (long long)r * H : L.shared_gate;
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            wv[2 * j] = __ldg(W + 64 * j + lane);
            wv[2 * j + 1] = __ldg(W + 64 * j + 32 + lane);
        }
    };
    if (router_warp && row0 <= E) load_row(row0);
    // Everything above reads only the layer's weights. The launch may overlap the previous
    // kernel on the stream (programmatic dependent launch): wait for it to complete before
    // touching x, the scratch or the arrival counters, and let the next launch get ready.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if ((reinterpret_cast<unsigned long long>(P.x) & 15ull) == 0) {
        const float4 *x4 = reinterpret_cast<const float4 *>(P.x);
        float4 *d4 = reinterpret_cast<float4 *>(S.u.x);
        const int n4 = B * H / 4;
        for (int base = 0; base < n4; base += 8 * kThreads) {  // eight loads in flight per thread
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = base + u * kThreads + tid;
                if (i < n4) v[u] = __ldg(x4 + i);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = base + u * kThreads + tid;
                if (i < n4) d4[i] = v[u];
            }
        }
    } else {
        for (int i = tid; i < B * H; i += kThreads) S.u.x[i] = __ldg(P.x + i);
    }
    __syncthreads();
    if (router_warp) {
        auto store_logit = [&](int r, int t, float v) {
            if (r < E) P.logits[(long long)t * E + r] = L.bias ? __fadd_rn(v, L.bias[r]) : v;
            else P.sg[t] = v;
        };
        for (int r = row0; r <= E; r += G * RWARPS) {
            if (r != row0) load_row(r);
            int t = 0;
            for (; SPLIT && t + 1 < B; t += 2) {  // several tokens: two at a time, four independent chains
                const float *xa = S.u.x + t * H, *xb = xa + H;
                float la = 0.0f, ha = 0.0f, lb = 0.0f, hb = 0.0f;
#pragma unroll
                for (int j = 0; j < NG; ++j) {
                    la = __fadd_rn(la, __fmul_rn(wv[2 * j], xa[64 * j + lane]));
                    ha = __fadd_rn(ha, __fmul_rn(wv[2 * j + 1], xa[64 * j + 32 + lane]));
                    lb = __fadd_rn(lb, __fmul_rn(wv[2 * j], xb[64 * j + lane]));
                    hb = __fadd_rn(hb, __fmul_rn(wv[2 * j + 1], xb[64 * j + 32 + lane]));
                }
                const float va = tree64(la, ha), vb = tree64(lb, hb);
                if (lane == 0) {
                    store_logit(r, t, va);
                    store_logit(r, t + 1, vb);
                }
            }
            for (; t < B; ++t) {
                const float *xv = S.u.x + t * H;
                float lo = 0.0f, hi = 0.0f;
#pragma unroll
                for (int j = 0; j < NG; ++j) {
                    lo = __fadd_rn(lo, __fmul_rn(wv[2 * j], xv[64 * j + lane]));
                    hi = __fadd_rn(hi, __fmul_rn(wv[2 * j + 1], xv[64 * j + 32 + lane]));
                }
                const float v = tree64(lo, hi);
                if (lane == 0) store_logit(r, t, v);
            }
        }
        // the CTA's rows are written: arrive now (routing needs only the logits); the x
        // operands below are built while the grid gathers
        named_sync(kRowsBarrier, 32 * RWARPS);
        if (tid == 0) {
            __threadfence();
            atomicAdd(&P.sync[0], 1u);
        }
    }
    const int xw0 = RWARPS < kWarps ? RWARPS : 0;  // first x-operand warp (all warps, after their rows, if none is free)
    if (warp >= xw0) {
        const int bi = tid - 32 * xw0, nb = kThreads - 32 * xw0;
        for (int t = 0; t < B; ++t) {  // per-token max |x| (NaN ignored, as fmaxf; max is order-free)
            float mx = 0.0f;
            if constexpr (SPLIT) {  // several tokens: 16-byte loads, two chains
                const float4 *x4 = reinterpret_cast<const float4 *>(S.u.x + t * H);
                float m1 = 0.0f;
                for (int e = bi; e < H / 4; e += nb) {
                    const float4 v = x4[e];
                    mx = fmaxf(mx, fmaxf(fabsf(v.x), fabsf(v.y)));
                    m1 = fmaxf(m1, fmaxf(fabsf(v.z), fabsf(v.w)));
                }
                mx = fmaxf(mx, m1);
            } else {
                for (int e = bi; e < H; e += nb) mx = fmaxf(mx, fabsf(S.u.x[t * H + e]));
            }
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
            if (lane == 0) atomicMax(&S.xmax[t], __float_as_uint(mx));
        }
        named_sync(kXBuildBarrier, nb);
        // blocks of 16 elements (token, group, q); B * NG * 4 is a multiple of 32, so whole
        // warps run each iteration and the group-sum shuffles see all four blocks of a group
        // (measured: letting the router warps join through a shared counter cost 0.25 us at
        // one token and saved 0.2 us at eight)
        for (int b = bi; b < B * NG * 4; b += nb) {
            const int t = b / (NG * 4), grp = (b >> 2) % NG, qq = b & 3;
            const int k = scale_exp(__uint_as_float(S.xmax[t]));
            const float mul = pow2f(k);  // exact power of two
            if (grp == 0 && qq == 0) S.xscale[t] = pow2f(-k);
            const float4 *src = reinterpret_cast<const float4 *>(S.u.x + t * H + 64 * grp + 16 * qq);
            int v[16];
            int part = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 f = src[i];
                v[4 * i] = __float2int_rn(f.x * mul);
                v[4 * i + 1] = __float2int_rn(f.y * mul);
                v[4 * i + 2] = __float2int_rn(f.z * mul);
                v[4 * i + 3] = __float2int_rn(f.w * mul);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) part += v[i];
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if (qq == 0) S.xsum[t][grp] = part;
            block_frags(v, &S.xf[(((grp * 2 + 0) * kMaxTokens + t) * 4 + qq) * 3], &S.xf[(((grp * 2 + 1) * kMaxTokens + t) * 4 + qq) * 3]);
        }
    }
    __syncthreads();  // the x operands are complete

    // ------------------------------------------------------------------ unit arithmetic
    // Column tokens of the current unit: token slot ts -> token index.
    int n_cur = 0, slot_cur = 0;
    auto tok_of = [&](int ts) -> int { return slot_cur == 0 ? ts : S.slot_pair[slot_cur][ts] / K; };

    // Gate/up of unit ui: CPT chunks, then silu(gate) * up into S.hid[token slot][64].
    // One copy of the unit code (instruction fetch, not arithmetic, limited the kernel when
    // every column-group count had its own): sized for four column groups, the groups past
    // ncg = ceil(n_cur / 2) are skipped by warp-uniform branches.
    constexpr int NCG = 4;
    auto gate_up = [&](int ui) {
        const int ncg = (n_cur + 1) / 2;
        int tokB[NCG], tokC[NCG];
        const int d = g & 3;
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            const int tsB = 2 * cg + (g >> 2), tsC = 2 * cg + (q >> 1);
            tokB[cg] = d < 3 && tsB < n_cur ? tok_of(tsB) : -1;
            tokC[cg] = tsC < n_cur ? tok_of(tsC) : -1;
        }
        // lane (g, q) finishes row g (even q) or row g + 8 (odd q) of token slot 2 cg + q / 2: the
        // lane pair swaps the digit pieces of the other one's row (one shuffle per group)
        float acc[NCG];
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) acc[cg] = 0.0f;
        const bool odd = q & 1;
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        for (int sub = 0; sub < CPT; ++sub) {
            const int k = ui * CPT + sub, st = k % SGU;
            if (!stalled && (!UNIT_BOX || sub == 0) && !__all_sync(0xffffffffu, wait_bar(&S.bar_gu[warp][st], (k / SGU) & 1))) fail_wait();
            if (!stalled) {
                const unsigned base = smem_u32(S.gu_codes[warp][st]);
                const unsigned short *scl = S.gu_scales[warp][ui & 1] + sub * 8;  // row r: scl[r * NG + group in chunk]
                unsigned w[4][4];
#pragma unroll
                for (int gp = 0; gp < 4; ++gp) {
                    const int c = 2 * gp + (lane >> 4);
                    ldsm_x4(base + r * 128 + ((c ^ (r & 7)) << 4), w[gp][0], w[gp][1], w[gp][2], w[gp][3]);
                }
                // expert scales are finite FP16 (rejected on load otherwise, src/model.js:164): the
                // hardware conversion is exact for them
                float s_row[8];  // this lane's row: one 16-byte load of 8 FP16 scales
                {
                    const uint4 v = *reinterpret_cast<const uint4 *>(scl + (g + (odd ? 8 : 0)) * NG);
                    const unsigned wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wv[i]));
                        s_row[2 * i] = f.x;
                        s_row[2 * i + 1] = f.y;
                    }
                }
                // issue order matters (the MMA and ldmatrix statements keep their order): all
                // operands, then 16 independent MMAs, then the combines
#pragma unroll
                for (int cg = 0; cg < NCG; ++cg) {
                    if (cg >= ncg) break;
                    uint2 bf[8][2];
#pragma unroll
                    for (int gl = 0; gl < 8; ++gl)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            bf[gl][h] = tokB[cg] >= 0 ? S.xf[((((sub * 8 + gl) * 2 + h) * kMaxTokens + tokB[cg]) * 4 + q) * 3 + d] : make_uint2(0u, 0u);
                    int c4[8][4];
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int gl = 0; gl < 8; ++gl) {
                            const unsigned wl = w[gl >> 1][(gl & 1) ? 2 : 0], wh = w[gl >> 1][(gl & 1) ? 3 : 1];
                            imma_acc(h > 0, c4[gl], (wl >> (4 * h)) & 0x03030303u, (wh >> (4 * h)) & 0x03030303u, (wl >> (4 * h + 2)) & 0x03030303u,
                                 (wh >> (4 * h + 2)) & 0x03030303u, bf[gl][h].x, bf[gl][h].y);
                        }
                    const int* xsr = S.xsum[tokC[cg] >= 0 ? tokC[cg] : 0] + sub * 8;
#pragma unroll
                    for (int gl = 0; gl < 8; ++gl) {
                        const int send = odd ? c4[gl][0] : c4[gl][2] + 256 * c4[gl][3];
                        const int recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        const int v = odd ? recv + 65536 * c4[gl][2] : c4[gl][0] + 256 * c4[gl][1] + 65536 * recv;
                        acc[cg] = fmaf(s_row[gl], (float)(v - xsr[gl]), acc[cg]);
                    }
                }
            }
            ++gu_done;
            pump();
        }
        // lane (g, q) holds row g (even q) or g + 8 (odd q) of token slot 2cg + q/2; row g (gate
        // when g is even) pairs with row g+1 (up) four lanes down. Hidden index of row g:
        // 8 warp + g/2 (+4 for row g+8). Each warp also records its largest |hidden| per token
        // slot (NaN ignored, as fmaxf).
        const int buf = ui & 1;
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            if (cg >= ncg) break;
            const float sc = tokC[cg] >= 0 ? S.xscale[tokC[cg]] : 0.0f;
            const float gv = acc[cg] * sc;
            const float up = __shfl_down_sync(0xffffffffu, gv, 4);
            const bool own = !(g & 1) && tokC[cg] >= 0;
            float hv = 0.0f;
            if (own) {
                hv = __fmul_rn(ref_silu(gv), up);
                S.hid[buf][2 * cg + (q >> 1)][8 * warp + (odd ? 4 : 0) + (g >> 1)] = hv;
            }
            float m = fmaxf(0.0f, fabsf(hv));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            if (g == 0 && !(q & 1) && tokC[cg] >= 0) S.hmaxw[buf][warp][2 * cg + (q >> 1)] = m;
        }
    };

    // Down slice of unit ui: rows RW warp .. RW (warp+1), scale group j; adds into y.
    auto down = [&](int ui, int j) {
        const int ncg = (n_cur + 1) / 2;
        // Hidden B fragments, built by each lane for its own column (token slot tsB, digit d):
        // v = round(h * 2^k), k from the slot's largest |h| over the eight warps' maxima. The four
        // q lanes of a column hold the group's 64 elements between them, so their sum(v) is a
        // two-step shuffle; combine lanes (even q, token slot tsC) read it from the lane with
        // g = 4 (q / 2), whose column is that slot.
        const int buf = ui & 1, d = g & 3;
        uint2 hb[NCG][2];
        int tokC[NCG], hsC[NCG], prow[NCG];
        float hmC[NCG];
        const int PP = B * K + B;
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            if (cg >= ncg) break;
            const int tsB = min(2 * cg + (g >> 2), n_cur - 1), tsC = 2 * cg + (q >> 1);
            float mx = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, S.hmaxw[buf][w][tsB]);
            const int k = scale_exp(mx);
            const float mul = pow2f(k);
            int v[16];
            int part = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v[i] = __float2int_rn(S.hid[buf][tsB][16 * q + i] * mul);
                part += v[i];
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            const bool live = d < 3 && 2 * cg + (g >> 2) < n_cur;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int lo[4] = {v[2 * h], v[2 * h + 4], v[2 * h + 8], v[2 * h + 12]};
                const int hi[4] = {v[2 * h + 1], v[2 * h + 5], v[2 * h + 9], v[2 * h + 13]};
                hb[cg][h] = live ? make_uint2(pack_digit(lo, d), pack_digit(hi, d)) : make_uint2(0u, 0u);
            }
            const int src = 16 * (q >> 1) + q;
            hsC[cg] = __shfl_sync(0xffffffffu, part, src);
            const float inv = __shfl_sync(0xffffffffu, pow2f(-k), src);
            tokC[cg] = tsC < n_cur ? tok_of(tsC) : -1;
            prow[cg] = tsC >= n_cur ? 0 : slot_cur == 0 ? B * K + tsC : S.slot_pair[slot_cur][tsC];  // partial row: pair, or shared token
            const float w = tsC >= n_cur ? 0.0f : slot_cur == 0 ? S.sgw[tsC] : S.wts[S.slot_pair[slot_cur][tsC]];
            hmC[cg] = inv * w;
        }
        cp_async_wait_all();  // this lane's copies (the only cp.async group in flight)
        __syncwarp();         // ... and every lane's
        if (!stalled) {
            const unsigned base = smem_u32(S.u.down[warp]);
            const unsigned short *dsc = reinterpret_cast<const unsigned short *>(S.u.down[warp] + Gm::DN_CODES);
            constexpr int MB = 4;  // 16-row tiles per batch: two ldmatrix.x4, then all MMAs, then the epilogues
#pragma unroll 1
            for (int mb = 0; mb < RW / 16; mb += MB) {
                unsigned wt[MB][2];
#pragma unroll
                for (int pp = 0; pp < MB / 2; ++pp)
                    ldsm_x4(base + (16 * (mb + 2 * pp) + 8 * (lane >> 3) + (lane & 7)) * 16, wt[2 * pp][0], wt[2 * pp][1], wt[2 * pp + 1][0],
                            wt[2 * pp + 1][1]);
                float s_lo[MB], s_hi[MB];
#pragma unroll
                for (int m = 0; m < MB; ++m) {
                    const int rl = 16 * (mb + m) + g;
                    s_lo[m] = __half2float(__ushort_as_half(dsc[2 * rl + (j & 1)]));
                    s_hi[m] = __half2float(__ushort_as_half(dsc[2 * (rl + 8) + (j & 1)]));
                }
#pragma unroll
                for (int cg = 0; cg < NCG; ++cg) {
                    if (cg >= ncg) break;
                    int c4[MB][4];
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int m = 0; m < MB; ++m) {
                            const unsigned wl = wt[m][0], wh = wt[m][1];
                            imma_acc(h > 0, c4[m], (wl >> (4 * h)) & 0x03030303u, (wh >> (4 * h)) & 0x03030303u, (wl >> (4 * h + 2)) & 0x03030303u,
                                 (wh >> (4 * h + 2)) & 0x03030303u, hb[cg][h].x, hb[cg][h].y);
                        }
                    float *pr = P.part + ((long long)j * PP + prow[cg]) * H + RW * warp + 16 * mb + g;
                    const bool store = !(q & 1) && tokC[cg] >= 0;
#pragma unroll
                    for (int m = 0; m < MB; ++m) {
                        const int d2lo = __shfl_down_sync(0xffffffffu, c4[m][0], 1), d2hi = __shfl_down_sync(0xffffffffu, c4[m][2], 1);
                        const float flo = (float)(c4[m][0] + 256 * c4[m][1] + 65536 * d2lo - hsC[cg]) * s_lo[m] * hmC[cg];
                        const float fhi = (float)(c4[m][2] + 256 * c4[m][3] + 65536 * d2hi - hsC[cg]) * s_hi[m] * hmC[cg];
                        if (store) {
                            __stcg(pr + 16 * m, flo);
                            __stcg(pr + 16 * m + 8, fhi);
                        }
                    }
                }
            }
        }
        ++dn_done;
        pump();
    };
    // The shared-expert unit's gate/up part runs while the grid arrives.
    const bool early_unit = cta < NJ;
    if (early_unit) {
        slot_cur = 0;
        n_cur = B;
        gate_up(0);
    }

    // ------------------------------------------------------------------ arrival: routing
    // Three or more tokens: routing is split over the last B CTAs (CTA G-1-t routes token t
    // with all eight warps and publishes its ids and weights; a third arrival hands them to
    // every CTA). Fewer tokens: every CTA routes every token itself, which spares the
    // arrival (route_group with 8 or 4 warps per token is as fast as one token on a CTA).
    int n_units = 0;
    if constexpr (SPLIT) {
        if (G - 1 - cta < B) split_route_token<H, F>(P, S, G - 1 - cta);
        split_route_receive<H, F>(P, S);
    } else {
        cta_spin_until(&P.sync[0], (unsigned)G, P.spin_limit, &S.abort_flag);
        if (!S.abort_flag) {
            if ((E & 3) == 0) {
                for (int i = tid; i < B * E / 4; i += kThreads) {
                    const int t = i / (E / 4), e4 = i % (E / 4);
                    reinterpret_cast<float4 *>(S.u.r.lg[t])[e4] = __ldcg(reinterpret_cast<const float4 *>(P.logits) + i);
                }
            } else {
                for (int i = tid; i < B * E; i += kThreads) S.u.r.lg[i / E][i % E] = __ldcg(P.logits + i);
            }
            for (int e = tid; e < E; e += kThreads) {
                S.u.r.owner[e] = 0x7fffffff;
                S.u.r.cnt[e] = 0;
            }
            if (tid < B) {
                S.u.r.nzc[tid] = 0;
                S.sgw[tid] = ref_sigmoid(__ldcg(P.sg + tid));
            }
            __syncthreads();
            const int W = B == 1 ? 8 : B == 2 ? 4 : B <= 4 ? 2 : 1;
            const int t = warp / W;
            if (t < B) {
                float *lg = S.u.r.lg[t];
                float *red = S.u.r.red[t];
                unsigned long long *cand = S.u.r.cand[t];
                float *sel = S.u.r.sel[t];
                int *ids = S.ids + t * K;
                float *wts = S.wts + t * K;
                switch (W) {
                    case 8: route_group<8>(lg, E, K, red, cand, &S.u.r.nzc[t], ids, sel, wts, 1 + t); break;
                    case 4: route_group<4>(lg, E, K, red, cand, &S.u.r.nzc[t], ids, sel, wts, 1 + t); break;
                    case 2: route_group<2>(lg, E, K, red, cand, &S.u.r.nzc[t], ids, sel, wts, 1 + t); break;
                    default: route_group<1>(lg, E, K, red, cand, &S.u.r.nzc[t], ids, sel, wts, 1 + t); break;
                }
            }
            __syncthreads();
            if (cta == 0)
                for (int p = tid; p < B * K; p += kThreads) {
                    P.ids[p] = S.ids[p];
                    P.weights[p] = S.wts[p];
                }
        }
    }
    if (!S.abort_flag) {
        const int P2 = B * K;
        // expert slots in first-appearance order (token-major), as src/prefill.js:56-60; an id
        // outside [0, E) (only when fewer than topK experts have a probability) gets no slot.
        // Pair p = thread p (B * topK <= 256): the lowest pair of an expert opens its slot,
        // slots are numbered by a ballot prefix over pairs; a slot's tokens are listed in
        // arrival order, which only permutes MMA columns within the CTA.
        if (B == 1) {
            // one token: its pairs are its selections in k order and their experts are distinct,
            // so slot s (>= 1) is the s-th valid selection; one thread fills the table
            if (tid == 0) {
                int n = 1;
                for (int k = 0; k < K; ++k) {
                    const int e = S.ids[k];
                    if (e < 0 || e >= E) continue;
                    S.slot_expert[n] = (short)e;
                    S.slot_n[n] = 1;
                    S.slot_pair[n][0] = (short)k;
                    ++n;
                }
                S.n_slots = n;
            }
            __syncthreads();
        } else {
        int pe = -1, prank = 0;
        bool pvalid = false;
        if (tid < P2) {
            pe = S.ids[tid];
            pvalid = pe >= 0 && pe < E;
            if (pvalid) {
                atomicMin(&S.u.r.owner[pe], tid);
                prank = atomicAdd(&S.u.r.cnt[pe], 1);
            }
        }
        __syncthreads();
        const bool pfirst = pvalid && S.u.r.owner[pe] == tid;
        const unsigned bal = __ballot_sync(0xffffffffu, pfirst);
        if (lane == 0) S.u.r.wcount[warp] = __popc(bal);
        __syncthreads();
        if (pfirst) {
            int sidx = 1 + __popc(bal & ((1u << lane) - 1u));
            for (int w = 0; w < warp; ++w) sidx += S.u.r.wcount[w];
            S.slot_expert[sidx] = (short)pe;
            S.slot_n[sidx] = (unsigned char)S.u.r.cnt[pe];
            S.u.r.slot_of[pe] = (short)sidx;
        }
        if (tid == 0) {
            int n = 1;
            for (int w = 0; w < kWarps; ++w) n += S.u.r.wcount[w];
            S.n_slots = n;
        }
        __syncthreads();
        if (pvalid) S.slot_pair[S.u.r.slot_of[pe]][prank] = (short)tid;
        __syncthreads();
        }
        const int NU = S.n_slots * NJ;
        if constexpr (SPLIT) {
            while (unit_index(n_units) < NU) ++n_units;
        } else {
            n_units = cta < NU ? (NU - 1 - cta) / G + 1 : 0;
        }
        gu_known = n_units * CPT;
        dn_known = n_units;
        pump();
    }

    // ------------------------------------------------------------------ units
    for (int ui = 0; ui < n_units; ++ui) {
        int slot, j, m, e;
        unit_of(ui, slot, j, m, e);
        slot_cur = slot;
        n_cur = slot == 0 ? B : S.slot_n[slot];
        if (!(ui == 0 && early_unit)) gate_up(ui);
        if (__syncthreads_or(stalled ? 1 : 0)) break;  // a warp's copies timed out: all leave together
        down(ui, j);
    }

    // ------------------------------------------------------------------ second arrival: y
    for (int k = gu_done; k < gu_issued; ++k)
        if (!UNIT_BOX || k % SGU == 0) wait_bar(&S.bar_gu[warp][k % SGU], (k / SGU) & 1);
    cp_async_wait_all();
    if (stalled) atomicOr(&S.abort_flag, 1);
    __syncthreads();
    if (tid == 0 && !grid_arrive_wait(&P.sync[1], (unsigned)G, P.spin_limit)) S.abort_flag = 1;
    __syncthreads();
    if (!S.abort_flag) {
        // y[t][r]: the terms of one float4 column (group j, then the shared expert and the
        // routed pairs in selection order: NJ (K + 1) of them) are split over a warp's lanes
        // (lane l adds terms l, l + 32, ...; a pair without an expert adds zero), then summed
        // by a fixed shuffle tree: the order never changes, so y has the same bits every run.
        const int PP = B * K + B, H4 = H / 4, NT = NJ * (K + 1);
        const float4 *part4 = reinterpret_cast<const float4 *>(P.part);
        // Several tokens: NB items of a warp at once (their loads all in flight; each item's
        // additions in the same order as one at a time).
        constexpr int NB = SPLIT ? 4 : 1;
        const int stride = G * kWarps;
        for (int item0 = cta * kWarps + warp; item0 < B * H4; item0 += NB * stride) {
            float4 acc[NB];
#pragma unroll
            for (int n = 0; n < NB; ++n) acc[n] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int m0 = 0; m0 < NT; m0 += 96) {  // three terms per lane: their loads are all in flight before the adds
                float4 u[NB][3];
#pragma unroll
                for (int n = 0; n < NB; ++n) {
                    const int item = item0 + n * stride, t = min(item / H4, B - 1), c = item % H4;  // t clamped: past the end, nothing is read
#pragma unroll
                    for (int v = 0; v < 3; ++v) {
                        const int m = m0 + lane + 32 * v;
                        const int jj = m / (K + 1), kk = m % (K + 1);  // kk == 0: shared expert, else routed pair kk - 1
                        const int row = kk == 0 ? B * K + t : t * K + kk - 1;
                        const bool ok = item < B * H4 && m < NT && (kk == 0 || (unsigned)S.ids[t * K + kk - 1] < (unsigned)E);
                        u[n][v] = ok ? __ldcg(part4 + ((long long)jj * PP + row) * H4 + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
                }
#pragma unroll
                for (int n = 0; n < NB; ++n)
#pragma unroll
                    for (int v = 0; v < 3; ++v) {
                        acc[n].x += u[n][v].x;
                        acc[n].y += u[n][v].y;
                        acc[n].z += u[n][v].z;
                        acc[n].w += u[n][v].w;
                    }
            }
#pragma unroll
            for (int n = 0; n < NB; ++n) {
#pragma unroll
                for (int sft = 16; sft > 0; sft >>= 1) {
                    acc[n].x += __shfl_xor_sync(0xffffffffu, acc[n].x, sft);
                    acc[n].y += __shfl_xor_sync(0xffffffffu, acc[n].y, sft);
                    acc[n].z += __shfl_xor_sync(0xffffffffu, acc[n].z, sft);
                    acc[n].w += __shfl_xor_sync(0xffffffffu, acc[n].w, sft);
                }
                const int item = item0 + n * stride;
                if (lane == 0 && item < B * H4) reinterpret_cast<float4 *>(P.y)[item] = acc[n];
            }
        }
    }

    // ------------------------------------------------------------------ exit
    __syncthreads();
    if (tid == 0) {
        if (S.abort_flag) raise_error(P.err, kErrWaitTimeout);
        __threadfence();
        const unsigned prev = atomicAdd(&P.sync[2], 1u);
        if (prev == (unsigned)G - 1) {  // last CTA out resets the arrival counters for the next launch
            P.sync[0] = 0;
            P.sync[1] = 0;
            if constexpr (SPLIT) P.sync[3] = 0;
            __threadfence();
            P.sync[2] = 0;
        }
    }
}

}  // namespace fast

static int g_fast_pdl = -1;  // programmatic dependent launch with the cooperative launch: -1 untried, 1 accepted, 0 refused
int moe_fast_pdl_state() { return g_fast_pdl; }

size_t moe_fast_scratch_bytes(int tokens, int width, int ff, int experts, int topK) {
    auto a = [](size_t n) { return (n + 255) & ~size_t(255); };
    return a(sizeof(float) * tokens * experts) + a(sizeof(float) * tokens) +
           a(sizeof(float) * (size_t)(ff / 64) * (size_t)(tokens * topK + tokens) * width);
}

bool moe_fast_supported(int tokens, int width, int ff, int topK, int grid) {
    return tokens >= 1 && tokens <= fast::kMaxTokens && topK >= 1 && topK <= 32 && grid >= 1 &&
           ((width == 2048 && ff == 512) || (width == 2560 && ff == 640));
}

namespace {

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

bool map3d(CUtensorMap *m, const void *base, unsigned long long d0, unsigned long long d1, unsigned long long d2,
           unsigned long long s1, unsigned long long s2, unsigned b0, unsigned b1, CUtensorMapSwizzle sw, CUtensorMapL2promotion l2) {
    auto fn = encoder();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Gate/up codes as {128-byte chunk, rows, chunks, experts} (strides: row H/4, chunk 128, blob):
// one box {128, 16, CH, 1} copies 16 whole rows in one request and lays them out chunk-major,
// [chunk][row][128 B] with the 128-byte swizzle, as CH separate {128, 16} boxes would. Measured
// on B200 (all SMs streaming 8 KB tiles): 60 GB/s per SM, against 24 GB/s for four {128, 16}
// boxes of the same rows.
bool map_gu_rows(CUtensorMap *m, const void *base, unsigned long long H, unsigned long long F, unsigned long long ne,
                 unsigned long long blob_bytes) {
    auto fn = encoder();
    if (!fn) return false;
    cuuint64_t dims[4] = {128, 2 * F, H / 512, ne}, strides[3] = {H / 4, 128, blob_bytes};
    cuuint32_t box[4] = {128, 16, (cuuint32_t)(H / 512), 1}, es[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encoded maps of the last layers used, keyed by their blob addresses.
struct MapSet {
    const void *blobs, *shared;
    int width, ff, experts;
    CUtensorMap gu[2];
    MoeMaps all;  // the maps of the medium-batch layer
};
std::mutex g_map_mutex;
MapSet g_maps[64];
int g_map_next = 0;

// gu2 receives the two gate/up maps, all (nullable) the medium-batch layer's maps.
bool layer_maps(const MoeLayerDev &L, CUtensorMap *gu2, MoeMaps *all) {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    auto use = [&](const MapSet &m) {
        std::memcpy(gu2, m.gu, sizeof m.gu);
        if (all) *all = m.all;
    };
    for (const MapSet &m : g_maps)
        if (m.blobs == L.blobs && m.shared == L.shared_blob && m.width == L.width && m.ff == L.ff && m.experts == L.experts) {
            use(m);
            return true;
        }
    MapSet m;
    m.blobs = L.blobs;
    m.shared = L.shared_blob;
    m.width = L.width;
    m.ff = L.ff;
    m.experts = L.experts;
    const long long H = L.width, F = L.ff, bb = L.blob_words * 4;
    for (int i = 0; i < 2; ++i) {
        const unsigned char *base = reinterpret_cast<const unsigned char *>(i == 0 ? L.blobs : L.shared_blob);
        const unsigned long long ne = i == 0 ? (unsigned long long)L.experts : 1ull;
        if (!map3d(&m.gu[i], base, H / 4, 2 * F, ne, H / 4, bb, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return false;
        // the medium-batch layer copies 128 rows at a time (one box per CTA step)
        if (!map3d(&m.all.gu[i], base, H / 4, 2 * F, ne, H / 4, bb, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return false;
        // gate/up scales {2 NG bytes, 2F rows}, box {16 bytes = 8 groups, 128 rows}
        if (!map3d(&m.all.gs[i], base + 3 * F * H / 4, H / 32, 2 * F, ne, H / 32, bb, 16, 128, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE))
            return false;
        // down codes {F/4 bytes, H rows}, box {F/4, 128 rows}: 128-byte swizzle for 128-byte rows
        if (!map3d(&m.all.dc[i], base + 2 * F * H / 4, F / 4, H, ne, F / 4, bb, F / 4, 128,
                   F / 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return false;
        if (!map_gu_rows(&m.all.gu16r[i], base, H, F, ne, bb)) return false;
        if (!map3d(&m.all.dn64[i], base + 2 * F * H / 4, F / 4, H, ne, F / 4, bb, F / 4, 64,
                   F / 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return false;
        // the same in boxes of 16 rows (one-token decode: a CTA's 16 output rows of one expert)
        if (!map3d(&m.all.dn16[i], base + 2 * F * H / 4, F / 4, H, ne, F / 4, bb, F / 4, 16,
                   F / 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return false;
    }
    g_maps[g_map_next] = m;
    g_map_next = (g_map_next + 1) % 64;
    use(m);
    return true;
}

}  // namespace

bool moe_tensor_maps(const MoeLayerDev &L, MoeMaps *maps) {
    CUtensorMap gu[2];
    return layer_maps(L, gu, maps);
}

bool moe_decode_maps(const MoeLayerDev &L, CUtensorMap *gu16, MoeMaps *maps) { return layer_maps(L, gu16, maps); }

namespace {

// Cooperative (the grid arrivals need every CTA resident) and, where the runtime accepts the
// combination, programmatic stream serialisation: the launch is prepared while the previous
// kernel on the stream finishes; the kernel reads only weights before griddepcontrol.wait.
template <int H, int F, bool SPLIT>
cudaError_t launch_fast_as(const fast::Params &p, int grid, cudaStream_t s) {
    const size_t smem = sizeof(fast::Smem<H, F>) + 1024;  // + slack for the 1024-byte stage alignment
    static int device_ready = -1;  // device whose attribute is set (the library drives one device per context)
    int dev = 0;
    STRATA_CUDA_TRY(cudaGetDevice(&dev));
    if (device_ready != dev) {
        STRATA_CUDA_TRY(cudaFuncSetAttribute(fast::k_moe_fast<H, F, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        device_ready = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(fast::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (g_fast_pdl < 0) {  // STRATA_FAST_PDL=0 launches without programmatic dependent launch
        const char *env = std::getenv("STRATA_FAST_PDL");
        if (env && env[0] == '0') g_fast_pdl = 0;
    }
    if (g_fast_pdl != 0) {
        cfg.numAttrs = 2;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, fast::k_moe_fast<H, F, SPLIT>, p);
        if (e == cudaSuccess || g_fast_pdl == 1) {
            g_fast_pdl = e == cudaSuccess ? 1 : g_fast_pdl;
            return e;
        }
        cudaGetLastError();  // refused: launch without it from now on
        g_fast_pdl = 0;
    }
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fast::k_moe_fast<H, F, SPLIT>, p);
}

// Split routing from kSplitRouteTokens tokens on, when the grid has a CTA per token beyond
// the shared-expert units' CTAs.
template <int H, int F>
cudaError_t launch_fast(const fast::Params &p, int grid, cudaStream_t s) {
    if (p.tokens >= fast::kSplitRouteTokens && grid >= F / 64 + p.tokens) return launch_fast_as<H, F, true>(p, grid, s);
    return launch_fast_as<H, F, false>(p, grid, s);
}

}  // namespace

cudaError_t moe_forward_fast(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights, void *scratch,
                             unsigned *sync, int grid, cudaStream_t s, unsigned *err) {
    char *p = static_cast<char *>(scratch);
    auto a = [](size_t n) { return (n + 255) & ~size_t(255); };
    fast::Params prm;
    std::memset(&prm, 0, sizeof prm);
    prm.L = L;
    prm.x = x;
    prm.tokens = tokens;
    prm.y = y;
    prm.ids = ids;
    prm.weights = weights;
    prm.logits = reinterpret_cast<float *>(p);
    p += a(sizeof(float) * tokens * L.experts);
    prm.sg = reinterpret_cast<float *>(p);
    p += a(sizeof(float) * tokens);
    prm.part = reinterpret_cast<float *>(p);
    prm.sync = sync;
    prm.err = err;
    prm.spin_limit = 1ull << 20;  // grid waits sleep 32 ns per try; an mbarrier try suspends for a short, system-defined time
    MoeMaps all;
    if (!layer_maps(L, prm.tm_gu, &all)) return cudaErrorInvalidValue;
    prm.tm_gu4[0] = all.gu16r[0];
    prm.tm_gu4[1] = all.gu16r[1];
    if (L.width == 2048 && L.ff == 512) return launch_fast<2048, 512>(prm, grid, s);
    if (L.width == 2560 && L.ff == 640) return launch_fast<2560, 640>(prm, grid, s);
    return cudaErrorInvalidValue;
}

}  // namespace strata
