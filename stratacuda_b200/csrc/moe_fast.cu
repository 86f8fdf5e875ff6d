// Fast fused mixture-of-experts layer for decode batches (tokens <= 8): ONE persistent
// cooperative launch, one CTA per SM, 8 warps.
//
// Phase 0 (no routing needed yet)
//   * router logits: row r of the 512 (+1 shared-gate row) goes to CTA r % G, warp r / G,
//     in the reference's exact order (kernels/strata.cu:156-165), so the routing below is
//     bit-identical to the reference;
//   * every CTA turns the activations into integer tensor-core operands (below) and zeroes
//     its slice of y;
//   * the shared expert's gate/up tiles need no routing: their copies are issued at entry
//     and computed while the grid arrives at barrier A.
// Phase 1 (after arrival A: all logits written)
//   * every CTA routes all tokens redundantly (one warp per token, route.cuh) and builds the
//     expert slots in shared memory, so the routing needs no grid barrier of its own;
//   * gate/up tiles of the routed experts (16 interleaved gate/up rows x full width): the
//     hidden values silu(g)*u go to global memory.
// Phase 2 (after arrival B: all hidden values written)
//   * down tiles (16 output rows of one expert), contiguous per CTA; results times the
//     routing weight (sigmoid of the shared-gate logit for the shared expert) are added into
//     y with atomics, so y is not bit-reproducible run to run (order of the adds); it stays
//     within 1e-5 relative L2 of the reference (tested).
//
// Memory pipeline: each warp owns kStages shared-memory stages. Chunks move by TMA tensor
// copies (cp.async.bulk.tensor): a gate/up chunk is one 16-row x 128-byte box of codes
// (8 scale groups, 128B swizzle) plus one 16 x 16-byte box of FP16 scales; a down tile is
// one 16 x 128-byte box (ff 512, 128B swizzle) or five 16 x 32-byte boxes (ff 640, 32B
// swizzle) plus one bulk copy of its scales. The swizzles make ldmatrix conflict-free.
//
// Tensor-core math (exact integer products): mma.sync m16n8k32 u8 x s8 -> s32.
//   A = weight codes c in {0..3} as u8: four codes per register by one shift and one mask.
//   B = activations as three signed 8-bit digits: v = round(x * 2^k) (k per token, |v| <
//       2^22), v = d0 + 256 d1 + 65536 d2; one MMA column per token, one MMA per digit.
//   Per 64-group: sum((c-1) x) * 2^k = (acc0 + 256 acc1 + 65536 acc2) - sum(v), exact in
//   int32; then total += scale * float(that) in F32, and the row is multiplied by 2^-k.
// The only rounding is v (2^-22 of the token's largest |x|) and the F32 accumulation.
//
// All waits (grid arrivals, mbarriers) are bounded: past the limit the kernel records
// kErrWaitTimeout, waits (bounded) for its own copies in flight and leaves.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "route.cuh"

namespace strata {
namespace fast {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;         // per warp
constexpr int kStageBytes = 3072;  // 1024-aligned; >= 16 x ff/4 + 32 x ff/64 (ff <= 640)
constexpr int kMaxTokens = 8;
constexpr int kMaxPairs = kMaxTokens * 32;
constexpr int kDigits = 3;

__device__ __forceinline__ unsigned smem_u32(const void *p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(unsigned long long *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect(unsigned long long *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned long long *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(2000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, unsigned bytes, unsigned long long *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_3d(void *dst, const CUtensorMap *map, int x, int y, int z, unsigned long long *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned &r0, unsigned &r1, unsigned &r2, unsigned &r3) {
    asm volatile("ldmatrix.sync.aligned.x4.m8n8.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void imma(int (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Element e (0..63) of a 64-group in the B-fragment layout of MMA h: register b0 byte i holds
// element 16q + 2h + 4i, register b1 byte i holds element 16q + 2h + 1 + 4i. (A register
// (w >> (4h)) & 0x03030303 of word q holds codes 2h + 4i; (w >> (4h+2)) & ... codes 2h+1+4i.)
__device__ __forceinline__ void frag_pos(int e, int &h, int &q, int &byte) {
    q = e >> 4;
    const int r = e & 15;
    h = (r >> 1) & 1;
    byte = (r & 1) * 4 + (r >> 2);
}
// Signed 24-bit value as three signed 8-bit digits d0 + 256 d1 + 65536 d2.
__device__ __forceinline__ void digits(int v, int &d0, int &d1, int &d2) {
    d0 = ((v + 128) & 255) - 128;
    const int v1 = (v - d0) >> 8;
    d1 = ((v1 + 128) & 255) - 128;
    d2 = (v1 - d1) >> 8;
}
// Scale exponent: 2^k * maxabs < 2^22.
__device__ __forceinline__ int scale_exp(float maxabs) {
    if (!(maxabs > 0.0f) || !isfinite(maxabs)) return 0;
    int e;
    frexpf(maxabs, &e);  // maxabs = m * 2^e, m in [0.5, 1)
    return 22 - e;
}

struct Params {
    MoeLayerDev L;
    const float *x;
    int tokens;
    float *y;
    int *ids;
    float *weights;
    float *logits;   // [tokens][experts]
    float *sg;       // [tokens]
    float *hbuf;     // [(tokens*topK + tokens)][ff] hidden values
    unsigned *sync;  // arrive A, arrive B, exit count
    unsigned *err;
    unsigned long long spin_limit;
    // TMA maps: [0] routed experts, [1] the shared expert
    CUtensorMap tm_gu[2];  // gate/up codes: {H/4 bytes, 2F rows, experts}, box {128, 16, 1}, 128B swizzle
    CUtensorMap tm_gs[2];  // gate/up scales: {2*H/64 bytes, 2F rows, experts}, box {16, 16, 1}
    CUtensorMap tm_dc[2];  // down codes: {F/4 bytes, H rows, experts}, box {128|32, 16, 1}, 128B|32B swizzle
};

template <int NG, int NGD>
struct Smem {
    unsigned char stages[kWarps][kStages][kStageBytes];  // 1024-aligned
    unsigned long long bars[kWarps][kStages];
    // B fragments: x as [NG][2 h][3 d][8 token][4 q], later hidden as [NGD][2 h][3 d][16 = 2 slots x 8][4 q]
    uint2 bfrag[(NG * 2 * kDigits * 8 * 4) > (NGD * 2 * kDigits * 16 * 4) ? (NG * 2 * kDigits * 8 * 4) : (NGD * 2 * kDigits * 16 * 4)];
    int xsum[kMaxTokens][NG];
    float xscale[kMaxTokens];
    int hsum[2][kMaxTokens][NGD];
    float hscale[2][kMaxTokens];
    float hs_weight[2][kMaxTokens];
    int hs_token[2][kMaxTokens];
    int hs_pos[2][kMaxTokens];
    int hs_n[2];
    int ids[kMaxPairs];
    float wts[kMaxPairs];
    float sel[kWarps][32];
    alignas(16) float lg[kWarps][512];  // filled with 16-byte vector stores
    unsigned char first[kMaxPairs];
    unsigned char rank[kMaxPairs];
    short slot_of_pair[kMaxPairs];
    short slot_expert[kMaxPairs];
    short slot_pairs[kMaxPairs][kMaxTokens];
    int slot_n[kMaxPairs];
    short pos_tab[kMaxPairs][kMaxTokens];
    int n_slots;
    int abort_flag;
};

// One warp: 3-digit B fragments + 64-group sums + scale 2^-k of one vector of GROUPS*64
// values into column `col` of a fragment table with `cols` columns. Every lane first loads
// all of its values (independent loads, one memory latency), then converts in registers.
template <int GROUPS>
__device__ __forceinline__ void vector_to_frags(const float *__restrict__ v, uint2 *frag, int cols, int col, int *gsum, float *scale_out,
                                                int lane) {
    float val[2 * GROUPS];
#pragma unroll
    for (int i = 0; i < 2 * GROUPS; ++i) val[i] = __ldcg(v + 32 * i + lane);  // element 32 i + lane
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 2 * GROUPS; ++i) mx = fmaxf(mx, fabsf(val[i]));
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
    const int k = scale_exp(mx);
    const float mul = ldexpf(1.0f, k);  // exact power of two
    if (lane == 0) *scale_out = ldexpf(1.0f, -k);
    unsigned char *fb = reinterpret_cast<unsigned char *>(frag);
#pragma unroll
    for (int grp = 0; grp < GROUPS; ++grp) {
        int part = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int e = half * 32 + lane;
            const int iv = __float2int_rn(val[2 * grp + half] * mul);
            part += iv;
            int d0, d1, d2;
            digits(iv, d0, d1, d2);
            int h, q, byte;
            frag_pos(e, h, q, byte);
            const int base = (((grp * 2 + h) * kDigits) * cols + col) * 4 + q;  // digit 0 entry
            fb[(base)*8 + byte] = (unsigned char)(d0 & 255);
            fb[(base + cols * 4) * 8 + byte] = (unsigned char)(d1 & 255);
            fb[(base + 2 * cols * 4) * 8 + byte] = (unsigned char)(d2 & 255);
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) part += __shfl_xor_sync(0xffffffffu, part, s);
        if (lane == 0) gsum[grp] = part;
    }
}

// Groups [grp0, grp0 + NGROUPS) of one 16-row tile in the stage at shared address `base`:
// rows g and g+8 of this thread, columns (tokens) 2q and 2q+1. colsum[col * sum_stride + grp]
// is a column's integer group sum; scales[row * scale_stride + local group] the FP16 scales.
// SW128: codes in one 16 x 128-byte box with 128-byte swizzle; else 16 x 32-byte boxes of
// two groups each with 32-byte swizzle.
template <int NGROUPS, bool SW128>
__device__ __forceinline__ void tile_math(unsigned base, int lane, const uint2 *__restrict__ bfrag, int cols, int colbase, int grp0,
                                          const int *__restrict__ colsum, int sum_stride, const unsigned short *__restrict__ scales,
                                          int scale_stride, float (&acc)[2][2]) {
    const int g = lane >> 2, q = lane & 3;
    const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
    unsigned w[NGROUPS / 2][4];
#pragma unroll
    for (int gp = 0; gp < NGROUPS / 2; ++gp) {
        const int c = 2 * gp + (lane >> 4);  // group of this lane's ldmatrix row address
        const unsigned addr = SW128 ? base + r * 128 + ((c ^ (r & 7)) << 4) : base + gp * 512 + r * 32 + (((c & 1) ^ ((r >> 2) & 1)) << 4);
        ldsm_x4(addr, w[gp][0], w[gp][1], w[gp][2], w[gp][3]);
    }
#pragma unroll
    for (int gl = 0; gl < NGROUPS; ++gl) {
        const unsigned wl = w[gl >> 1][(gl & 1) ? 2 : 0], wh = w[gl >> 1][(gl & 1) ? 3 : 1];
        const int grp = grp0 + gl;
        int d[kDigits][4];
#pragma unroll
        for (int dd = 0; dd < kDigits; ++dd) d[dd][0] = d[dd][1] = d[dd][2] = d[dd][3] = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const unsigned a0 = (wl >> (4 * h)) & 0x03030303u, a1 = (wh >> (4 * h)) & 0x03030303u;
            const unsigned a2 = (wl >> (4 * h + 2)) & 0x03030303u, a3 = (wh >> (4 * h + 2)) & 0x03030303u;
#pragma unroll
            for (int dd = 0; dd < kDigits; ++dd) {
                const uint2 b = bfrag[(((grp * 2 + h) * kDigits + dd) * cols + colbase + g) * 4 + q];
                imma(d[dd], a0, a1, a2, a3, b.x, b.y);
            }
        }
        // expert scales are finite FP16 (rejected on load otherwise, src/model.js:164): the
        // hardware conversion is exact for them
        const float s_lo = __half2float(__ushort_as_half(scales[g * scale_stride + gl]));
        const float s_hi = __half2float(__ushort_as_half(scales[(g + 8) * scale_stride + gl]));
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int xs = colsum[(2 * q + cc) * sum_stride + grp];
            const int vlo = d[0][cc] + 256 * d[1][cc] + 65536 * d[2][cc] - xs;
            const int vhi = d[0][2 + cc] + 256 * d[1][2 + cc] + 65536 * d[2][2 + cc] - xs;
            acc[0][cc] = fmaf(s_lo, (float)vlo, acc[0][cc]);
            acc[1][cc] = fmaf(s_hi, (float)vhi, acc[1][cc]);
        }
    }
}

template <int NG, int NGD>
__global__ void __launch_bounds__(kThreads, 1) k_moe_fast(const __grid_constant__ Params P) {
    extern __shared__ unsigned char smem_raw[];
    auto &S = *reinterpret_cast<Smem<NG, NGD> *>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
    const MoeLayerDev &L = P.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const int G = gridDim.x, cta = blockIdx.x;
    const int B = P.tokens, K = L.topK, E = L.experts, H = L.width, F = L.ff;
    const int TS = F / 8;    // gate/up tiles per expert (16 blob rows each)
    const int CT = H / 16;   // down tiles per expert (16 output rows each)
    const int CPT = NG / 8;  // chunks per gate/up tile
    constexpr bool kDownSw128 = NGD == 8;  // ff 512: one 128-byte box; ff 640: five 32-byte boxes
    const long long d_scales_b = 3LL * F * H / 4 + 2LL * F * (H / 64) * 2;

    if (tid == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int s = 0; s < kStages; ++s) mbar_init(&S.bars[w][s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
        S.n_slots = 0;
    }
    __syncthreads();

    // ---------------------------------------------------------------- chunk list of this warp
    // gate/up tiles of this CTA: shared tiles j with j % G == cta, then routed tiles i with
    // i % G == G-1-cta (reverse order balances the two lists); warp w takes elements w, w+8...
    // Down tiles: a contiguous range of the slot-major list; warp w takes w, w+8, ...
    const int ns_cta = cta < TS ? (TS - 1 - cta) / G + 1 : 0;
    auto routed_count = [&](int U) {
        const int total = U * TS, first = G - 1 - cta;
        return total > first ? (total - 1 - first) / G + 1 : 0;
    };
    auto warp_count = [&](int n) { return n > warp ? (n - 1 - warp) / kWarps + 1 : 0; };
    int known_chunks = warp_count(ns_cta) * CPT;
    int n_gu_chunks = known_chunks;
    int down_first = 0, down_count = 0;
    auto chunk_of = [&](int k, int &kind, int &slot, int &tile, int &sub) {
        if (k < n_gu_chunks) {
            kind = 0;
            const int e = warp + kWarps * (k / CPT);
            sub = k % CPT;
            if (e < ns_cta) {
                slot = 0;
                tile = cta + e * G;
            } else {
                const int i = (G - 1 - cta) + (e - ns_cta) * G;
                slot = 1 + i / TS;
                tile = i % TS;
            }
        } else {
            kind = 1;
            const int d = down_first + warp + kWarps * (k - n_gu_chunks);
            slot = d / CT;
            tile = d % CT;
            sub = 0;
        }
    };
    int issued = 0, consumed = 0;
    auto issue = [&](int k) {
        int kind, slot, tile, sub;
        chunk_of(k, kind, slot, tile, sub);
        const int st = k % kStages;
        unsigned char *dst = S.stages[warp][st];
        unsigned long long *bar = &S.bars[warp][st];
        const int m = slot == 0 ? 1 : 0;
        const int e = slot == 0 ? 0 : S.slot_expert[slot - 1];
        if (lane == 0) {
            if (kind == 0) {
                mbar_expect(bar, 2048 + 256);
                tma_3d(dst, &P.tm_gu[m], 128 * sub, 16 * tile, e, bar);
                tma_3d(dst + 2048, &P.tm_gs[m], 16 * sub, 16 * tile, e, bar);
            } else {
                mbar_expect(bar, 16 * (F / 4) + 32 * NGD);
                if (kDownSw128) {
                    tma_3d(dst, &P.tm_dc[m], 0, 16 * tile, e, bar);
                } else {
#pragma unroll
                    for (int i = 0; i < NGD / 2; ++i) tma_3d(dst + 512 * i, &P.tm_dc[m], 32 * i, 16 * tile, e, bar);
                }
                const unsigned char *blob =
                    reinterpret_cast<const unsigned char *>(slot == 0 ? L.shared_blob : L.blobs + (long long)e * L.blob_words);
                bulk_copy(dst + 16 * (F / 4), blob + d_scales_b + 16LL * tile * (NGD * 2), 32 * NGD, bar);
            }
        }
    };
    auto pump = [&]() {  // stages being refilled were last read through the generic proxy: order before the copies
        if (issued < known_chunks && issued < consumed + kStages) {
            __syncwarp();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            while (issued < known_chunks && issued < consumed + kStages) issue(issued++);
            __syncwarp();
        }
    };
    auto wait_chunk = [&](int k) -> bool {
        unsigned long long *bar = &S.bars[warp][k % kStages];
        const unsigned parity = (k / kStages) & 1;
        for (unsigned long long i = 0;; ++i) {
            if (mbar_try(bar, parity)) return true;
            if (i > P.spin_limit) return false;
        }
    };
    auto drain = [&]() {
        for (int k = consumed; k < issued; ++k) wait_chunk(k);
        consumed = issued;
    };
    auto grid_wait = [&](unsigned *counter) -> bool {
        for (unsigned long long i = 0;; ++i) {
            if (ld_acquire(counter) >= (unsigned)G) return true;
            if (i > P.spin_limit) return false;
            __nanosleep(64);
        }
    };

    pump();  // shared-expert gate/up chunks: no routing needed

    // ---------------------------------------------------------------- phase 0
    for (int r = cta + G * warp; r < E + 1; r += G * kWarps) {
        const float *W = r < E ? L.router + (long long)r * H : L.shared_gate;
        float wv[2 * NG];
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            wv[2 * j] = __ldg(W + 64 * j + lane);
            wv[2 * j + 1] = __ldg(W + 64 * j + 32 + lane);
        }
        for (int t = 0; t < B; ++t) {
            const float *xv = P.x + (long long)t * H;
            float lo = 0.0f, hi = 0.0f;
#pragma unroll
            for (int j = 0; j < NG; ++j) {
                lo = __fadd_rn(lo, __fmul_rn(wv[2 * j], __ldg(xv + 64 * j + lane)));
                hi = __fadd_rn(hi, __fmul_rn(wv[2 * j + 1], __ldg(xv + 64 * j + 32 + lane)));
            }
            const float v = tree64(lo, hi);
            if (lane == 0) {
                if (r < E) P.logits[(long long)t * E + r] = L.bias ? __fadd_rn(v, L.bias[r]) : v;
                else P.sg[t] = v;
            }
        }
    }
    if (warp < B) vector_to_frags<NG>(P.x + (long long)warp * H, S.bfrag, 8, warp, S.xsum[warp], &S.xscale[warp], lane);
    for (long long i = (long long)cta * kThreads + tid; i < (long long)B * H; i += (long long)G * kThreads) P.y[i] = 0.0f;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&P.sync[0], 1u);
    }

    float acc_t[2][2];
    auto gate_up_chunk = [&](int k) {
        int kind, slot, tile, sub;
        chunk_of(k, kind, slot, tile, sub);
        const unsigned char *st = S.stages[warp][k % kStages];
        if (sub == 0) acc_t[0][0] = acc_t[0][1] = acc_t[1][0] = acc_t[1][1] = 0.0f;
        tile_math<8, true>(smem_u32(st), lane, S.bfrag, 8, 0, sub * 8, &S.xsum[0][0], NG, reinterpret_cast<const unsigned short *>(st + 2048), 8,
                           acc_t);
        if (sub != CPT - 1) return;
        // epilogue: row g (gate if g even) pairs with row g+1 (up); tokens 2q, 2q+1
        const int pair_a = g >> 1;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int t = 2 * q + cc;
            const float sc = t < B ? S.xscale[t] : 0.0f;
            const float gv0 = acc_t[0][cc] * sc, gv1 = acc_t[1][cc] * sc;
            const float up0 = __shfl_down_sync(0xffffffffu, gv0, 4), up1 = __shfl_down_sync(0xffffffffu, gv1, 4);
            int pos = -1;
            if (t < B) pos = slot == 0 ? B * K + t : S.pos_tab[slot - 1][t];
            if (!(g & 1) && pos >= 0) {
                float *hrow = P.hbuf + (long long)pos * F + 8 * tile;
                hrow[pair_a] = __fmul_rn(ref_silu(gv0), up0);
                hrow[pair_a + 4] = __fmul_rn(ref_silu(gv1), up1);
            }
        }
    };

    while (consumed < n_gu_chunks) {
        if (!wait_chunk(consumed)) { atomicOr(&S.abort_flag, 1); break; }
        gate_up_chunk(consumed);
        ++consumed;
        pump();
    }

    // ---------------------------------------------------------------- arrival A: routing
    if (tid == 0 && !grid_wait(&P.sync[0])) S.abort_flag = 1;
    __syncthreads();
    const int P2 = B * K;
    if (!S.abort_flag) {
        if (warp < B) {
            if ((E & 3) == 0) {
                const float4 *src = reinterpret_cast<const float4 *>(P.logits + (long long)warp * E);
                float4 *dst = reinterpret_cast<float4 *>(S.lg[warp]);
#pragma unroll 4
                for (int i = lane; i < E / 4; i += 32) dst[i] = __ldcg(src + i);
            } else {
                for (int e = lane; e < E; e += 32) S.lg[warp][e] = __ldcg(P.logits + (long long)warp * E + e);
            }
            __syncwarp();
            route_warp(S.lg[warp], E, K, S.ids + warp * K, S.wts + warp * K, S.sel[warp]);
            __syncwarp();
            if (cta == 0)
                for (int k = lane; k < K; k += 32) {
                    P.ids[warp * K + k] = S.ids[warp * K + k];
                    P.weights[warp * K + k] = S.wts[warp * K + k];
                }
        }
        __syncthreads();
        // expert slots in first-appearance order (token-major), as src/prefill.js:56-60
        for (int p = tid; p < P2; p += kThreads) {
            const int e = S.ids[p];
            int rank = 0;
            for (int r = 0; r < p; ++r) rank += S.ids[r] == e;
            S.first[p] = rank == 0;
            S.rank[p] = (unsigned char)rank;
        }
        __syncthreads();
        for (int p = tid; p < P2; p += kThreads) {
            if (S.first[p]) {
                int s = 0;
                for (int r = 0; r < p; ++r) s += S.first[r];
                S.slot_of_pair[p] = (short)s;
                S.slot_expert[s] = (short)S.ids[p];
                S.slot_n[s] = 0;
                for (int t = 0; t < kMaxTokens; ++t) S.pos_tab[s][t] = -1;
            }
            if (p == 0) {
                int n = 0;
                for (int r = 0; r < P2; ++r) n += S.first[r];
                S.n_slots = n;
            }
        }
        __syncthreads();
        for (int p = tid; p < P2; p += kThreads) {
            const int e = S.ids[p];
            int f = 0;
            while (S.ids[f] != e) ++f;
            const int s = S.slot_of_pair[f];
            S.slot_pairs[s][S.rank[p]] = (short)p;
            S.pos_tab[s][p / K] = (short)p;
            atomicAdd(&S.slot_n[s], 1);
        }
        __syncthreads();
        const int U = S.n_slots;
        n_gu_chunks = warp_count(ns_cta + routed_count(U)) * CPT;
        const int TD = (U + 1) * CT;
        down_first = (int)((long long)cta * TD / G);
        down_count = (int)((long long)(cta + 1) * TD / G) - down_first;
        known_chunks = n_gu_chunks + warp_count(down_count);
        pump();
        while (consumed < n_gu_chunks) {
            if (!wait_chunk(consumed)) { atomicOr(&S.abort_flag, 1); break; }
            gate_up_chunk(consumed);
            ++consumed;
            pump();
        }
    }

    // ---------------------------------------------------------------- arrival B: down
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&P.sync[1], 1u);
        if (!S.abort_flag && !grid_wait(&P.sync[1])) S.abort_flag = 1;
    }
    __syncthreads();
    if (!S.abort_flag && down_count > 0) {
        const int s_first = down_first / CT;
        const int ns = (down_first + down_count - 1) / CT - s_first + 1;  // <= 2 (tokens*topK + 1 <= grid)
        if (tid < 2 * kMaxTokens) {
            const int sl = tid / kMaxTokens, j = tid % kMaxTokens, slot = s_first + sl;
            if (sl < ns) {
                const int n = slot == 0 ? B : S.slot_n[slot - 1];
                if (j == 0) S.hs_n[sl] = n;
                if (j < n) {
                    int pos, t;
                    float w;
                    if (slot == 0) {
                        t = j;
                        pos = B * K + j;
                        w = ref_sigmoid(__ldcg(P.sg + j));
                    } else {
                        pos = S.slot_pairs[slot - 1][j];
                        t = pos / K;
                        w = S.wts[pos];
                    }
                    S.hs_token[sl][j] = t;
                    S.hs_weight[sl][j] = w;
                    S.hs_pos[sl][j] = pos;
                }
            }
        }
        __syncthreads();
        for (int pr = warp; pr < ns * kMaxTokens; pr += kWarps) {
            const int sl = pr / kMaxTokens, j = pr % kMaxTokens;
            if (j < S.hs_n[sl])
                vector_to_frags<NGD>(P.hbuf + (long long)S.hs_pos[sl][j] * F, S.bfrag, 16, sl * kMaxTokens + j, S.hsum[sl][j],
                                     &S.hscale[sl][j], lane);
        }
        __syncthreads();
        while (consumed < known_chunks) {
            if (!wait_chunk(consumed)) { S.abort_flag = 1; break; }
            int kind, slot, tile, sub;
            chunk_of(consumed, kind, slot, tile, sub);
            const unsigned char *st = S.stages[warp][consumed % kStages];
            const int sl = slot - s_first, n = S.hs_n[sl];
            float tot[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
            tile_math<NGD, kDownSw128>(smem_u32(st), lane, S.bfrag, 16, sl * kMaxTokens, 0, &S.hsum[sl][0][0], NGD,
                                       reinterpret_cast<const unsigned short *>(st + 16 * (F / 4)), NGD, tot);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int j = 2 * q + cc;
                if (j < n) {
                    const int t = S.hs_token[sl][j];
                    const float w = S.hs_weight[sl][j] * S.hscale[sl][j];
                    const long long c = 16LL * tile + g;
                    atomicAdd(P.y + (long long)t * H + c, tot[0][cc] * w);
                    atomicAdd(P.y + (long long)t * H + c + 8, tot[1][cc] * w);
                }
            }
            ++consumed;
            pump();
        }
    }

    // ---------------------------------------------------------------- exit
    drain();
    __syncthreads();
    if (tid == 0) {
        if (S.abort_flag) raise_error(P.err, kErrWaitTimeout);
        __threadfence();
        const unsigned prev = atomicAdd(&P.sync[2], 1u);
        if (prev == (unsigned)G - 1) {  // last CTA out resets the arrival counters for the next launch
            P.sync[0] = 0;
            P.sync[1] = 0;
            __threadfence();
            P.sync[2] = 0;
        }
    }
}

}  // namespace fast

size_t moe_fast_scratch_bytes(int tokens, int width, int ff, int experts, int topK) {
    const size_t pos = (size_t)tokens * topK + tokens;
    auto a = [](size_t n) { return (n + 255) & ~size_t(255); };
    return a(sizeof(float) * tokens * experts) + a(sizeof(float) * tokens) + a(sizeof(float) * pos * ff);
}

bool moe_fast_supported(int tokens, int width, int ff, int topK, int grid) {
    // tokens * topK + 1 <= grid bounds the expert slots so that each CTA's contiguous range of
    // down tiles spans at most two slots (the shared-memory staging holds two).
    return tokens >= 1 && tokens <= fast::kMaxTokens && topK <= 32 && tokens * topK + 1 <= grid &&
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
           unsigned long long s1, unsigned long long s2, unsigned b0, unsigned b1, CUtensorMapSwizzle sw) {
    auto fn = encoder();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encoded maps of the last layers used, keyed by their blob addresses.
struct MapSet {
    const void *blobs, *shared;
    int width, ff, experts;
    CUtensorMap gu[2], gs[2], dc[2];
};
std::mutex g_map_mutex;
MapSet g_maps[64];
int g_map_next = 0;

bool layer_maps(const MoeLayerDev &L, fast::Params &p) {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    for (const MapSet &m : g_maps)
        if (m.blobs == L.blobs && m.shared == L.shared_blob && m.width == L.width && m.ff == L.ff && m.experts == L.experts) {
            std::memcpy(p.tm_gu, m.gu, sizeof m.gu);
            std::memcpy(p.tm_gs, m.gs, sizeof m.gs);
            std::memcpy(p.tm_dc, m.dc, sizeof m.dc);
            return true;
        }
    MapSet m;
    m.blobs = L.blobs;
    m.shared = L.shared_blob;
    m.width = L.width;
    m.ff = L.ff;
    m.experts = L.experts;
    const long long H = L.width, F = L.ff, bb = L.blob_words * 4;
    const long long d_codes = 2 * F * H / 4, gu_scales = 3 * F * H / 4;
    const bool sw128 = F == 512;
    for (int i = 0; i < 2; ++i) {
        const unsigned char *base = reinterpret_cast<const unsigned char *>(i == 0 ? L.blobs : L.shared_blob);
        const unsigned long long ne = i == 0 ? (unsigned long long)L.experts : 1ull;
        if (!map3d(&m.gu[i], base, H / 4, 2 * F, ne, H / 4, bb, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !map3d(&m.gs[i], base + gu_scales, 2 * (H / 64), 2 * F, ne, 2 * (H / 64), bb, 16, 16, CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !map3d(&m.dc[i], base + d_codes, F / 4, H, ne, F / 4, bb, sw128 ? 128 : 32, 16,
                   sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B))
            return false;
    }
    g_maps[g_map_next] = m;
    g_map_next = (g_map_next + 1) % 64;
    std::memcpy(p.tm_gu, m.gu, sizeof m.gu);
    std::memcpy(p.tm_gs, m.gs, sizeof m.gs);
    std::memcpy(p.tm_dc, m.dc, sizeof m.dc);
    return true;
}

template <int NG, int NGD>
cudaError_t launch_fast(const fast::Params &p, int grid, cudaStream_t s) {
    const size_t smem = sizeof(fast::Smem<NG, NGD>) + 1024;  // + slack for the 1024-byte stage alignment
    STRATA_CUDA_TRY(cudaFuncSetAttribute(fast::k_moe_fast<NG, NGD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(fast::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fast::k_moe_fast<NG, NGD>, p);
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
    prm.hbuf = reinterpret_cast<float *>(p);
    prm.sync = sync;
    prm.err = err;
    prm.spin_limit = 1ull << 20;  // grid waits sleep 64 ns per try, mbarrier tries suspend <= 2 us: bounded to ~2 s
    if (!layer_maps(L, prm)) return cudaErrorInvalidValue;
    if (L.width == 2048 && L.ff == 512) return launch_fast<32, 8>(prm, grid, s);
    if (L.width == 2560 && L.ff == 640) return launch_fast<40, 10>(prm, grid, s);
    return cudaErrorInvalidValue;
}

}  // namespace strata
