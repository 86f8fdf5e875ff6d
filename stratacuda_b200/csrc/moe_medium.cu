// Medium-batch fused mixture-of-experts layer (9 .. 64 tokens): integer tensor-core products on
// the raw 2-bit codes (as the decode kernel, csrc/moe_fast.cu), one whole expert per work unit,
// after the exact router kernels.
//
// At these batch sizes an expert sees one or two tokens on average (640 token-expert pairs
// over ~370 distinct experts at 64 tokens), so the layer is a bandwidth-bound product of the
// weights with a few columns: dequantising every weight to FP16 for the tcgen05 GEMMs of the
// prefill path costs far more than the weight bytes themselves. Here the weights stay as
// codes (u8 x s8 mma.sync, activations as three signed 8-bit digits, exact integer products).
//
// Launches: the exact router logits (k_pf_logits) and top-k (k_pf_route) of the prefill path,
// then ONE persistent cooperative kernel, one CTA per SM, 8 warps:
//   A. CTA c turns tokens c, c + G, ... into their digit records in global memory (the digits
//      of the 64-element groups in the MMA operand layout, each group's digit sum and the
//      scale 2^-k) and arrives. Every CTA builds the pair table: pairs (t * topK + k) ordered
//      by expert, token-major within an expert (a stable counting sort; src/prefill.js:55-61
//      orders them the same way), and numbers the token groups: the shared expert's groups of
//      two tokens first (its weights are read again from L2 for each; groups of eight made its
//      units the slowest of the layer), then each routed expert's pairs in groups of eight.
//   B. Work unit = one token group with its whole expert, dealt round-robin (unit u on CTA
//      u % G). The unit copies its tokens' digit records into shared memory (one bulk copy
//      each, issued while the unit before finishes), then
//        gate/up: warp w takes the 16-row tiles w, w + 8, ... of the 2F interleaved rows (a
//        tile is 8 hidden values), full width, and forms silu(gate) * up;
//        hidden -> digits: each token's F hidden values as three signed 8-bit digits (one
//        rounding, 2^-22 of the token's largest |h|), the same operand layout as x;
//        down: warp w takes H/8 rows, 16 full rows per copy;
//      and stores weight * result as one partial row of y per pair (per token for the shared
//      expert).
//   C. After a second arrival every CTA sums a slice of y from the partial rows in a fixed
//      order (the shared expert, then the routed pairs in selection order): the same bits
//      every run.
// Whole experts per unit keep every copy a TMA box of full rows, and every box one contiguous
// range of the blob: a step is one warp's work, either a gate/up tile (16 interleaved rows,
// full width: one 4D box laid out chunk-major, 128-byte swizzle) or a down block (64 full
// rows), plus one bulk copy of the step's scales. Measured on B200 with all SMs streaming,
// boxes of contiguous rows moved 60 GB/s per SM, boxes of 128-byte pieces of strided rows
// (a 128-row x 128-byte gate/up box, the earlier step of this kernel) 18-24 GB/s per SM.
// Step c of the CTA belongs to warp c % 8 and lands in stage c % NST of one shared ring; the
// warp that consumed step c issues step c + NST into the same stage at once (the stage has no
// other reader), so no warp waits for another to refill and no copy waits behind compute.
// Every wait is bounded: past the limit the kernel records kErrWaitTimeout and leaves.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "q2mma.cuh"

namespace strata {
namespace medium {

using namespace q2;

constexpr int kMaxBatch = 64;
constexpr int kMaxTopK = 32;
constexpr int kMaxPairs = kMaxBatch * kMaxTopK;
constexpr int kMaxExperts = 512;
constexpr int kSharedGroup = 2;  // tokens per shared-expert unit (its weights are read once per unit, from L2 after the first)
constexpr int kMWarps = 16;      // warps of a CTA: four per scheduler, to hide the MMA and load latencies
constexpr int kMThreads = kMWarps * 32;
constexpr int kUnitTokens = 4;   // token slots of a unit (MMA column pairs: kUnitTokens / 2)
constexpr int kUnitCG = kUnitTokens / 2;

// Digit record of one vector of N elements: digits uint2[N/64][2][4][3] (group, MMA half,
// 16-element block q, digit), int sum[N/64], float scale (2^-k). In shared memory, slots are
// STRIDE bytes apart, 96 modulo 128, so the two slots a warp reads together mostly fall on
// distinct banks.
template <int N>
struct Rec {
    static constexpr int NGR = N / 64;
    static constexpr int DIGITS = NGR * 2 * 4 * 3;
    static constexpr int SUM = DIGITS * 8;
    static constexpr int SCALE = SUM + NGR * 4;
    static constexpr int BYTES = (SCALE + 4 + 15) / 16 * 16;
    static constexpr int STRIDE = BYTES + (96 - BYTES % 128 + 128) % 128;
    static_assert(BYTES % 16 == 0 && STRIDE % 128 == 96, "record layout");
};

// A step: one warp's gate/up tile (16 rows x H/4 bytes) or down block (64 rows x F/4 bytes)
// with its scales; both are STAGE bytes of codes at the supported shapes.
template <int H, int F>
struct MGeo {
    static constexpr int NG = H / 64;                // gate/up scale groups per row
    static constexpr int NJ = F / 64;                // down scale groups per row
    static constexpr int CPT = NG / 8;               // gate/up column chunks (128 bytes) per row
    static constexpr int GU_STEPS = 2 * F / 16;      // per unit: 16-row gate/up tiles
    static constexpr int DN_STEPS = H / 64;          // per unit: 64-row down blocks
    static constexpr int STEPS = GU_STEPS + DN_STEPS;
    static constexpr int DROW = F / 4;               // bytes of a down row
    static constexpr int GU_BYTES = 16 * (H / 4), DN_BYTES = 64 * DROW;
    static constexpr int GU_SBYTES = 16 * NG * 2, DN_SBYTES = 64 * NJ * 2;
    static constexpr int STAGE = GU_BYTES > DN_BYTES ? GU_BYTES : DN_BYTES;          // codes of a step (1024-aligned)
    static constexpr int SSTAGE = GU_SBYTES > DN_SBYTES ? GU_SBYTES : DN_SBYTES;     // scales of a step
    static constexpr int NST = F == 512 ? 16 : 8;    // stages (shared-memory budget)
    static_assert(NG % 8 == 0 && H % 512 == 0 && STAGE % 1024 == 0 && SSTAGE % 128 == 0, "geometry");
    // step c of a CTA belongs to warp c % kMWarps, and a stage's use v - 2 was consumed by the
    // warp that consumes its use v (the parity waits below rely on it)
    static_assert((2 * NST) % kMWarps == 0, "step ownership");
};

struct Params {
    MoeLayerDev L;
    const float *x;
    int tokens;
    float *y;
    const int *ids;        // [tokens][topK], from the router kernel
    const float *weights;  // [tokens][topK]
    const float *sg;       // [tokens] shared-gate logits
    unsigned char *xrec;   // [tokens] digit records of x (Rec<H>::BYTES each)
    float *part;           // [tokens*topK + tokens][H] partial rows of y
    unsigned *sync;        // [0] digit records written, [1] partial rows written, [2] exits
    unsigned *err;
    unsigned long long spin_limit;
    MoeMaps maps;  // [0] routed experts, [1] the shared expert
};

template <int H, int F>
struct Smem {
    using G = MGeo<H, F>;
    unsigned char codes[G::NST][G::STAGE];  // 1024-aligned
    alignas(128) unsigned short scl[G::NST][G::SSTAGE / 2];
    alignas(128) unsigned char xrec[kUnitTokens][Rec<H>::STRIDE];  // the unit's tokens: x digits
    alignas(128) unsigned char hrec[kUnitTokens][Rec<F>::STRIDE];  // the unit's tokens: hidden digits
    float hid[kUnitTokens][F];
    float hmaxw[kMWarps][kUnitTokens];  // per-warp max |hidden| of each token slot
    short pairs[kMaxPairs];           // pairs ordered by expert, token-major within one
    int off[kMaxExperts + 1];         // expert e's pairs: pairs[off[e] .. off[e+1])
    int gstart[kMaxExperts + 1];      // expert e's token groups: [gstart[e], gstart[e+1])
    int run[kMaxExperts];             // pair counts, then placement cursors
    int ids[kMaxPairs];               // the routed ids
    int scan_w[2][kMWarps];
    float sgw[kMaxBatch];     // sigmoid(shared-gate logit) per token
    int urow[2][kUnitTokens];  // unit token slot -> partial row (by unit parity)
    float uw[2][kUnitTokens];  // unit token slot -> weight
    unsigned xmax;
    unsigned long long full[G::NST], empty[G::NST];
    int issued[G::NST];  // uses of each stage issued so far
    unsigned long long bar_x;
    int abort_flag;
};

// Block-wide exclusive scan of two sequences over [0, n) (n <= 2 kMThreads: thread i holds
// entries 2i and 2i+1); out[n] receives each total.
template <int H, int F>
__device__ __forceinline__ void scan2(Smem<H, F> &S, const int (&a)[2], const int (&b)[2], int n, int *out_a, int *out_b, int base_b) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int sa = a[0] + a[1], sb = b[0] + b[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ua = __shfl_up_sync(0xffffffffu, sa, o), ub = __shfl_up_sync(0xffffffffu, sb, o);
        if (lane >= o) {
            sa += ua;
            sb += ub;
        }
    }
    if (lane == 31) {
        S.scan_w[0][warp] = sa;
        S.scan_w[1][warp] = sb;
    }
    __syncthreads();
    int wa = 0, wb = 0, ta = 0, tb = 0;
    for (int w = 0; w < kMWarps; ++w) {
        if (w < warp) {
            wa += S.scan_w[0][w];
            wb += S.scan_w[1][w];
        }
        ta += S.scan_w[0][w];
        tb += S.scan_w[1][w];
    }
    const int ea = wa + sa - (a[0] + a[1]), eb = wb + sb - (b[0] + b[1]);  // exclusive prefix of entry 2 tid
    if (2 * tid < n) {
        out_a[2 * tid] = ea;
        out_b[2 * tid] = base_b + eb;
    }
    if (2 * tid + 1 < n) {
        out_a[2 * tid + 1] = ea + a[0];
        out_b[2 * tid + 1] = base_b + eb + b[0];
    }
    if (tid == 0) {
        out_a[n] = ta;
        out_b[n] = base_b + tb;
    }
}

// GPC values of 16 bits from shared memory into floats (FP16 -> F32, exact), vector loads
// where the row allows them.
template <int GPC, int SCLN>
__device__ __forceinline__ void load_scales(const unsigned short *row, float (&s)[GPC]) {
    if constexpr (GPC % 8 == 0 && SCLN % 8 == 0) {
#pragma unroll
        for (int i = 0; i < GPC / 8; ++i) {
            const uint4 v = reinterpret_cast<const uint4 *>(row)[i];
            const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[j]));
                s[8 * i + 2 * j] = f.x;
                s[8 * i + 2 * j + 1] = f.y;
            }
        }
    } else {
        static_assert(GPC % 2 == 0 && SCLN % 2 == 0, "scale pairs");
#pragma unroll
        for (int i = 0; i < GPC / 2; ++i) {
            const float2 f = __half22float2(reinterpret_cast<const __half2 *>(row)[i]);
            s[2 * i] = f.x;
            s[2 * i + 1] = f.y;
        }
    }
}

// 16 rows x GPC groups of one chunk against the digit records of the unit's token slots (MMA
// columns: token slot 2 cg + g / 4, digit g % 4, the fourth digit zero). `code` is the rows'
// codes in shared memory (SWZ: 128-byte rows with the 128-byte swizzle; else ROWB-byte rows),
// the groups starting at 16-byte column `col0`, `scl` their scales [16 rows][SCLN] (from the
// first group), `g0` the first
// group in the records (RSTRIDE bytes apart, group sums at byte `sum_off`). Adds
// scale * sum((c - 1) v) per group into acc[cg] of row g (even q) or g + 8 (odd q), token slot
// 2 cg + q / 2: the two lanes of a pair swap the partial digit sums the other one's row needs.
template <int GPC, bool SWZ, int ROWB, int SCLN, int RSTRIDE>
__device__ __forceinline__ void mma_chunk(unsigned code, int col0, const unsigned short *scl, const unsigned char *recs, int sum_off, int g0,
                                          const int (&tsB)[kUnitCG], const int (&tsC)[kUnitCG], int ncg, float (&acc)[kUnitCG]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3, d = g & 3;
    const bool odd = q & 1;
    const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
    unsigned w[GPC / 2][4];
#pragma unroll
    for (int gp = 0; gp < GPC / 2; ++gp) {
        const int c = col0 + 2 * gp + (lane >> 4);
        const unsigned addr = SWZ ? code + r * 128 + ((c ^ (r & 7)) << 4) : code + r * ROWB + (c << 4);
        ldsm_x4(addr, w[gp][0], w[gp][1], w[gp][2], w[gp][3]);
    }
    // expert scales are finite FP16 (checked on upload, src/model.js:164): exact conversion
    float s_row[GPC];
    load_scales<GPC, SCLN>(scl + (g + (odd ? 8 : 0)) * SCLN, s_row);
#pragma unroll
    for (int cg = 0; cg < kUnitCG; ++cg) {
        if (cg >= ncg) break;
        const uint2 *dg = reinterpret_cast<const uint2 *>(recs + (tsB[cg] >= 0 ? tsB[cg] : 0) * RSTRIDE);
        uint2 bf[GPC][2];
#pragma unroll
        for (int gl = 0; gl < GPC; ++gl)
#pragma unroll
            for (int h = 0; h < 2; ++h) bf[gl][h] = tsB[cg] >= 0 ? dg[(((g0 + gl) * 2 + h) * 4 + q) * 3 + d] : make_uint2(0u, 0u);
        int c4[GPC][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int gl = 0; gl < GPC; ++gl) {
                const unsigned wl = w[gl >> 1][(gl & 1) ? 2 : 0], wh = w[gl >> 1][(gl & 1) ? 3 : 1];
                imma_acc(h > 0, c4[gl], (wl >> (4 * h)) & 0x03030303u, (wh >> (4 * h)) & 0x03030303u, (wl >> (4 * h + 2)) & 0x03030303u,
                     (wh >> (4 * h + 2)) & 0x03030303u, bf[gl][h].x, bf[gl][h].y);
            }
        // lane (g, q) holds rows g and g + 8 at columns 2q, 2q + 1: digits 0, 1 (even q) or 2 and
        // the zero column (odd q). Even q keeps row g, odd q row g + 8; each sends its partner the
        // piece of the other row: digits 0 + 256 * 1 of row g + 8, or digit 2 of row g.
        const int *xsr = reinterpret_cast<const int *>(recs + (tsC[cg] >= 0 ? tsC[cg] : 0) * RSTRIDE + sum_off) + g0;
#pragma unroll
        for (int gl = 0; gl < GPC; ++gl) {
            const int send = odd ? c4[gl][0] : c4[gl][2] + 256 * c4[gl][3];
            const int recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const int v = odd ? recv + 65536 * c4[gl][2] : c4[gl][0] + 256 * c4[gl][1] + 65536 * recv;
            acc[cg] = fmaf(s_row[gl], (float)(v - xsr[gl]), acc[cg]);
        }
    }
}

template <int H, int F>
__global__ void __launch_bounds__(kMThreads, 1) k_moe_medium(const __grid_constant__ Params P) {
    using Gm = MGeo<H, F>;
    using RX = Rec<H>;
    using RH = Rec<F>;
    constexpr int NG = Gm::NG, NJ = Gm::NJ, CPT = Gm::CPT, NST = Gm::NST, GU_STEPS = Gm::GU_STEPS, DN_STEPS = Gm::DN_STEPS;
    constexpr int STEPS = Gm::STEPS;
    extern __shared__ unsigned char smem_raw[];
    auto &S = *reinterpret_cast<Smem<H, F> *>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
    const MoeLayerDev &L = P.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const int G = gridDim.x, cta = blockIdx.x;
    const int B = P.tokens, K = L.topK, E = L.experts, P2 = B * K, SG = (B + kSharedGroup - 1) / kSharedGroup;
    const long long gu_scales_b = 3LL * F * H / 4, d_scales_b = gu_scales_b + 2LL * F * (H / 64) * 2;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
            S.issued[s] = 0;
        }
        mbar_init(&S.bar_x, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
        for (int i = 0; i < 2; ++i) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.maps.gu16r[i])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.maps.dn64[i])) : "memory");
        }
    }
    for (int e = tid; e < E; e += kMThreads) S.run[e] = 0;
    __syncthreads();

    // ------------------------------------------------------------------ A1: digit records of tokens cta, cta + G, ...
    for (int t = cta; t < B; t += G) {
        const float *xt = P.x + (long long)t * H;
        unsigned char *rec = P.xrec + (long long)t * RX::BYTES;
        if (tid == 0) S.xmax = 0u;
        __syncthreads();
        float mx = 0.0f;  // largest |x| (NaN ignored, as fmaxf; max is order-free)
        for (int i = tid; i < H / 4; i += kMThreads) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(xt) + i);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
        if (lane == 0) atomicMax(&S.xmax, __float_as_uint(mx));
        __syncthreads();
        const int k = scale_exp(__uint_as_float(S.xmax));
        const float mul = pow2f(k);  // exact power of two
        // blocks of 16 elements (group, q), one per thread; NG * 4 is a multiple of 32, so whole
        // warps take part and the group-sum shuffles see all four blocks of a group
        for (int b = tid; b < NG * 4; b += kMThreads) {
            const int grp = b >> 2, qq = b & 3;
            const float4 *src = reinterpret_cast<const float4 *>(xt + 64 * grp + 16 * qq);
            int v[16];
            int part = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 f = __ldg(src + i);
                v[4 * i] = __float2int_rn(f.x * mul);
                v[4 * i + 1] = __float2int_rn(f.y * mul);
                v[4 * i + 2] = __float2int_rn(f.z * mul);
                v[4 * i + 3] = __float2int_rn(f.w * mul);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) part += v[i];
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            uint2 *dg = reinterpret_cast<uint2 *>(rec);
            block_frags(v, dg + ((grp * 2 + 0) * 4 + qq) * 3, dg + ((grp * 2 + 1) * 4 + qq) * 3);
            if (qq == 0) reinterpret_cast<int *>(rec + RX::SUM)[grp] = part;
        }
        if (tid == 0) *reinterpret_cast<float *>(rec + RX::SCALE) = pow2f(-k);
        __syncthreads();
    }
    const int n_rec_ctas = min(G, B);  // CTAs that write records
    if (cta < B && tid == 0) {         // the records are read by bulk copies (async proxy) on other SMs
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        atomicAdd(&P.sync[0], 1u);
    }

    // ------------------------------------------------------------------ A2: pair table, token groups
    for (int p = tid; p < P2; p += kMThreads) {
        const int e = __ldg(P.ids + p);
        S.ids[p] = e;
        if (e >= 0 && e < E) atomicAdd(&S.run[e], 1);
    }
    for (int t = tid; t < B; t += kMThreads) S.sgw[t] = ref_sigmoid(__ldg(P.sg + t));
    __syncthreads();
    {
        int c[2], ng[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int e = 2 * tid + i;
            c[i] = e < E ? S.run[e] : 0;
            ng[i] = (c[i] + kUnitTokens - 1) / kUnitTokens;
        }
        scan2(S, c, ng, E, S.off, S.gstart, SG);
    }
    __syncthreads();
    for (int e = tid; e < E; e += kMThreads) S.run[e] = S.off[e];  // placement cursors
    __syncthreads();
    if (warp == 0) {  // stable placement, 32 pairs at a time in pair order
        for (int base = 0; base < P2; base += 32) {
            const int p = base + lane;
            const int e = p < P2 ? S.ids[p] : -1;
            const bool valid = e >= 0 && e < E;
            const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1 - lane);
            const int rank = __popc(same & ((1u << lane) - 1u));
            if (valid) S.pairs[S.run[e] + rank] = (short)p;
            __syncwarp();
            if (valid && rank == __popc(same) - 1) S.run[e] += __popc(same);  // the last lane of each expert advances its cursor
            __syncwarp();
        }
    }
    __syncthreads();
    const int NU = S.gstart[E];
    const int n_units = cta < NU ? (NU - 1 - cta) / G + 1 : 0;

    // ------------------------------------------------------------------ copy pipeline
    // Step c of this CTA: unit c / STEPS; within it the gate/up tiles first, then the down
    // blocks. Warp c % 8 consumes it from stage c % NST and then issues step c + NST there.
    const int total = n_units * STEPS;
    bool stalled = false;          // this warp saw a wait time out
    int memo_gi = -1, memo_e = 0;  // the last routed group looked up
    // unit ui -> token group gi, map m (1: shared expert), expert e, group index tg within it
    auto unit_of = [&](int ui, int &gi, int &m, int &e, int &tg) {
        gi = cta + ui * G;
        if (gi < SG) {
            m = 1;
            e = 0;
            tg = gi;
            return;
        }
        if (gi != memo_gi) {
            int lo = 0, hi = E;  // the expert with gstart[e] <= gi < gstart[e + 1]
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (S.gstart[mid] <= gi) lo = mid;
                else hi = mid;
            }
            memo_gi = gi;
            memo_e = lo;
        }
        m = 0;
        e = memo_e;
        tg = gi - S.gstart[e];
    };
    auto blob_of = [&](int m, int e) {
        return reinterpret_cast<const unsigned char *>(m ? L.shared_blob : L.blobs + (long long)e * L.blob_words);
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
    auto produce = [&](int c) {  // one thread: step c into its stage, whose last use has been consumed
        const int st = c % NST, ui = c / STEPS, idx = c % STEPS;
        int gi, m, e, tg;
        unit_of(ui, gi, m, e, tg);
        if (idx < GU_STEPS) {  // gate/up tile idx: blob rows 16 idx .. 16 idx + 15, [chunk][row][128 B]
            mbar_expect(&S.full[st], Gm::GU_BYTES + Gm::GU_SBYTES);
            tma_4d(S.codes[st], &P.maps.gu16r[m], 0, 16 * idx, 0, e, &S.full[st]);
            bulk_copy(S.scl[st], blob_of(m, e) + gu_scales_b + (long long)16 * idx * NG * 2, Gm::GU_SBYTES, &S.full[st]);
        } else {  // down block d: rows 64 d .. 64 d + 63
            const int row0 = 64 * (idx - GU_STEPS);
            mbar_expect(&S.full[st], Gm::DN_BYTES + Gm::DN_SBYTES);
            tma_3d(S.codes[st], &P.maps.dn64[m], 0, row0, e, &S.full[st]);
            bulk_copy(S.scl[st], blob_of(m, e) + d_scales_b + (long long)row0 * NJ * 2, Gm::DN_SBYTES, &S.full[st]);
        }
        S.issued[st] = c / NST + 1;
    };
    // This warp's step c once it has landed (-1 after a timeout). The stage's previous use was
    // consumed first (the empty barrier): only then is the full barrier's parity unambiguous.
    auto take = [&](int c) -> int {
        const int st = c % NST, v = c / NST;
        if (!stalled && !__all_sync(0xffffffffu, (v == 0 || wait_bar(&S.empty[st], (v - 1) & 1)) && wait_bar(&S.full[st], v & 1)))
            fail_wait();
        return stalled ? -1 : st;
    };
    // this warp is done reading step c: free its stage and refill it with step c + NST (the stage
    // was read through the generic proxy)
    auto release = [&](int c) {
        __syncwarp();
        if (lane == 0) {
            const int st = c % NST;
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&S.empty[st])) : "memory");
            if (!stalled && c + NST < total) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                produce(c + NST);
            }
        }
        __syncwarp();
    };
    // Token slots of unit ui (warp 0): partial rows and weights (by unit parity), and lane n's
    // bulk copy of slot n's x digit record. Called once every warp has finished reading the x
    // digits of the unit before.
    auto stage_unit = [&](int ui) {
        int gi, m, e, tg;
        unit_of(ui, gi, m, e, tg);
        const int n = m ? min(kSharedGroup, B - kSharedGroup * tg) : min(kUnitTokens, S.off[e + 1] - S.off[e] - kUnitTokens * tg);
        const int buf = ui & 1;
        int tok = 0;
        if (lane < n) {
            if (m) {
                tok = kSharedGroup * tg + lane;
                S.urow[buf][lane] = P2 + tok;
                S.uw[buf][lane] = S.sgw[tok];
            } else {
                const int pr = S.pairs[S.off[e] + kUnitTokens * tg + lane];
                tok = pr / K;
                S.urow[buf][lane] = pr;
                S.uw[buf][lane] = __ldg(P.weights + pr);
            }
        }
        __syncwarp();
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect(&S.bar_x, (unsigned)(n * RX::BYTES));
        }
        __syncwarp();
        if (lane < n) bulk_copy(S.xrec[lane], P.xrec + (long long)tok * RX::BYTES, RX::BYTES, &S.bar_x);
    };

    if (tid == 0)  // weights need no digits: the first steps' copies start now
        for (int c = 0; c < NST && c < total; ++c) produce(c);

    // ------------------------------------------------------------------ arrival: digit records
    if (tid == 0) {
        for (unsigned long long i = 0;; ++i) {
            if (ld_acquire(&P.sync[0]) >= (unsigned)n_rec_ctas) break;
            if (i > P.spin_limit) {
                S.abort_flag = 1;
                break;
            }
            __nanosleep(32);
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");  // the records are read by bulk copies
    }
    __syncthreads();
    if (S.abort_flag) stalled = true;
    int x_staged = -1;  // the last unit whose x digits were requested (the same on every thread)
    if (n_units > 0 && !stalled) {
        if (warp == 0) stage_unit(0);
        x_staged = 0;
    }

    // ------------------------------------------------------------------ units
    constexpr int NCG = kUnitCG;
    for (int ui = 0; ui < n_units; ++ui) {
        int gi, m, e, tg;
        unit_of(ui, gi, m, e, tg);
        const int n_cur = m ? min(kSharedGroup, B - kSharedGroup * tg) : min(kUnitTokens, S.off[e + 1] - S.off[e] - kUnitTokens * tg);
        const int ncg = (n_cur + 1) / 2, buf = ui & 1;
        int tsB[NCG], tsC[NCG];
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            const int b = 2 * cg + (g >> 2), c = 2 * cg + (q >> 1);
            tsB[cg] = (g & 3) < 3 && b < n_cur ? b : -1;
            tsC[cg] = c < n_cur ? c : -1;
        }
        if (!stalled && !__all_sync(0xffffffffu, wait_bar(&S.bar_x, ui & 1))) fail_wait();  // the slots' x digits

        // gate/up: tiles warp + 8 i; a tile holds 8 hidden values (rows 2h, 2h+1 interleaved)
        float hmax[NCG];
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) hmax[cg] = 0.0f;
        const int c0 = ui * STEPS;  // this unit's first step; step c belongs to warp c % kMWarps
        const int first = ((warp - c0) % kMWarps + kMWarps) % kMWarps;
        for (int tile = first; tile < GU_STEPS; tile += kMWarps) {  // rows 16 tile .. 16 tile + 15
            float acc[NCG];
#pragma unroll
            for (int cg = 0; cg < NCG; ++cg) acc[cg] = 0.0f;
            const int st = take(c0 + tile);
            if (st >= 0)
#pragma unroll 1
                for (int hc = 0; hc < 2 * CPT; ++hc) {  // half chunks: 4 scale groups of one 128-byte column chunk
                    const int sub = hc >> 1, half = hc & 1;
                    mma_chunk<4, true, 128, NG, RX::STRIDE>(smem_u32(S.codes[st]) + 2048 * sub, 4 * half, S.scl[st] + 8 * sub + 4 * half,
                                                            &S.xrec[0][0], RX::SUM, 8 * sub + 4 * half, tsB, tsC, ncg, acc);
                }
            release(c0 + tile);
            // lane (g, q) holds row g (even q) or g + 8 (odd q) for token slot 2cg + q/2; row g
            // (gate when g is even) pairs with row g + 1 (up) four lanes down: hidden 8 tile + g/2
            // (+ 4 for rows g + 8)
#pragma unroll
            for (int cg = 0; cg < NCG; ++cg) {
                if (cg >= ncg) break;
                const float sc = tsC[cg] >= 0 ? *reinterpret_cast<const float *>(S.xrec[tsC[cg]] + RX::SCALE) : 0.0f;
                const float gv = acc[cg] * sc;
                const float up = __shfl_down_sync(0xffffffffu, gv, 4);
                if (!(g & 1) && tsC[cg] >= 0) {
                    const float hv = __fmul_rn(ref_silu(gv), up);
                    S.hid[tsC[cg]][8 * tile + ((q & 1) ? 4 : 0) + (g >> 1)] = hv;
                    hmax[cg] = fmaxf(hmax[cg], fabsf(hv));  // NaN ignored, as fmaxf
                }
            }
        }
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            if (cg >= ncg) break;
            float mh = hmax[cg];
            mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, 1));
            mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, 4));
            mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, 8));
            mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, 16));
            if (g == 0 && !(q & 1) && tsC[cg] >= 0) S.hmaxw[warp][tsC[cg]] = mh;
        }
        if (__syncthreads_or(stalled ? 1 : 0)) break;  // a warp's copies timed out: all leave together
        if (ui + 1 < n_units) {                       // every warp is done with this unit's x digits
            if (warp == 0) stage_unit(ui + 1);
            x_staged = ui + 1;
        }

        // hidden -> digit records: blocks of 16 values (slot, group, q), 32 per warp iteration
        for (int b0 = warp * 32; b0 < n_cur * NJ * 4; b0 += kMThreads) {
            const int b = b0 + lane;
            const bool live = b < n_cur * NJ * 4;
            const int ts = live ? b / (NJ * 4) : 0, grp = (b >> 2) % NJ, qq = b & 3;
            float mx = 0.0f;
#pragma unroll
            for (int w = 0; w < kMWarps; ++w) mx = fmaxf(mx, S.hmaxw[w][ts]);
            const int k = scale_exp(mx);
            const float mul = pow2f(k);
            int v[16];
            int part = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v[i] = live ? __float2int_rn(S.hid[ts][64 * grp + 16 * qq + i] * mul) : 0;
                part += v[i];
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if (live) {
                unsigned char *rec = S.hrec[ts];
                uint2 *dg = reinterpret_cast<uint2 *>(rec);
                block_frags(v, dg + ((grp * 2 + 0) * 4 + qq) * 3, dg + ((grp * 2 + 1) * 4 + qq) * 3);
                if (qq == 0) reinterpret_cast<int *>(rec + RH::SUM)[grp] = part;
                if (grp == 0 && qq == 0) *reinterpret_cast<float *>(rec + RH::SCALE) = pow2f(-k);
            }
        }
        __syncthreads();

        // down: warp w takes the 64-row blocks w, w + 8, ... (tiles of 16 rows: row g for even q,
        // g + 8 for odd q; token slot 2cg + q/2)
        float wsc[NCG];
        int prow[NCG];
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {
            wsc[cg] = tsC[cg] >= 0 ? *reinterpret_cast<const float *>(S.hrec[tsC[cg]] + RH::SCALE) * S.uw[buf][tsC[cg]] : 0.0f;
            prow[cg] = tsC[cg] >= 0 ? S.urow[buf][tsC[cg]] : 0;
        }
        const int first_dn = ((warp - c0 - GU_STEPS) % kMWarps + kMWarps) % kMWarps;
        for (int blk = first_dn; blk < DN_STEPS; blk += kMWarps) {  // rows 64 blk .. 64 blk + 63, 16 per tile
            const int st = take(c0 + GU_STEPS + blk);
#pragma unroll 1
            for (int tt = 0; tt < 4; ++tt) {
                float acc[NCG];
#pragma unroll
                for (int cg = 0; cg < NCG; ++cg) acc[cg] = 0.0f;
                if (st >= 0) {
                    const unsigned cb = smem_u32(S.codes[st]) + 16 * Gm::DROW * tt;
                    const unsigned short *sb = S.scl[st] + 16 * NJ * tt;
#pragma unroll 1
                    for (int g4 = 0; g4 < NJ / 4; ++g4)
                        mma_chunk<4, Gm::DROW == 128, Gm::DROW, NJ, RH::STRIDE>(cb, 4 * g4, sb + 4 * g4, &S.hrec[0][0], RH::SUM, 4 * g4, tsB, tsC,
                                                                                ncg, acc);
                    if constexpr (NJ % 4 != 0)
                        mma_chunk<NJ % 4, Gm::DROW == 128, Gm::DROW, NJ, RH::STRIDE>(cb, NJ / 4 * 4, sb + NJ / 4 * 4, &S.hrec[0][0], RH::SUM,
                                                                                     NJ / 4 * 4, tsB, tsC, ncg, acc);
                }
                const int row = 64 * blk + 16 * tt + g + ((q & 1) ? 8 : 0);
#pragma unroll
                for (int cg = 0; cg < NCG; ++cg) {
                    if (cg >= ncg) break;
                    if (st >= 0 && tsC[cg] >= 0) __stcg(P.part + (long long)prow[cg] * H + row, acc[cg] * wsc[cg]);
                }
            }
            release(c0 + GU_STEPS + blk);
        }
    }

    // ------------------------------------------------------------------ second arrival: y
    __syncthreads();
    if (tid < NST && S.issued[tid] > 0)  // no copy may be in flight at exit: each stage's last use has landed
        wait_bar(&S.full[tid], (S.issued[tid] - 1) & 1);
    if (x_staged >= 0) wait_bar(&S.bar_x, x_staged & 1);  // no copy may be in flight at exit
    if (stalled) atomicOr(&S.abort_flag, 1);
    __syncthreads();
    if (tid == 0 && !grid_arrive_wait(&P.sync[1], (unsigned)G, P.spin_limit)) S.abort_flag = 1;
    __syncthreads();
    if (!S.abort_flag) {
        // y[t][4c .. 4c + 3], one thread each: the shared expert's term, then the routed pairs'
        // terms in selection order (kernels/strata.cu:360-365 adds them in that order; a pair
        // without an expert adds nothing). Eight terms' loads are in flight at once.
        const int H4 = H / 4;
        const float4 *part4 = reinterpret_cast<const float4 *>(P.part);
        for (int item = cta * kMThreads + tid; item < B * H4; item += G * kMThreads) {
            const int t = item / H4, c = item % H4;
            float4 v = __ldcg(part4 + (long long)(P2 + t) * H4 + c);
            for (int k0 = 0; k0 < K; k0 += 8) {
                float4 u[8];
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const int k = k0 + n;
                    const bool ok = k < K && (unsigned)S.ids[t * K + k] < (unsigned)E;
                    u[n] = ok ? __ldcg(part4 + (long long)(t * K + k) * H4 + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const int k = k0 + n;
                    if (k < K && (unsigned)S.ids[t * K + k] < (unsigned)E) {
                        v.x = __fadd_rn(v.x, u[n].x);
                        v.y = __fadd_rn(v.y, u[n].y);
                        v.z = __fadd_rn(v.z, u[n].z);
                        v.w = __fadd_rn(v.w, u[n].w);
                    }
                }
            }
            reinterpret_cast<float4 *>(P.y)[item] = v;
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
            __threadfence();
            P.sync[2] = 0;
        }
    }
}

static_assert(sizeof(Smem<2048, 512>) + 1024 <= 227 * 1024 && sizeof(Smem<2560, 640>) + 1024 <= 227 * 1024, "shared memory per CTA");

}  // namespace medium

size_t moe_medium_scratch_bytes(int tokens, int width, int ff, int experts, int topK) {
    auto a = [](size_t n) { return (n + 255) & ~size_t(255); };
    const size_t rec = width == 2048 ? medium::Rec<2048>::BYTES : medium::Rec<2560>::BYTES;
    return a(sizeof(float) * tokens * experts) + a(sizeof(float) * tokens) + a(moe_logits_tail_bytes(width)) + a(rec * tokens) +
           a(sizeof(float) * (size_t)(tokens * topK + tokens) * width);
}

bool moe_medium_supported(int tokens, int width, int ff, int experts, int topK, int grid) {
    return tokens > q2::kMaxTokens && tokens <= medium::kMaxBatch && topK >= 1 && topK <= medium::kMaxTopK && experts >= 1 &&
           experts <= medium::kMaxExperts && grid >= 1 && ((width == 2048 && ff == 512) || (width == 2560 && ff == 640));
}

namespace {

template <int H, int F>
cudaError_t launch_medium(const medium::Params &p, int grid, cudaStream_t s) {
    const size_t smem = sizeof(medium::Smem<H, F>) + 1024;  // + slack for the 1024-byte stage alignment
    static int device_ready = -1;
    int dev = 0;
    STRATA_CUDA_TRY(cudaGetDevice(&dev));
    if (device_ready != dev) {
        STRATA_CUDA_TRY(cudaFuncSetAttribute(medium::k_moe_medium<H, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        device_ready = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(medium::kMThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // the grid arrivals need every CTA resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, medium::k_moe_medium<H, F>, p);
}

}  // namespace

cudaError_t moe_forward_medium(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights, void *scratch,
                               unsigned *sync, int grid, cudaStream_t s, unsigned *err) {
    char *p = static_cast<char *>(scratch);
    auto a = [](size_t n) { return (n + 255) & ~size_t(255); };
    float *logits = reinterpret_cast<float *>(p);
    p += a(sizeof(float) * tokens * L.experts);
    float *sg = reinterpret_cast<float *>(p);
    p += a(sizeof(float) * tokens);
    float *tail = reinterpret_cast<float *>(p);
    p += a(moe_logits_tail_bytes(L.width));
    unsigned char *xrec = reinterpret_cast<unsigned char *>(p);
    p += a((L.width == 2048 ? medium::Rec<2048>::BYTES : medium::Rec<2560>::BYTES) * (size_t)tokens);
    float *part = reinterpret_cast<float *>(p);
    STRATA_CUDA_TRY(moe_route_exact(L, x, tokens, logits, sg, tail, ids, weights, grid, s, err));

    medium::Params prm;
    std::memset(&prm, 0, sizeof prm);
    prm.L = L;
    prm.x = x;
    prm.tokens = tokens;
    prm.y = y;
    prm.ids = ids;
    prm.weights = weights;
    prm.sg = sg;
    prm.xrec = xrec;
    prm.part = part;
    prm.sync = sync;
    prm.err = err;
    prm.spin_limit = 1ull << 20;  // grid waits sleep 32 ns per try; an mbarrier try suspends for a short, system-defined time
    if (!moe_tensor_maps(L, &prm.maps)) return cudaErrorInvalidValue;
    if (L.width == 2048 && L.ff == 512) return launch_medium<2048, 512>(prm, grid, s);
    if (L.width == 2560 && L.ff == 640) return launch_medium<2560, 640>(prm, grid, s);
    return cudaErrorInvalidValue;
}

}  // namespace strata
