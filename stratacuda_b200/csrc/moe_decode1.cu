// Fused mixture-of-experts layer for ONE decode token (BASELINE config 2 at batch 1): one
// persistent launch of 8-CTA thread-block clusters, one CTA per SM (8 warps). Same arithmetic as
// the batch decode kernel (csrc/moe_fast.cu: u8 x s8 mma.sync on the raw 2-bit codes,
// activations and hidden values as three signed 8-bit digits, routing bit-identical to the
// reference).
//
// Work split (slot 0 = the shared expert, slot s >= 1 = the s-th valid selection in k order):
//   * cluster s < 11 handles slot s. CTA rank j computes hidden values [64 j, 64 j + 64): warp
//     w one gate/up tile (16 interleaved gate/up blob rows 16 (8 j + w) .., full width, one TMA
//     request), silu(gate) * up for its 8 values into the CTA's shared memory. A cluster barrier,
//     then every CTA of the cluster gathers the slot's F hidden values from its peers' shared
//     memory (distributed shared memory: no global round trip) and computes output rows
//     [256 j, 256 j + 256) of the slot's down projection (32 rows per warp; the rows' codes are
//     one contiguous 32 KB block, fetched as four 8 KB boxes into the gate/up stages the warps
//     have finished with).
//   * the routed clusters store their rows as tagged words (below); cluster 0 (the shared
//     expert, whose work needs no routing and runs while the grid exchanges logits) collects
//     them and writes y in the reference's combine order (kernels/strata.cu:360-365: shared *
//     sigmoid(gate), then + part_k * w_k for k in order). y has the same bits run to run.
//   * router logits: rows r = rc, rc + R, ... (rc = the CTA's index among the CTAs of clusters
//     >= 1, R their count) in the reference's exact order (kernels/strata.cu:156-165), from
//     router rows staged before griddepcontrol.wait (they are weights). Clusters >= 11 only
//     compute router rows.
// Grid-wide exchanges (logits, the routed slots' rows) use tagged words: an F32 value in the low
// half of an 8-byte word, this launch's tag in the high half. A reader polls the words until
// each carries the tag: no arrival counters, no fences between data and flags. The words live
// in a buffer of the context's own (zeroed once, written only by this kernel), and the tag is
// the launch count + 1, so an older word never carries the current tag.
//
// Every wait on the GPU is bounded except the cluster barriers, which every CTA of clusters
// 0..10 passes at the same two points on every path (a timed-out wait only sets the error).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "q2mma.cuh"
#include "route.cuh"

namespace strata {
namespace d1 {

using namespace q2;

constexpr int kMaxSlots = 11;  // the shared expert + topK <= 10 routed experts
constexpr int kCluster = 8;    // CTAs per slot: F / 64 hidden groups
constexpr int kClusters = 15;  // clusters of the grid (15 x 8 CTAs fit one per SM on a B200)
constexpr int kRowWarps = 5;   // router rows per CTA of clusters >= 1
constexpr int kH = 2048, kF = 512;

struct Geo {
    static constexpr int NG = kH / 64;       // scale groups of a gate/up row
    static constexpr int CH = kH / 512;      // 128-byte chunks of a gate/up row
    static constexpr int DG = kF / 64;       // scale groups of a down row
    static constexpr int TILE = CH * 2048;   // gate/up tile: 16 rows x H/4 bytes
    static constexpr int TSC = 16 * NG * 2;  // its FP16 scales (bytes)
    static constexpr int DROWS = kH / kCluster;  // down rows per CTA (256)
    static_assert(kF / 64 == kCluster && kF / 4 == 128, "one CTA per 64 hidden values; 128-byte down rows");
    static_assert(TILE == kH * 4, "a router row fills one gate/up stage");
    static_assert(DROWS == 4 * 64, "the CTA's down rows are four 64-row boxes");
    static_assert(DROWS == kThreads, "the collector takes one row per thread");
    static_assert(NG * 4 == 128 && kThreads == 256, "the x digits' 128 blocks on the upper half of the threads");
};

struct Params {
    MoeLayerDev L;
    const float *x;
    float *y;
    int *ids;
    float *weights;
    unsigned long long *lgx;   // [513] tagged router logits (the shared-gate logit at [experts]), then [kPresence]
                               // presence words: one per CTA, stored as soon as it holds the tag
    unsigned long long *part;  // [kMaxSlots - 1][H] tagged down rows of the routed slots
    unsigned *sync;            // [0] launch count (tag = count + 1)
    unsigned *err;
    unsigned long long spin_limit;
    CUtensorMap tm_gu[2];  // gate/up codes {128, 2F rows, H/512 chunks, experts}, box {128, 16, H/512, 1}; [0] routed, [1] shared
    CUtensorMap tm_dn[2];  // down codes {128, H rows, experts}, box {128, 64, 1}; 128-byte swizzle
};

struct Smem {
    using G1 = Geo;
    unsigned char gu[kWarps][G1::TILE];  // warp w's gate/up tile; first the router rows (clusters >= 1),
                                         // later stages 0..3 take the CTA's down rows (64 each)
    alignas(16) unsigned short gus[kWarps][G1::TSC / 2];
    alignas(16) unsigned short dns[G1::DROWS * G1::DG];  // the CTA's down rows' scales
    union U {
        float x[kH];  // before the exchange of logits
        struct R {
            float lg[512];
            alignas(16) unsigned long long cand[8 * 32];
            float red[kWarps];
            float sel[32];
        } r;  // routing
        struct D {
            float h[kF];                   // the slot's hidden values, gathered from the cluster
            uint2 hf[G1::DG * 2 * 4 * 3];  // their digits [group][half][q][digit]
            int hsum[G1::DG];
            float hinv;
        } d;  // down
    } u;
    uint2 xf[G1::NG * 2 * 4 * 3];  // x digits [group][half][q][digit]
    int xsum[G1::NG];
    float hloc[64];  // this CTA's hidden values (read by the cluster's CTAs)
    float res[G1::DROWS];
    int ids[32];
    float wts[32];
    short slot_expert[kMaxSlots];
    signed char slot_of_k[32];
    int n_slots, nzc, abort_flag;
    unsigned armed;  // barriers with copies issued: bit w gate/up stage w, 8 + st down stage st, 12 down scales, 13 router rows, 14 x
    unsigned tag, xmax;
    float xscale, sgw, sg_raw;
    unsigned long long exp_tab[32];  // the expf table (common.cuh), staged for the routing
    unsigned long long bar_gu[kWarps], bar_dn[4], bar_dns, bar_rows, bar_x;
};

// ---- tagged exchange words: one 8-byte store (single-copy atomic), relaxed loads that reach L2
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, unsigned tag) {
    __stcg(p, ((unsigned long long)tag << 32) | __float_as_uint(v));
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Bounded poll of one word; false (v untouched) when the limit ran out.
__device__ __forceinline__ bool poll_tagged(const unsigned long long *p, unsigned tag, unsigned long long limit, float &v) {
    for (unsigned long long i = 0;; ++i) {
        const unsigned long long w = ld_relaxed64(p);
        if ((unsigned)(w >> 32) == tag) {
            v = __uint_as_float((unsigned)w);
            return true;
        }
        if (i > limit) return false;
        if (i > 16) __nanosleep(64);
    }
}
// ---- clusters
__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cluster_id() {
    unsigned r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {  // every thread of every CTA of the cluster
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Execution-only cluster barrier: every thread has arrived, nothing ordered (the peers' reads of
// this CTA's shared memory have completed: their values were used before the arrival).
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_peer(const float *local, unsigned rank) {  // the same variable in CTA `rank`'s shared memory
    unsigned remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

__device__ __forceinline__ unsigned cluster_size() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// The cluster shape is part of the kernel (not of a launch attribute), so that every launch of
// it, including a replay by a profiler, has 8-CTA clusters: the distributed-shared-memory reads
// name ranks 0..7.
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads, 1) k_moe_decode1(const __grid_constant__ Params P) {
    // a launch of another shape would make the peers' ranks, the slots and the router rows
    // wrong: report it and touch nothing
    if (cluster_size() != (unsigned)kCluster || gridDim.x != (unsigned)(kClusters * kCluster) || blockDim.x != (unsigned)kThreads) {
        if (threadIdx.x == 0) raise_error(P.err, kErrIndex);
        return;
    }
    using G1 = Geo;
    constexpr int NG = G1::NG, CH = G1::CH, DG = G1::DG, DROWS = G1::DROWS;
    extern __shared__ unsigned char smem_raw[];
    auto &S = *reinterpret_cast<Smem *>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
    const MoeLayerDev &L = P.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const int G = gridDim.x, E = L.experts, K = L.topK;
    const int cl = (int)cluster_id(), j = (int)cluster_rank();
    const long long gu_scales_b = 3LL * kF * kH / 4, d_scales_b = gu_scales_b + 2LL * kF * (kH / 64) * 2;
    const bool slot_cluster = cl < kMaxSlots;  // passes the two cluster barriers
    // router rows: the CTAs of clusters >= 1, CTA rc takes rows rc, rc + R, ...
    const int rc = cl >= 1 ? (int)blockIdx.x - kCluster : -1, R = G - kCluster;
    const int nrows = rc < 0 ? 0 : min(kRowWarps, max(0, (E + 1 - rc + R - 1) / R));

    auto blob_of = [&](int slot) -> const unsigned char * {
        return reinterpret_cast<const unsigned char *>(slot == 0 ? L.shared_blob : L.blobs + (long long)S.slot_expert[slot] * L.blob_words);
    };
    // copies (one thread each); every mbarrier is armed at most once per launch (parity 0)
    auto issue_tile = [&](int w, int slot) {  // warp w's tile of this CTA: blob rows 16 (8 j + w) ..
        const int m = slot == 0 ? 1 : 0, e = slot == 0 ? 0 : S.slot_expert[slot], tt = 8 * j + w;
        atomicOr(&S.armed, 1u << w);
        mbar_expect(&S.bar_gu[w], G1::TILE + G1::TSC);
        tma_4d(S.gu[w], &P.tm_gu[m], 0, 16 * tt, 0, e, &S.bar_gu[w]);
        bulk_copy(S.gus[w], blob_of(slot) + gu_scales_b + (long long)16 * tt * NG * 2, G1::TSC, &S.bar_gu[w]);
    };
    auto issue_down = [&](int st, int slot) {  // down rows DROWS j + 64 st .. (64 rows) into stage st
        const int m = slot == 0 ? 1 : 0, e = slot == 0 ? 0 : S.slot_expert[slot];
        atomicOr(&S.armed, 1u << (8 + st));
        mbar_expect(&S.bar_dn[st], 8192);
        tma_3d(S.gu[st], &P.tm_dn[m], 0, DROWS * j + 64 * st, e, &S.bar_dn[st]);
    };
    auto issue_down_scales = [&](int slot) {
        atomicOr(&S.armed, 1u << 12);
        mbar_expect(&S.bar_dns, DROWS * DG * 2);
        bulk_copy(S.dns, blob_of(slot) + d_scales_b + (long long)DROWS * j * DG * 2, DROWS * DG * 2, &S.bar_dns);
    };
    auto wait_bar = [&](unsigned long long *bar) -> bool {  // parity 0, bounded
        for (unsigned long long i = 0;; ++i) {
            if (mbar_try(bar, 0)) return true;
            if (i > P.spin_limit) return false;
        }
    };
    auto warp_wait = [&](unsigned long long *bar) -> bool {  // warp-uniform result
        const bool ok = __all_sync(0xffffffffu, S.abort_flag == 0 && wait_bar(bar));
        if (!ok && lane == 0) atomicOr(&S.abort_flag, 1);
        return ok;
    };

    // ------------------------------------------------------------------ entry: weights only
    if (tid == 0) {
        for (int w = 0; w < kWarps; ++w) mbar_init(&S.bar_gu[w], 1);
        for (int st = 0; st < 4; ++st) mbar_init(&S.bar_dn[st], 1);
        mbar_init(&S.bar_dns, 1);
        mbar_init(&S.bar_rows, 1);
        mbar_init(&S.bar_x, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
        S.armed = 0u;
        S.xmax = 0u;
        S.n_slots = 0;
        S.slot_expert[0] = 0;
        for (int i = 0; i < 2; ++i) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.tm_gu[i])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<unsigned long long>(&P.tm_dn[i])) : "memory");
        }
        if (cl == 0) {  // the shared expert's tiles and down scales: no routing needed
            for (int w = 0; w < kWarps; ++w) issue_tile(w, 0);
            issue_down_scales(0);
        } else if (nrows > 0) {
            S.armed |= 1u << 13;
            mbar_expect(&S.bar_rows, (unsigned)(nrows * kH * 4));
            for (int w = 0; w < nrows; ++w) {
                const int r = rc + R * w;
                bulk_copy(S.gu[w], r < E ? L.router + (long long)r * kH : L.shared_gate, kH * 4, &S.bar_rows);
            }
        }
    }
    if (tid < 32) S.exp_tab[tid] = __ldg(&c_exp2_tab[tid]);
    __syncthreads();

    // ------------------------------------------------------------------ phase 1: x, logits, digits
    // Everything above read only the layer's weights. Wait for the previous kernel on the stream
    // (programmatic dependent launch) before x, the exchange words or the counters, and let the
    // next launch get ready.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 32) S.tag = __ldcg(&P.sync[0]) + 1u;  // the previous launch's count is final (griddepcontrol.wait)
    const bool x_bulk = (reinterpret_cast<unsigned long long>(P.x) & 15ull) == 0;
    if (x_bulk) {
        if (tid == 0) {
            atomicOr(&S.armed, 1u << 14);
            mbar_expect(&S.bar_x, kH * 4);
            bulk_copy(S.u.x, P.x, kH * 4, &S.bar_x);
        }
        warp_wait(&S.bar_x);
    } else {
        for (int i = tid; i < kH; i += kThreads) S.u.x[i] = __ldg(P.x + i);
    }
    __syncthreads();
    if (tid == 0) st_tagged(&P.lgx[513 + blockIdx.x], 0.0f, S.tag);  // this CTA holds the tag
    // The router rows first (they are on the critical path; the x digits are not). Thread t of
    // warp w holds the reference's lanes 2t and 2t + 1 of row rc + R w (kernels/strata.cu:156-165:
    // lane l adds x[k] w[k] over k = l mod 64 in increasing k, then the tree partial[l] +=
    // partial[l + s], s = 32 .. 1): one 8-byte load of each operand per step; the tree's level s
    // is a shuffle by s / 2 threads, the last level joins the two lanes of thread 0.
    if (warp < nrows) {
        const int r = rc + R * warp;
        if (warp_wait(&S.bar_rows)) {
            const float2 *W2 = reinterpret_cast<const float2 *>(S.gu[warp]);
            const float2 *X2 = reinterpret_cast<const float2 *>(S.u.x);
            float ev = 0.0f, od = 0.0f;
#pragma unroll 8
            for (int c = 0; c < NG; ++c) {
                const float2 w = W2[32 * c + lane], xv = X2[32 * c + lane];
                ev = __fadd_rn(ev, __fmul_rn(w.x, xv.x));
                od = __fadd_rn(od, __fmul_rn(w.y, xv.y));
            }
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) {
                ev = __fadd_rn(ev, __shfl_down_sync(0xffffffffu, ev, s));
                od = __fadd_rn(od, __shfl_down_sync(0xffffffffu, od, s));
            }
            const float v = __fadd_rn(ev, od);
            if (lane == 0) st_tagged(&P.lgx[r], r < E && L.bias ? __fadd_rn(v, L.bias[r]) : v, S.tag);
        }
    }
    {  // largest |x| (NaN ignored, as fmaxf; order-free)
        float mx = 0.0f;
        for (int i = tid; i < kH; i += kThreads) mx = fmaxf(mx, fabsf(S.u.x[i]));
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
        if (lane == 0) atomicMax(&S.xmax, __float_as_uint(mx));
    }
    __syncthreads();
    if (slot_cluster)  // x digits: block b = (group, q) of 16 elements, one per thread of warps 4..7 (0.. compute router rows)
        for (int b = tid ^ 128; b < NG * 4; b += kThreads) {
            const int grp = b >> 2, qq = b & 3;
            const int k = scale_exp(__uint_as_float(S.xmax));
            const float mul = pow2f(k);
            if (b == 0) S.xscale = pow2f(-k);
            const float4 *src = reinterpret_cast<const float4 *>(S.u.x + 64 * grp + 16 * qq);
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
            if (qq == 0) S.xsum[grp] = part;
            block_frags(v, &S.xf[((grp * 2 + 0) * 4 + qq) * 3], &S.xf[((grp * 2 + 1) * 4 + qq) * 3]);
        }
    __syncthreads();  // logits stored, x digits complete

    // ------------------------------------------------------------------ gate/up of warp w's tile
    // One 128-byte chunk (8 scale groups) of the tile's 16 rows: the partial sum of row g (lane
    // q = 0) or row g + 8 (lane q = 1); lanes q = 2, 3 hold nothing of use. The MMA leaves digits
    // 0 and 1 of rows g and g + 8 in lane q = 0 and digit 2 in lane q = 1: the pair swaps the
    // pieces of the other one's row (one shuffle), then each lane finishes one row.
    auto gu_chunk = [&](int w, int c, float &acc) {
        acc = 0.0f;
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        const bool live = g < 3;  // B columns 0..2: the token's three digits; 3..7 zero
        const unsigned base = smem_u32(S.gu[w] + 2048 * c);
        const unsigned short *scl = S.gus[w] + 8 * c;  // row r: scl[r * NG + group in chunk]
        unsigned wd[4][4];
#pragma unroll
        for (int gp = 0; gp < 4; ++gp) {
            const int cc = 2 * gp + (lane >> 4);
            ldsm_x4(base + r * 128 + ((cc ^ (r & 7)) << 4), wd[gp][0], wd[gp][1], wd[gp][2], wd[gp][3]);
        }
        const bool odd = q & 1;
        float s_row[8];  // this lane's row: 8 FP16 scales, one 16-byte load
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
        uint2 bf[8][2];
#pragma unroll
        for (int gl = 0; gl < 8; ++gl)
#pragma unroll
            for (int h = 0; h < 2; ++h) bf[gl][h] = live ? S.xf[(((8 * c + gl) * 2 + h) * 4 + q) * 3 + g] : make_uint2(0u, 0u);
        int c4[8][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int gl = 0; gl < 8; ++gl) {
                const unsigned wl = wd[gl >> 1][(gl & 1) ? 2 : 0], wh = wd[gl >> 1][(gl & 1) ? 3 : 1];
                imma_acc(h > 0, c4[gl], (wl >> (4 * h)) & 0x03030303u, (wh >> (4 * h)) & 0x03030303u, (wl >> (4 * h + 2)) & 0x03030303u,
                     (wh >> (4 * h + 2)) & 0x03030303u, bf[gl][h].x, bf[gl][h].y);
            }
#pragma unroll
        for (int gl = 0; gl < 8; ++gl) {
            const int send = odd ? c4[gl][0] : c4[gl][2] + 256 * c4[gl][3];
            const int recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const int v = odd ? recv + 65536 * c4[gl][2] : c4[gl][0] + 256 * c4[gl][1] + 65536 * recv;
            acc = fmaf(s_row[gl], (float)(v - S.xsum[8 * c + gl]), acc);
        }
    };
    // Warp w's tile: chunk sums added in chunk order; lane (g, q = 0) holds row g, lane (g, q = 1)
    // row g + 8; gate row g (even) pairs with up row g + 1 four lanes down. Hidden value of row g:
    // 8 w + g / 2 (+ 4 for row g + 8) of this CTA's 64. Then the stage is free: warps 0..3 fetch
    // the CTA's down rows into theirs.
    auto gate_up = [&](int w, int slot) {
        if (warp_wait(&S.bar_gu[w])) {
            float acc = 0.0f;
#pragma unroll 1
            for (int c = 0; c < CH; ++c) {
                float pc;
                gu_chunk(w, c, pc);
                acc = __fadd_rn(acc, pc);
            }
            const float gv = acc * S.xscale;
            const float up = __shfl_down_sync(0xffffffffu, gv, 4);
            if (q < 2 && !(g & 1)) S.hloc[8 * w + 4 * q + (g >> 1)] = __fmul_rn(ref_silu(gv, S.exp_tab), up);
        }
        __syncwarp();
        if (w < 4 && lane == 0) {  // the stage was last read through the generic proxy (ldmatrix)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_down(w, slot);
        }
    };

    // ------------------------------------------------------------------ the shared expert (cluster 0)
    // Its tiles were requested at entry; it needs no routing, so it runs while the grid's logits
    // are exchanged.
    if (cl == 0) gate_up(warp, 0);

    // ------------------------------------------------------------------ phase 2: routing (clusters 0..10)
    if (slot_cluster) {
        // the grid-wide exchange: every CTA polls the 513 tagged logit words until each carries
        // this launch's tag; a thread requests all of its words at once and re-reads only those
        // still without the tag (one L2 round trip once they are there; no arrival counter)
        float *lg = S.u.r.lg;
        {
            constexpr int NW = (513 + kThreads - 1) / kThreads;
            unsigned miss = 0u;
#pragma unroll
            for (int i = 0; i < NW; ++i) {
                const int e = tid + kThreads * i;
                if (e <= E) miss |= 1u << i;
                else if (e < 512) lg[e] = 0.0f;
            }
            for (unsigned long long it = 0; miss; ++it) {
                unsigned long long w[NW];
#pragma unroll
                for (int i = 0; i < NW; ++i)
                    if (miss >> i & 1u) w[i] = ld_relaxed64(&P.lgx[tid + kThreads * i]);
#pragma unroll
                for (int i = 0; i < NW; ++i)
                    if ((miss >> i & 1u) && (unsigned)(w[i] >> 32) == S.tag) {
                        const int e = tid + kThreads * i;
                        const float v = __uint_as_float((unsigned)w[i]);
                        if (e == E) S.sg_raw = v;
                        if (e < 512) lg[e] = e < E ? v : 0.0f;
                        miss &= ~(1u << i);
                    }
                if (!miss) break;
                if (it > P.spin_limit) {
                    atomicOr(&S.abort_flag, 1);
                    break;
                }
                if (it > 16) __nanosleep(64);
            }
        }
        if (tid == 0) S.nzc = 0;
        if (cl == 0 && j == 0)  // every CTA of the grid holds this launch's tag (see the exit)
            for (int b = tid; b < G; b += kThreads) {
                float v;
                if (!poll_tagged(&P.lgx[513 + b], S.tag, P.spin_limit, v)) atomicOr(&S.abort_flag, 1);
            }
        __syncthreads();
        if (!S.abort_flag) {
            // This cluster's slot is the cl-th valid selection: as soon as the ids are final (before
            // the weights), lane 0 of every warp finds it and requests the warp's tile (its stage
            // held a router row, read through the generic proxy); the last warp also the down scales.
            route_group<8>(S.u.r.lg, E, K, S.u.r.red, S.u.r.cand, &S.nzc, S.ids, S.u.r.sel, S.wts, 1, S.exp_tab, [&] {
                if (cl >= 1 && lane == 0) {
                    int e_cl = -1;
                    if (S.nzc >= K) {  // every selection valid: slot cl is selection cl - 1
                        if (cl <= K) e_cl = S.ids[cl - 1];
                    } else {
                        int n = 0;
                        for (int k = 0; k < K; ++k) {
                            const int e = S.ids[k];
                            if (e >= 0 && e < E && ++n == cl) e_cl = e;
                        }
                    }
                    if (e_cl >= 0) {
                        S.slot_expert[cl] = (short)e_cl;  // the same value from every warp
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        issue_tile(warp, cl);
                        if (warp == kWarps - 1) issue_down_scales(cl);
                    }
                }
            });
            // (route_group ends with a barrier of all eight warps: every thread sees ids and weights.)
            if (tid == 0) {  // slot s >= 1: the s-th valid selection (ids of one token are distinct)
                int n = 1;
                for (int k = 0; k < K; ++k) {
                    const int e = S.ids[k];
                    if (e >= 0 && e < E) {
                        S.slot_expert[n] = (short)e;
                        S.slot_of_k[k] = (signed char)n;
                        ++n;
                    } else {
                        S.slot_of_k[k] = -1;
                    }
                }
                S.n_slots = n;
            }
            if (tid == 32) S.sgw = ref_sigmoid(S.sg_raw, S.exp_tab);
            if (cl == 0 && j == 0)
                for (int k = tid; k < K; k += kThreads) {
                    P.ids[k] = S.ids[k];
                    P.weights[k] = S.wts[k];
                }
        }
        __syncthreads();
    }
    const bool active = slot_cluster && !S.abort_flag && cl < S.n_slots;  // S.n_slots stays 0 on an abort

    // ------------------------------------------------------------------ phase 3: the routed slot's tiles
    if (active && cl >= 1) gate_up(warp, cl);
    __syncthreads();

    // ------------------------------------------------------------------ phase 4: down rows of the slot
    if (slot_cluster) cluster_sync_all();  // A: every CTA of the cluster has its 64 hidden values in hloc
    if (active) {
        // the slot's hidden values from the cluster's CTAs (two loads per thread; every warp reading
        // all 512 for itself from the peers was 6 us slower), then warp 0 forms their digits
        for (int i = tid; i < kF; i += kThreads) S.u.d.h[i] = ld_peer(&S.hloc[i % 64], (unsigned)(i / 64));
        __syncthreads();
        if (warp == 0) {  // digits of the slot's hidden values: lane = block (group lane / 4, q) of 16
            float hv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) hv[i] = S.u.d.h[16 * lane + i];
            float mx = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(hv[i]));
#pragma unroll
            for (int sft = 16; sft > 0; sft >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, sft));
            const int k = scale_exp(mx);
            const float mul = pow2f(k);
            int v[16];
            int part = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                v[i] = __float2int_rn(hv[i] * mul);
                part += v[i];
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            const int grp = lane >> 2;
            if (q == 0) S.u.d.hsum[grp] = part;
            if (lane == 0) S.u.d.hinv = pow2f(-k);
            block_frags(v, &S.u.d.hf[((grp * 2 + 0) * 4 + q) * 3], &S.u.d.hf[((grp * 2 + 1) * 4 + q) * 3]);
        }
        __syncthreads();
        // warp w: the CTA's rows 32 w .. 32 w + 31 (two 16-row tiles), in stage (32 w) / 64
        const int st = warp >> 1;
        if (warp_wait(&S.bar_dn[st]) && warp_wait(&S.bar_dns)) {
            const unsigned base = smem_u32(S.gu[st]);
            const int r16 = (lane & 7) + ((lane >> 3) & 1) * 8;
            const bool live = g < 3;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int row0 = 32 * warp + 16 * t;  // the CTA's row of this tile's first row
                const int brow = row0 - 64 * st + r16;  // row in the stage's box
                // lane q = 0: row row0 + g, lane q = 1: row row0 + g + 8 (the digit pieces swapped as in
                // the gate/up chunks)
                const bool odd = q & 1;
                const int myrow = row0 + g + (odd ? 8 : 0);
                float acc = 0.0f;
#pragma unroll
                for (int gp = 0; gp < DG / 2; ++gp) {
                    unsigned w0, w1, w2, w3;
                    const int cc = 2 * gp + (lane >> 4);
                    ldsm_x4(base + brow * 128 + ((cc ^ (brow & 7)) << 4), w0, w1, w2, w3);
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int gl = 2 * gp + hh;
                        const unsigned wl = hh ? w2 : w0, wh = hh ? w3 : w1;
                        int c4[4];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const uint2 b = live ? S.u.d.hf[((gl * 2 + h) * 4 + q) * 3 + g] : make_uint2(0u, 0u);
                            imma_acc(h > 0, c4, (wl >> (4 * h)) & 0x03030303u, (wh >> (4 * h)) & 0x03030303u, (wl >> (4 * h + 2)) & 0x03030303u,
                                 (wh >> (4 * h + 2)) & 0x03030303u, b.x, b.y);
                        }
                        const int send = odd ? c4[0] : c4[2] + 256 * c4[3];
                        const int recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        const int v = odd ? recv + 65536 * c4[2] : c4[0] + 256 * c4[1] + 65536 * recv;
                        const float sc = __half2float(__ushort_as_half(S.dns[myrow * DG + gl]));
                        acc = fmaf(sc, (float)(v - S.u.d.hsum[gl]), acc);
                    }
                }
                if (q < 2) {
                    const float val = acc * S.u.d.hinv;
                    if (cl == 0) S.res[myrow] = val;
                    else st_tagged(P.part + (long long)(cl - 1) * kH + DROWS * j + myrow, val, S.tag);  // tagged, for cluster 0
                }
            }
        }
        __syncthreads();
        // cluster 0: y rows DROWS j .. in the reference's combine order (kernels/strata.cu:360-365)
        if (cl == 0 && !S.abort_flag) {
            // every routed slot's word of this row requested at once, then re-read only while some
            // lack the tag (one L2 round trip per pass instead of one per slot)
            const int row = tid;  // kThreads == DROWS
            const unsigned long long *src = P.part + DROWS * j + row;
            float pv[kMaxSlots - 1];
            unsigned missing = 0;
            for (int s = 1; s < S.n_slots; ++s) missing |= 1u << s;
            for (unsigned long long i = 0; missing; ++i) {
                unsigned long long w[kMaxSlots - 1];
#pragma unroll
                for (int s = 1; s < kMaxSlots; ++s)
                    if (missing >> s & 1u) w[s - 1] = ld_relaxed64(src + (long long)(s - 1) * kH);
#pragma unroll
                for (int s = 1; s < kMaxSlots; ++s)
                    if ((missing >> s & 1u) && (unsigned)(w[s - 1] >> 32) == S.tag) {
                        pv[s - 1] = __uint_as_float((unsigned)w[s - 1]);
                        missing &= ~(1u << s);
                    }
                if (!missing) break;
                if (i > P.spin_limit) {
                    atomicOr(&S.abort_flag, 1);
                    break;
                }
                __nanosleep(64);
            }
            if (!missing) {  // kernels/strata.cu:360-365
                float v = __fmul_rn(S.res[row], S.sgw);
                for (int k = 0; k < K; ++k) {
                    const int s = S.slot_of_k[k];
                    if (s > 0) v = __fadd_rn(v, __fmul_rn(pv[s - 1], S.wts[k]));
                }
                P.y[DROWS * j + row] = v;
            }
        }
    }
    if (slot_cluster) cluster_sync_relaxed();  // B: no CTA leaves while a peer may still read its hloc

    // ------------------------------------------------------------------ exit
    __syncthreads();
    if (tid == 0) {
        if (S.abort_flag) {  // leave no copy in flight: wait (bounded) for every barrier armed above
            const unsigned a = S.armed;
            for (int w = 0; w < kWarps; ++w)
                if (a >> w & 1u) wait_bar(&S.bar_gu[w]);
            for (int st = 0; st < 4; ++st)
                if (a >> (8 + st) & 1u) wait_bar(&S.bar_dn[st]);
            if (a >> 12 & 1u) wait_bar(&S.bar_dns);
            if (a >> 13 & 1u) wait_bar(&S.bar_rows);
            if (a >> 14 & 1u) wait_bar(&S.bar_x);
            raise_error(P.err, kErrWaitTimeout);
        }
        // The launch count moves on (the next launch's tag) once no CTA can still need the old
        // count: CTA 0 of cluster 0 has seen every CTA's presence word carry this launch's tag.
        // The next launch reads the count after griddepcontrol.wait, i.e. after every CTA of this
        // one is gone. Should the presence wait have run out, a late CTA of this launch may read
        // the new count and store words with tag + 1: the count then skips that tag.
        if (cl == 0 && j == 0) P.sync[0] = S.abort_flag ? S.tag + 1u : S.tag;
    }
}

}  // namespace d1

static_assert(sizeof(d1::Smem) + 1024 <= 113 * 1024, "two CTAs per SM: the next layer's launch overlaps this one's tail");

bool moe_decode1_supported(int tokens, int width, int ff, int experts, int topK, int grid) {
    // one token, the workload geometry, <= 10 routed experts, the router rows covered by the CTAs
    // of clusters 1.., the grid's clusters one CTA per SM
    return tokens == 1 && width == d1::kH && ff == d1::kF && topK >= 1 && topK <= d1::kMaxSlots - 1 && experts >= 1 &&
           experts + 1 <= (d1::kClusters - 1) * d1::kCluster * d1::kRowWarps && grid >= d1::kClusters * d1::kCluster;
}

constexpr int kPresence = d1::kClusters * d1::kCluster;  // one presence word per CTA
static size_t lgx_words() { return (513 + kPresence + 31) & ~size_t(31); }
size_t moe_decode1_xchg_bytes() { return sizeof(unsigned long long) * (lgx_words() + (size_t)(d1::kMaxSlots - 1) * d1::kH); }

namespace {
int g_d1_coop = -1;  // the cooperative attribute together with clusters: -1 untried, 1 accepted, 0 refused

cudaError_t launch_d1(const d1::Params &p, cudaStream_t s) {
    const size_t smem = sizeof(d1::Smem) + 1024;  // + slack for the 1024-byte alignment
    static int device_ready = -1;
    int dev = 0;
    STRATA_CUDA_TRY(cudaGetDevice(&dev));
    if (device_ready != dev) {
        STRATA_CUDA_TRY(cudaFuncSetAttribute(d1::k_moe_decode1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        device_ready = dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d1::kClusters * d1::kCluster);
    cfg.blockDim = dim3(q2::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];  // the 8-CTA clusters come from the kernel's __cluster_dims__
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;  // the grid-wide exchange needs every CTA resident
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    if (g_d1_coop != 0) {
        cfg.numAttrs = 2;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, d1::k_moe_decode1, p);
        if (e == cudaSuccess || g_d1_coop == 1) {
            g_d1_coop = e == cudaSuccess ? 1 : g_d1_coop;
            return e;
        }
        cudaGetLastError();  // refused with clusters: the grid (one CTA per SM, under the co-resident
        g_d1_coop = 0;       // cluster count) is resident without the guarantee
    }
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, d1::k_moe_decode1, p);
}
}  // namespace

cudaError_t moe_forward_decode1(const MoeLayerDev &L, const float *x, float *y, int *ids, float *weights, void *xchg, unsigned *sync,
                                int grid, cudaStream_t s, unsigned *err) {
    (void)grid;
    d1::Params prm;
    std::memset(&prm, 0, sizeof prm);
    prm.L = L;
    prm.x = x;
    prm.y = y;
    prm.ids = ids;
    prm.weights = weights;
    prm.lgx = static_cast<unsigned long long *>(xchg);
    prm.part = prm.lgx + lgx_words();
    prm.sync = sync;
    prm.err = err;
    prm.spin_limit = 1ull << 20;
    MoeMaps maps;
    CUtensorMap gu16[2];
    if (!moe_decode_maps(L, gu16, &maps)) return cudaErrorInvalidValue;
    prm.tm_gu[0] = maps.gu16r[0];
    prm.tm_gu[1] = maps.gu16r[1];
    prm.tm_dn[0] = maps.dn64[0];
    prm.tm_dn[1] = maps.dn64[1];
    return launch_d1(prm, s);
}

}  // namespace strata
