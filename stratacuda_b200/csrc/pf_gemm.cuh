// Grouped Q2 x FP16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), the engine of
// the prefill path.
//
// One tile = (expert slot, 128 weight rows, up to 192 rows of the B matrix). D[128][N] =
// A[128][K] . B[N][K]^T accumulates in TMEM (FP32, 128 lanes x N columns). A is the slot's
// Q2 weights, dequantised to FP16 straight into TMEM (tcgen05.st), where the MMA reads it:
// w = (code - 1) * scale, exact in FP16 (the scale is an FP16 and code - 1 is in {-1, 0, 1,
// 2}). Keeping A out of shared memory leaves shared-memory bandwidth to B alone (writing and
// re-reading a dequantised A tile there cost as much as B itself). B rows are FP16
// activations (gate/up: the tokens of the slot, scaled per token by a power of two; down:
// the hidden values), by TMA into a 128-byte-swizzled K-major ring.
//
// Persistent kernel, one CTA per SM, tiles dealt round-robin (tile i on CTA i % G). Tile i is
// chunk i / NM of the chunk list (slot, first B row, rows) and weight block i % NM; the chunk
// list is ordered by decreasing rows, so the deal approximates longest-first. Warp roles:
//   warp 0      TMA producer of B: per 64-column K-block the B rows (64-row boxes, then
//               16-row boxes for the rest; 128-byte swizzle)
//   warp 18     TMA producer of A: per tile the rows' FP16 scales (one bulk copy); per
//               256-column super-block the packed codes (one 128-row x 64-byte box, 64-byte
//               swizzle). Its own thread, so the codes run ahead of the dequantisers while the
//               B producer waits for free stages
//   warp 1      allocates TMEM (512 columns: two 192-column accumulators and four 32-column
//               A stages) and issues the MMAs from one thread: per K-block four tcgen05.mma
//               (K = 16, A from TMEM, B from shared memory), then tcgen05.commit
//   warps 2-9   dequantise: warp w writes TMEM lanes 32 (w % 4) .. (a warp reaches only its
//               lane quarter): thread = one A row and half of its 64 codes of a K-block, 16
//               32-bit columns of two FP16 each
//   warps 10-17 epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes 32 (w % 4) ..;
//               warps 10-13 take the even 32-column chunks, 14-17 the odd ones), gate/up:
//               hidden = silu(gate) * up -> FP16 rows; down: weighted rows added to y
// The accumulators are double-buffered, so a tile's epilogue overlaps the next tile's MMAs.
// Every wait is bounded: past the limit the CTA records kErrWaitTimeout and all roles leave
// (the producer and the MMA thread first wait, bounded, for their own operations in flight).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace strata {
namespace pf {

constexpr int kGemmWarps = 19;
constexpr int kCodeWarp = 18;   // producer of scales and packed codes
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kDeqThreads = 256;  // warps 2-9
constexpr int kEpiWarp0 = 10;     // warps 10-17
constexpr int kEpiThreads = 256;
constexpr int kStages = 5;        // B stages
constexpr int kAStages = 4;       // dequantised-A stages (TMEM)
constexpr int kApkStages = 4;     // packed-code super-blocks
constexpr int kMaxN = 192;        // B rows per tile
constexpr int kAccCols = 192;     // TMEM columns per accumulator
constexpr int kACol0 = 2 * kAccCols;  // first TMEM column of the A stages (32 columns each)
constexpr int kKBlock = 64;       // K elements per stage (one scale group, one 128-byte swizzle row)
constexpr int kSuper = 4;         // K-blocks per packed super-block (256 codes = 64 bytes per row)

enum Mode { kGateUp = 0, kDown = 1 };

struct Chunk {
    int slot;   // expert id, or -1 for the shared expert
    int row0;   // first B row
    int n;      // B rows (1 .. kMaxN)
    int pad;
};
struct Tile {
    int slot, mtile, row0, n;
};

struct GemmParams {
    const Chunk *chunks;
    const int *n_chunks;       // device count
    int NM;                    // 128-row weight blocks per chunk: rows_total / 128
    // A: Q2 blobs
    const unsigned char *blobs;   // experts x blob_bytes
    const unsigned char *shared;  // one blob
    long long blob_bytes;
    long long codes_off, scales_off;  // byte offsets of this GEMM's code and scale regions in a blob
    int K;                            // H (gate/up) or F (down)
    int rows_total;                   // 2F (gate/up) or H (down)
    // B and outputs
    const float *row_scale;    // gate/up: 2^-k of each B row (x was stored times 2^k)
    const int *row_token;      // token of each B row
    const float *row_weight;   // down: routing weight of each B row
    __half *hidden;            // gate/up output: [B rows][rows_total / 2]
    float *y;                  // down output: y[token][rows_total] += weight * D
    unsigned *err;
    unsigned long long spin_limit;
    CUtensorMap tm_codes[2];   // [0] routed blobs {K/4 bytes, rows_total, experts}, [1] shared; box {64, 128}, 64B swizzle
    CUtensorMap tm_b;          // B {K, rows} FP16, box {64, 16}, 128B swizzle
    CUtensorMap tm_b64;        // the same matrix, box {64, 64}
};

__device__ __forceinline__ unsigned su32(const void *p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void bar_init(unsigned long long *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect(unsigned long long *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(unsigned long long *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(unsigned long long *b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void tma2(void *dst, const CUtensorMap *m, int x, int y, unsigned long long *b) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                     su32(dst)),
                 "l"(m), "r"(x), "r"(y), "r"(su32(b))
                 : "memory");
}
__device__ __forceinline__ void tma3(void *dst, const CUtensorMap *m, int x, int y, int z, unsigned long long *b) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            su32(dst)),
        "l"(m), "r"(x), "r"(y), "r"(z), "r"(su32(b))
        : "memory");
}
__device__ __forceinline__ void bulk(void *dst, const void *src, unsigned bytes, unsigned long long *b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)), "l"(src),
                 "r"(bytes), "r"(su32(b))
                 : "memory");
}
// AND of `ok` over the 256 epilogue threads (named barrier 1): their exits stay uniform.
__device__ __forceinline__ bool ep_all(bool ok) {
    unsigned r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, 1, 256, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((unsigned)ok)
        : "memory");
    return r != 0;
}

// Shared-memory matrix descriptor (tcgen05): K-major, 128-byte swizzle, 8-row groups 1024
// bytes apart (SBO), version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ unsigned long long sw128_desc(unsigned smem_addr) {
    return (unsigned long long)((smem_addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: F32 accumulate (bits 4-5 = 1), A and B FP16 (formats 0),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ unsigned idesc_f16(int M, int N) { return (1u << 4) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24); }

__device__ __forceinline__ void mma_f16(unsigned tmem_d, unsigned long long a, unsigned long long b, unsigned idesc, int accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(unsigned long long *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b)) : "memory");
}
// One lane of the converged warp (elect.sync): the warp computes the MMA operands as
// warp-uniform values and the elected lane issues.
__device__ __forceinline__ bool elect_one() {
    unsigned r;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r));
    return r != 0;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(unsigned taddr, float (&v)[32]) {
    unsigned r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, "
        "%19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
          "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
          "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(unsigned taddr, const unsigned (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]),
        "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void mma_f16_ts(unsigned tmem_d, unsigned tmem_a, unsigned long long b, unsigned idesc, int accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16 codes (one 32-bit word, code i at bits 2i) times one FP16 scale -> 16 FP16 in order,
// as 8 half2 words. The FP16 bits 0x6400 | c are 1024 + c; minus 1025 gives c - 1 exactly,
// and (c - 1) * s is exact (c - 1 in {-1, 0, 1, 2}).
__device__ __forceinline__ void dequant16(unsigned w, __half2 s2, unsigned (&out)[8]) {
    const __half2 k1025 = __floats2half2_rn(1025.0f, 1025.0f);
    unsigned pr[8];  // pr[j] = (code j, code j + 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const unsigned t = ((w >> (2 * j)) & 0x00030003u) | 0x64006400u;
        const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&t), k1025), s2);
        pr[j] = *reinterpret_cast<const unsigned *>(&h);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        out[j] = __byte_perm(pr[2 * j], pr[2 * j + 1], 0x5410);      // codes 2j, 2j+1
        out[4 + j] = __byte_perm(pr[2 * j], pr[2 * j + 1], 0x7632);  // codes 8+2j, 9+2j
    }
}

struct __align__(1024) GemmSmem {
    unsigned char b[kStages][kMaxN * 128];      // B rows, 128-byte swizzle (1024-aligned)
    unsigned char apk[kApkStages][128 * 64];    // packed codes of a super-block, 64-byte swizzle
    unsigned char staging[2 * 32 * 128 * 4];    // epilogue staging: gate/up hidden FP16 [N][64] / down F32 [2 halves][32][128]
    unsigned short scl[2][128 * 40];            // FP16 scales of the tile's 128 rows (<= 40 groups per row)
    float row_f[kMaxN];                         // epilogue: per B row scale (gate/up) or weight (down)
    int row_t[kMaxN];                           // epilogue: per B row token (down)
    unsigned long long full[kStages], empty[kStages];
    unsigned long long a_full[kAStages], a_empty[kAStages];
    unsigned long long apk_full[kApkStages], apk_empty[kApkStages];
    unsigned long long scl_full[2], scl_empty[2];
    unsigned long long tmem_full[2], tmem_empty[2];
    unsigned long long mma_done;
    unsigned tmem_base;
    int abort_flag;
};

template <int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) k_pf_gemm(const __grid_constant__ GemmParams P) {
    extern __shared__ unsigned char gsm_raw[];
    GemmSmem &S = *reinterpret_cast<GemmSmem *>(gsm_raw + ((1024 - (su32(gsm_raw) & 1023)) & 1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int n_tiles = *P.n_chunks * P.NM;
    auto tile_at = [&](int i) {
        const Chunk c = P.chunks[i / P.NM];
        return Tile{c.slot, i % P.NM, c.row0, c.n};
    };
    const int K = P.K, NKB = K / kKBlock, NSB = (NKB + kSuper - 1) / kSuper, NGRP = K / 64;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(&S.full[s], 1);
            bar_init(&S.empty[s], 1);
        }
        for (int s = 0; s < kAStages; ++s) {
            bar_init(&S.a_full[s], kDeqThreads);
            bar_init(&S.a_empty[s], 1);
        }
        for (int s = 0; s < kApkStages; ++s) {
            bar_init(&S.apk_full[s], 1);
            bar_init(&S.apk_empty[s], kDeqThreads);
        }
        for (int s = 0; s < 2; ++s) {
            bar_init(&S.scl_full[s], 1);
            bar_init(&S.scl_empty[s], kDeqThreads);
            bar_init(&S.tmem_full[s], 1);
            bar_init(&S.tmem_empty[s], kEpiThreads);
        }
        bar_init(&S.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        S.abort_flag = 0;
    }
    if (warp == 1) {  // TMEM: 512 columns: two accumulators and the A stages
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(&S.tmem_base)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const unsigned tmem = S.tmem_base;

    auto wait = [&](unsigned long long *b, unsigned parity) -> bool {
        for (unsigned long long i = 0;; ++i) {
            if (bar_try(b, parity)) return true;
            if (i > P.spin_limit || *(volatile int *)&S.abort_flag) {
                atomicOr(&S.abort_flag, 1);
                return false;
            }
        }
    };
    auto drain = [&](unsigned long long *b, unsigned parity) {  // own operations in flight: bounded, ignores the abort flag
        for (unsigned long long i = 0; i <= P.spin_limit; ++i)
            if (bar_try(b, parity)) return;
        atomicOr(&S.abort_flag, 1);
    };
    auto tile_blob = [&](const Tile &t) -> const unsigned char * {
        return t.slot < 0 ? P.shared : P.blobs + (long long)t.slot * P.blob_bytes;
    };

    if (warp == 0) {
        // ---------------------------------------------------------------- producer of B
        if (lane == 0) {
            int kb_count = 0;
            bool ok = true;
            for (int ti = cta; ti < n_tiles && ok; ti += G) {
                const Tile t = tile_at(ti);
                const int nb = (t.n + 15) >> 4;  // 16-row B boxes: nb / 4 boxes of 64 rows, then nb % 4 of 16
                for (int kb = 0; kb < NKB && ok; ++kb, ++kb_count) {
                    const int s = kb_count % kStages;
                    if (!(ok = wait(&S.empty[s], ((kb_count / kStages) & 1) ^ 1))) break;
                    bar_expect(&S.full[s], nb * 16 * 128);
                    int i = 0;
                    for (; i + 4 <= nb; i += 4) tma2(S.b[s] + i * 16 * 128, &P.tm_b64, kKBlock * kb, t.row0 + 16 * i, &S.full[s]);
                    for (; i < nb; ++i) tma2(S.b[s] + i * 16 * 128, &P.tm_b, kKBlock * kb, t.row0 + 16 * i, &S.full[s]);
                }
            }
            // every issued copy must land before the CTA leaves
            for (int k = max(0, kb_count - kStages); k < kb_count; ++k) drain(&S.full[k % kStages], (k / kStages) & 1);
        }
    } else if (warp == kCodeWarp) {
        // ---------------------------------------------------------------- producer of A (scales, codes)
        if (lane == 0) {
            int sb_count = 0, lt = 0;
            bool ok = true;
            for (int ti = cta; ti < n_tiles && ok; ti += G, ++lt) {
                const Tile t = tile_at(ti);
                const int ts = lt & 1;
                if (!(ok = wait(&S.scl_empty[ts], ((lt >> 1) & 1) ^ 1))) break;
                const unsigned sbytes = 128u * NGRP * 2;
                bar_expect(&S.scl_full[ts], sbytes);
                bulk(S.scl[ts], tile_blob(t) + P.scales_off + (long long)t.mtile * 128 * NGRP * 2, sbytes, &S.scl_full[ts]);
                for (int sb = 0; sb < NSB && ok; ++sb, ++sb_count) {
                    const int sa = sb_count % kApkStages;
                    if (!(ok = wait(&S.apk_empty[sa], ((sb_count / kApkStages) & 1) ^ 1))) break;
                    bar_expect(&S.apk_full[sa], 128 * 64);
                    tma3(S.apk[sa], &P.tm_codes[t.slot < 0 ? 1 : 0], 64 * sb, 128 * t.mtile, t.slot < 0 ? 0 : t.slot, &S.apk_full[sa]);
                }
            }
            for (int k = max(0, sb_count - kApkStages); k < sb_count; ++k) drain(&S.apk_full[k % kApkStages], (k / kApkStages) & 1);
            for (int k = max(0, lt - 2); k < lt; ++k) drain(&S.scl_full[k & 1], (k >> 1) & 1);  // lt = scale copies issued
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        // the warp runs converged (waits voted warp-wide) so the operands stay warp-uniform;
        // one elected lane issues the MMAs and commits
        int kb_count = 0, lt = 0;
        bool ok = true;
        for (int ti = cta; ti < n_tiles && ok; ti += G, ++lt) {
            const Tile t = tile_at(ti);
            const int buf = lt & 1;
            if (!(ok = __all_sync(0xffffffffu, wait(&S.tmem_empty[buf], ((lt >> 1) & 1) ^ 1)))) break;
            tc_fence_after();
            const int N = (t.n + 15) & ~15;
            const unsigned idesc = idesc_f16(128, N);
            const unsigned d = tmem + buf * kAccCols;
            for (int kb = 0; kb < NKB && ok; ++kb, ++kb_count) {
                const int s = kb_count % kStages, sa = kb_count % kAStages;
                if (!(ok = __all_sync(0xffffffffu, wait(&S.full[s], (kb_count / kStages) & 1) && wait(&S.a_full[sa], (kb_count / kAStages) & 1))))
                    break;
                tc_fence_after();
                const unsigned a = tmem + kACol0 + 32 * sa;
                const unsigned long long bd = sw128_desc(su32(S.b[s]));
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < kKBlock / 16; ++k)  // K = 16 per MMA: 8 TMEM columns of A, +32 bytes inside the swizzled B row
                        mma_f16_ts(d, a + 8 * k, bd + 2 * k, idesc, kb > 0 || k > 0);
                    mma_commit(&S.empty[s]);
                    mma_commit(&S.a_empty[sa]);
                }
                __syncwarp();
            }
            if (ok && elect_one()) mma_commit(&S.tmem_full[buf]);
            __syncwarp();
        }
        // every MMA issued must complete before TMEM is released
        if (elect_one()) mma_commit(&S.mma_done);
        __syncwarp();
        drain(&S.mma_done, 0);
    } else if (warp < kEpiWarp0) {
        // ---------------------------------------------------------------- dequantise
        const int quarter = warp & 3, hf = (warp - 2) >> 2;  // TMEM lane quarter; codes 32 hf .. 32 hf + 31
        const int r = 32 * quarter + lane;                   // A row 0..127 = TMEM lane
        const unsigned tlane = (unsigned)(32 * quarter) << 16;
        int kb_count = 0, sb_count = 0, lt = 0;
        bool ok = true;
        for (int ti = cta; ti < n_tiles && ok; ti += G, ++lt) {
            const int ts = lt & 1;
            // waits are voted warp-wide: the TMEM stores below need the whole warp converged
            if (!(ok = __all_sync(0xffffffffu, wait(&S.scl_full[ts], (lt >> 1) & 1)))) break;
            for (int sb = 0; sb < NSB && ok; ++sb, ++sb_count) {
                const int sp = sb_count % kApkStages;
                if (!(ok = __all_sync(0xffffffffu, wait(&S.apk_full[sp], (sb_count / kApkStages) & 1)))) break;
                const int kb_end = min(NKB, (sb + 1) * kSuper);
                for (int kb = sb * kSuper; kb < kb_end; ++kb, ++kb_count) {
                    const int sa = kb_count % kAStages;
                    if (!(ok = __all_sync(0xffffffffu, wait(&S.a_empty[sa], ((kb_count / kAStages) & 1) ^ 1)))) break;
                    tc_fence_after();
                    // row r's 16 code bytes of this K-block: chunk c of its 64-byte row, stored at
                    // c ^ ((r >> 1) & 3) by the 64-byte swizzle; this thread takes words 2 hf, 2 hf + 1
                    const int c = kb - sb * kSuper;
                    const uint2 w = *reinterpret_cast<const uint2 *>(S.apk[sp] + r * 64 + ((c ^ ((r >> 1) & 3)) << 4) + 8 * hf);
                    const __half sc = __ushort_as_half(S.scl[ts][r * NGRP + kb]);
                    const __half2 s2 = __halves2half2(sc, sc);
                    unsigned lo[8], hi[8], o[16];
                    dequant16(w.x, s2, lo);
                    dequant16(w.y, s2, hi);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        o[i] = lo[i];
                        o[8 + i] = hi[i];
                    }
                    // column j holds K elements 2j, 2j + 1: this half's 32 elements are 16 columns
                    __syncwarp();
                    tmem_st16(tmem + tlane + kACol0 + 32 * sa + 16 * hf, o);
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    bar_arrive(&S.a_full[sa]);
                }
                bar_arrive(&S.apk_empty[sp]);
            }
            bar_arrive(&S.scl_empty[ts]);
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int et = tid - 32 * kEpiWarp0;     // 0..255
        const int quarter = warp & 3;            // TMEM lanes 32 quarter .. (a warp reaches only its quarter)
        const int half = (warp - kEpiWarp0) >> 2;  // 32-column chunks half, half + 2, ...
        const int ht = et & 127;                 // thread within the half
        const int row = 32 * quarter + lane;     // accumulator row = weight row within the tile
        const int HID = P.rows_total / 2;
        int lt = 0;
        bool ok = true;
        for (int ti = cta; ti < n_tiles && ok; ti += G, ++lt) {
            const Tile t = tile_at(ti);
            const int buf = lt & 1;
            if (!(ok = ep_all(wait(&S.tmem_full[buf], (lt >> 1) & 1)))) break;
            tc_fence_after();
            const unsigned tbase = tmem + ((unsigned)(32 * quarter) << 16) + buf * kAccCols;
            const int N = (t.n + 15) & ~15;
            // the tile's B-row metadata, once
            for (int i = et; i < t.n; i += kEpiThreads) {
                S.row_f[i] = MODE == kGateUp ? __ldg(P.row_scale + t.row0 + i) : __ldg(P.row_weight + t.row0 + i);
                if (MODE == kDown) S.row_t[i] = __ldg(P.row_token + t.row0 + i);
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");
            for (int c0 = 32 * half; c0 < N; c0 += 64) {
                float v[32];
                __syncwarp();
                tmem_ld32(tbase + c0, v);
                if (MODE == kGateUp) {
                    // row 2i = gate_i, 2i + 1 = up_i (adjacent lanes); hidden index 64 mtile + row / 2
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = c0 + j;
                        const float sc = n < t.n ? S.row_f[n] : 0.0f;
                        const float a = v[j] * sc;
                        const float up = __shfl_xor_sync(0xffffffffu, a, 1);
                        if (!(lane & 1) && n < t.n) {
                            const float h = __fdividef(a, 1.0f + __expf(-a)) * up;  // silu(gate) * up (prefill tolerance 2e-3)
                            reinterpret_cast<__half *>(S.staging)[n * 64 + (row >> 1)] = __float2half_rn(h);
                        }
                    }
                } else {
                    // stage [32 columns][128 rows] F32 (this half's area), then coalesced 16-byte reductions into y
                    float *st = reinterpret_cast<float *>(S.staging) + half * 32 * 128;
#pragma unroll
                    for (int j = 0; j < 32; ++j) st[j * 128 + row] = v[j];
                    asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory");
                    for (int i = ht; i < 32 * 32; i += 128) {  // 32 columns x 32 float4
                        const int j = i >> 5, q = i & 31, n = c0 + j;
                        if (n < t.n) {
                            const float4 s4 = reinterpret_cast<const float4 *>(st)[j * 32 + q];
                            const float w = S.row_f[n];
                            float *dst = P.y + (long long)S.row_t[n] * P.rows_total + 128 * t.mtile + 4 * q;
                            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(s4.x * w), "f"(s4.y * w),
                                         "f"(s4.z * w), "f"(s4.w * w)
                                         : "memory");
                        }
                    }
                    asm volatile("bar.sync %0, 128;" ::"r"(2 + half) : "memory");
                }
            }
            // accumulator drained: the MMA warp may reuse it
            tc_fence_before();
            bar_arrive(&S.tmem_empty[buf]);
            if (MODE == kGateUp) {
                asm volatile("bar.sync 1, 256;" ::: "memory");
                // hidden rows: t.n x 64 FP16 (128 bytes each) at column 64 mtile
                for (int i = et; i < t.n * 8; i += kEpiThreads) {
                    const int n = i >> 3, q = i & 7;
                    const uint4 val = reinterpret_cast<const uint4 *>(S.staging)[n * 8 + q];
                    *reinterpret_cast<uint4 *>(P.hidden + (long long)(t.row0 + n) * HID + 64 * t.mtile + 8 * q) = val;
                }
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");  // staging and row metadata free for the next tile
        }
    }

    __syncthreads();
    if (tid == 0 && S.abort_flag) raise_error(P.err, kErrWaitTimeout);
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

}  // namespace pf
}  // namespace strata
