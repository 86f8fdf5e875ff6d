// Device building blocks of the integer tensor-core MoE kernels (the fused decode layer,
// csrc/moe_fast.cu, and the medium-batch layer, csrc/moe_medium.cu): copies (mbarrier, TMA,
// bulk and cp.async), the u8 x s8 mma.sync on raw 2-bit codes, grid arrivals, and the
// three-digit activation operands.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace strata {
namespace q2 {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxTokens = 8;

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
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
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
__device__ __forceinline__ void tma_4d(void *dst, const CUtensorMap *map, int x, int y, int z, int w, unsigned long long *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}
// L2 prefetches by the bulk-copy engine: a contiguous range (16-byte aligned, a multiple of 16
// bytes), or one box of a tensor map.
__device__ __forceinline__ void prefetch_l2_bulk(const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2_tile_3d(const CUtensorMap *map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
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
// The same with a zero accumulator: the first MMA of a chain needs no zeroed registers.
__device__ __forceinline__ void imma0(int (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_acc(bool acc, int (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                                         unsigned b1) {
    if (acc) imma(d, a0, a1, a2, a3, b0, b1);
    else imma0(d, a0, a1, a2, a3, b0, b1);
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }
__device__ __forceinline__ bool grid_arrive_wait(unsigned *counter, unsigned target, unsigned long long limit) {
    __threadfence();
    atomicAdd(counter, 1u);
    for (unsigned long long i = 0;; ++i) {
        if (ld_acquire(counter) >= target) return true;
        if (i > limit) return false;
        __nanosleep(32);
    }
}

// Scale exponent k for maxabs >= 0: 2^k * maxabs < 2^22 (maxabs = m 2^e, m in [0.5, 1): k =
// 22 - e), 0 for zero or non-finite maxabs, clamped to [-126, 126] so that 2^k and 2^-k are
// normal floats (a vector whose largest element is subnormal then keeps fewer bits).
__device__ __forceinline__ int scale_exp(float maxabs) {
    const unsigned b = __float_as_uint(maxabs);
    const int be = (int)(b >> 23);  // biased exponent (sign bit clear)
    int k = 22 - (be - 126);
    k = be == 0 ? 126 : k;
    k = be >= 255 || b == 0u ? 0 : k;
    return max(-126, min(126, k));
}
__device__ __forceinline__ float pow2f(int k) { return __uint_as_float((unsigned)(k + 127) << 23); }  // k in [-126, 127]
// Byte of signed digit d of v = d0 + 256 d1 + 65536 d2 (each digit in [-128, 127]):
// d0 = v mod 256, d1 = floor((v + 128) / 256) mod 256, d2 = floor((v + 32896) / 65536).
__device__ __forceinline__ unsigned digit_byte(int v, int d) {
    const int bias = d == 0 ? 0 : d == 1 ? 128 : 32896;
    return (unsigned)((v + bias) >> (8 * d)) & 255u;
}
__device__ __forceinline__ unsigned pack_digit(const int *v, int d) {
    return digit_byte(v[0], d) | digit_byte(v[1], d) << 8 | digit_byte(v[2], d) << 16 | digit_byte(v[3], d) << 24;
}
// B-fragment words of 16 consecutive elements e0..e15 of a 64-group (block q of 16): for MMA
// half h, register b0 byte i is element 2h + 4i, b1 byte i is element 2h + 1 + 4i (the A
// side: (w >> 4h) & 0x03030303 of the row's word q holds codes 16q + 2h + 4i).
__device__ __forceinline__ void block_frags(const int (&v)[16], uint2 *dst_h0, uint2 *dst_h1) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int lo[4] = {v[2 * h], v[2 * h + 4], v[2 * h + 8], v[2 * h + 12]};
        const int hi[4] = {v[2 * h + 1], v[2 * h + 5], v[2 * h + 9], v[2 * h + 13]};
        uint2 *dst = h ? dst_h1 : dst_h0;
#pragma unroll
        for (int d = 0; d < 3; ++d) dst[d] = make_uint2(pack_digit(lo, d), pack_digit(hi, d));
    }
}

template <int H, int F>
struct Geo {
    static constexpr int NG = H / 64;                  // scale groups per gate/up row
    static constexpr int NJ = F / 64;                  // units per expert
    static constexpr int CPT = NG / 8;                 // gate/up chunks per warp and unit
    static constexpr int SGU = NG == 32 ? 4 : 3;       // gate/up stages per warp
    static constexpr int RW = H / kWarps;              // down rows per warp
    static constexpr int DN_CODES = RW * 16;           // 16 code bytes per row
    static constexpr int DN_STAGE = (DN_CODES + RW * 4 + 127) / 128 * 128;  // + one scale word per row
    static constexpr int GS_BYTES = 16 * 2 * NG;       // FP16 scales of a warp's 16 gate/up rows
    static_assert(NG % 8 == 0 && RW % 32 == 0 && NJ % 2 == 0, "geometry");
};

}  // namespace q2
}  // namespace strata
