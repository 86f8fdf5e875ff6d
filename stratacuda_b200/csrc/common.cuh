// Device vocabulary shared by every kernel of libstrata_cuda.
//
// Exactness: the reference's numerical contract is F32 with every product and sum rounded
// separately (its WASM target has no fused multiply-add; kernels/strata.cu:5). Kernels that
// promise bit-identical results use the *_rn intrinsics below, which nvcc never contracts.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kernels.h"

#define STRATA_LANES 64  // a reference workgroup (kernels/strata.cu:3)

namespace strata {

__device__ __forceinline__ void raise_error(unsigned *err, unsigned bit) {
    if (err) atomicOr(err, bit);
}

// kernels/strata.cu:13-18: FP16 bits -> F32 (subnormals as fraction * 2^-24, NaN payload kept).
__device__ __forceinline__ float half_bits(unsigned h) {
    unsigned sign = (h & 32768u) << 16, exponent = (h >> 10) & 31u, fraction = h & 1023u;
    if (exponent == 0u) {
        if (fraction == 0u) return __uint_as_float(sign);
        float v = __fmul_rn((float)fraction, 0.000000059604644775390625f);
        return sign != 0u ? -v : v;
    }
    if (exponent == 31u) return __uint_as_float(sign | 2139095040u | (fraction << 13));
    return __uint_as_float(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

// The reference's expf, as its WASM build links it: the ARM optimized-routines expf of
// musl (src/math/expf.c, exp2f_data.c; Szabolcs Nagy 2017), restated from the published
// method: x*32/ln2 = k + r, 2^(k/32) from a 32-entry table, cubic in r, all in double
// without fused multiply-add, rounded once to float. The table holds
// bits(2^(i/32)) - (i << 47), computed from mathematics. Checked exhaustively on the host
// against the C library's expf (oracle), and on the device against that oracle. The table
// sits in global memory and is read through the L1 path: lanes index it divergently, which
// the constant cache would serialise.
static __device__ const unsigned long long c_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

// `tab`: the table's 32 words where the caller staged them (shared memory), else the global copy.
__device__ __forceinline__ float ref_expf(float x, const unsigned long long *tab = nullptr) {
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const unsigned ux = __float_as_uint(x);
    const unsigned abstop = (ux >> 20) & 0x7ffu;
    // Main path for every input (straight-line, so independent calls interleave); the rare
    // |x| >= 88 / NaN / inf cases are selected afterwards, exactly as the branches of the
    // published method resolve them.
    const double xd = (double)x;
    const double z = __dmul_rn(inv_ln2_n, xd);
    double kd = __dadd_rn(z, shift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, shift);
    const double r = __dsub_rn(z, kd);
    const unsigned long long t = (tab ? tab[ki & 31ull] : __ldg(&c_exp2_tab[ki & 31ull])) + (ki << 47);
    const double s = __longlong_as_double((long long)t);
    const double p = __dadd_rn(__dmul_rn(c0, r), c1);
    const double r2 = __dmul_rn(r, r);
    double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
    y = __dadd_rn(__dmul_rn(p, r2), y);
    y = __dmul_rn(y, s);
    const float main = __double2float_rn(y);
    // selects, not branches: unrolled callers keep independent evaluations interleaved
    float special = main;
    special = x < -0x1.9fe368p6f ? 0.0f : special;
    special = x > 0x1.62e42ep6f ? __uint_as_float(0x7f800000u) : special;
    special = abstop >= 0x7f8u ? __fadd_rn(x, x) : special;
    special = ux == 0xff800000u ? 0.0f : special;
    return abstop < 0x42bu ? main : special;
}

// kernels/strata.cu:7-8
__device__ __forceinline__ float ref_sigmoid(float x, const unsigned long long *tab = nullptr) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, ref_expf(-x, tab)));
}
__device__ __forceinline__ float ref_silu(float x, const unsigned long long *tab = nullptr) { return __fmul_rn(x, ref_sigmoid(x, tab)); }

// Paired F32 arithmetic (sm_100): each element of the pair is rounded to nearest exactly as
// the scalar __fmul_rn / __fadd_rn would round it (measured bit for bit). The compiler turns a
// paired product whose only use is a paired add into one fused multiply-add, which rounds
// once; a caller that needs both roundings gives every product a second use (xor3 below).
__device__ __forceinline__ unsigned long long mul2_rn(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long add2_rn(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// The rounded products of a paired multiply as an FMA with the addend neg0 = (-0, -0): a rounded
// product plus -0 is that product, bit for bit (a +0 product stays +0). neg0 must reach the kernel
// at run time (an argument): a literal -0 lets the compiler see a plain multiply and fuse it
// into the following add (measured: weights off by a few ulps), an unknown addend cannot be.
__device__ __forceinline__ unsigned long long mul_rn2(unsigned long long a, unsigned long long b, unsigned long long neg0) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(neg0));
    return d;
}
constexpr unsigned long long kNegZero2 = 0x8000000080000000ull;  // the host passes this as neg0
// Two floats as one 64-bit register pair (low = lo), and back: register moves, no arithmetic.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ unsigned xor3(unsigned a, unsigned b, unsigned c) {
    unsigned d;
    asm("lop3.b32 %0, %1, %2, %3, 0x96;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One warp emulates a reference workgroup of 64 lanes: thread t owns lanes t and t+32.
// The reference's tree (partial[l] += partial[l+s], s = 32..1) is the in-thread s=32 add
// followed by shuffle-down adds; the result is exact and valid in lane 0.
__device__ __forceinline__ float tree64(float lo, float hi) {
    float a = __fadd_rn(lo, hi);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, s));
    return a;
}

// 2-bit code of element `index` (LSB-first, 16 per word), minus 1: {-1, 0, 1, 2}.
__device__ __forceinline__ int q2_code(const unsigned *words, long long codeOffset, long long index) {
    return (int)((words[codeOffset + index / 16] >> ((index % 16) * 2)) & 3u) - 1;
}
__device__ __forceinline__ float half_at(const unsigned *words, long long halfIndex) {
    return half_bits((words[halfIndex / 2] >> ((halfIndex % 2) * 16)) & 65535u);
}

}  // namespace strata

#define STRATA_CUDA_TRY(expr)                                \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return _e;                    \
    } while (0)
