/*
 * TEST INFRASTRUCTURE (oracle). Not part of the product; only tests/, bench.py's
 * cpu_baseline leg and __graft_entry__.smoke() may use it, and only as a checker.
 *
 * expf as the reference's WASM build links it.
 *
 * The reference calls `expf` in strata_sigmoid (kernels/strata.cu:7) and in the router
 * softmax (kernels/strata.cu:249, :488). Its threaded-WASM path is compiled by Emscripten
 * (vendor/webcuda/src/wasm/compile.mjs:51) and therefore links musl's expf, which is the
 * ARM optimized-routines single-precision exp (Szabolcs Nagy, 2017; musl src/math/expf.c
 * with exp2f_data.c; the same algorithm is glibc's sysdeps/ieee754/flt-32/e_expf.c).
 * The reference pins neither the Emscripten nor the musl version.
 *
 * Published method, restated:
 *   x*N/ln2 = k + r  (N = 32, k integer by the 1.5*2^52 shift trick, |r| <= 1/2)
 *   exp(x)  = 2^(k/N) * 2^(r/N) ~= s * (C0 r^3 + C1 r^2 + C2 r + 1)
 *   s       = asdouble(T[k % N] + (k << 47)), T[i] = bits(2^(i/N)) - (i << 47)
 * evaluated in double without fused multiply-add (WASM has none), then rounded once to
 * float. The table is computed from mathematics by oracle/gen_exp2_table.py and checked
 * bit-for-bit there; the three polynomial coefficients are the published minimax values.
 * tests/test_oracle_expf.py compares this function with the host C library's expf over
 * every float input.
 */
#ifndef STRATA_ORACLE_EXPF_H
#define STRATA_ORACLE_EXPF_H
#include <stdint.h>
#include <string.h>

static const uint64_t strata_exp2_tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

static inline float strata_o_u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t strata_o_f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline double strata_o_u2d(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint64_t strata_o_d2u(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

/* Must be compiled with -ffp-contract=off: every product and sum rounds separately. */
static inline float strata_oracle_expf(float x) {
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    uint32_t ux = strata_o_f2u(x);
    uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) { /* |x| >= 88 or x is NaN/inf */
        if (ux == 0xff800000u) return 0.0f;          /* -inf */
        if (abstop >= 0x7f8u) return x + x;          /* +inf, NaN */
        if (x > 0x1.62e42ep6f) return strata_o_u2f(0x7f800000u);  /* overflow */
        if (x < -0x1.9fe368p6f) return 0.0f;         /* underflow */
    }
    double xd = (double)x;
    double z = inv_ln2_n * xd;
    double kd = z + shift;
    uint64_t ki = strata_o_d2u(kd);
    kd -= shift;
    double r = z - kd;
    uint64_t t = strata_exp2_tab[ki % 32u];
    t += ki << 47;
    double s = strata_o_u2d(t);
    double p = c0 * r + c1;
    double r2 = r * r;
    double y = c2 * r + 1.0;
    y = p * r2 + y;
    y = y * s;
    return (float)y;
}
#endif
