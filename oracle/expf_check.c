/*
 * TEST INFRASTRUCTURE (oracle). Compares strata_oracle_expf (the restated musl/ARM expf,
 * strata_expf.h) with the host C library's expf over every 32-bit float input, on 8 threads.
 * Prints "<mismatches> <nan-pairs>". Run with GLIBC_TUNABLES=glibc.cpu.hwcaps=-FMA,-AVX2 to
 * make glibc select its expf built without fused multiply-add, which is the variant that
 * matches WASM semantics.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>

#include "strata_expf.h"

#define THREADS 8
static unsigned long long mism[THREADS], nans[THREADS];

static void *work(void *arg) {
    long t = (long)arg;
    uint64_t begin = (0x100000000ull / THREADS) * (uint64_t)t, end = begin + 0x100000000ull / THREADS;
    for (uint64_t u = begin; u < end; ++u) {
        float x = strata_o_u2f((uint32_t)u);
        float a = strata_oracle_expf(x), b = expf(x);
        if (a != a && b != b) { nans[t]++; continue; }
        if (strata_o_f2u(a) != strata_o_f2u(b)) mism[t]++;
    }
    return 0;
}

int main(void) {
    pthread_t th[THREADS];
    for (long t = 0; t < THREADS; ++t) pthread_create(&th[t], 0, work, (void *)t);
    unsigned long long m = 0, n = 0;
    for (long t = 0; t < THREADS; ++t) { pthread_join(th[t], 0); m += mism[t]; n += nans[t]; }
    printf("%llu %llu\n", m, n);
    return 0;
}
