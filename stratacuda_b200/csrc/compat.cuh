// Shared by the reference-compatible entries (compat.cu, engine_ops.cu): bounds-checked
// buffer views, the mapping of 64-lane reference workgroups onto warps, and launch shapes.
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace strata {

template <typename T>
struct Buf {
    T *p;
    long long n;
    __device__ __forceinline__ T get(long long i, unsigned *err) const {
        if (i < 0 || i >= n) { raise_error(err, kErrIndex); return T(0); }
        return p[i];
    }
    __device__ __forceinline__ void set(long long i, T v, unsigned *err) const {
        if (i < 0 || i >= n) { raise_error(err, kErrIndex); return; }
        p[i] = v;
    }
};
using FB = Buf<float>;
using UB = Buf<unsigned>;
using IB = Buf<int>;

__device__ __forceinline__ float half_of(const UB &b, long long h, unsigned *err) {
    return half_bits((b.get(h / 2, err) >> ((h % 2) * 16)) & 65535u);
}
__device__ __forceinline__ int code_of(const UB &b, long long codeOffset, long long index, unsigned *err) {
    return (int)((b.get(codeOffset + index / 16, err) >> ((index % 16) * 2)) & 3u) - 1;
}

// kernels/strata.cu:22-31, the IQ4_NL codebook
__device__ __forceinline__ float iq4(int c) {
    const float t[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f, 1.f, 13.f, 25.f, 38.f, 53.f, 69.f, 89.f, 113.f};
    return (c >= 0 && c < 15) ? t[c] : 113.0f;
}

struct Grid {
    unsigned x, y, z;
};
constexpr int kWarpsPerBlock = 4;

// Workgroup (x, y, z) handled by this warp, or false when past the dispatch grid.
__device__ __forceinline__ bool my_group(const Grid g, unsigned &gx, unsigned &gy, unsigned &gz) {
    unsigned long long w = (unsigned long long)blockIdx.x * kWarpsPerBlock + threadIdx.x / 32;
    unsigned long long total = (unsigned long long)g.x * g.y * g.z;
    if (w >= total) return false;
    gx = (unsigned)(w % g.x);
    gy = (unsigned)((w / g.x) % g.y);
    gz = (unsigned)(w / ((unsigned long long)g.x * g.y));
    return true;
}


inline Grid grid_of(const unsigned g[3]) { return Grid{g[0], g[1], g[2]}; }
inline unsigned group_blocks(const unsigned g[3]) {
    unsigned long long total = (unsigned long long)g[0] * g[1] * g[2];
    return (unsigned)((total + kWarpsPerBlock - 1) / kWarpsPerBlock);
}
inline unsigned lane_blocks(const unsigned g[3]) { return (unsigned)(((unsigned long long)g[0] * STRATA_LANES + 255) / 256); }

#define F(i) FB{(float *)a[i].ptr, a[i].len}
#define U(i) UB{(unsigned *)a[i].ptr, a[i].len}
#define I(i) IB{(int *)a[i].ptr, a[i].len}
#define GROUPS group_blocks(g), kWarpsPerBlock * 32, 0, s
#define LANESL lane_blocks(g), 256, 0, s

}  // namespace strata
