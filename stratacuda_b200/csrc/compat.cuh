// Shared by the reference-compatible entries (compat.cu, engine_ops.cu): bounds-checked
// buffer views, the mapping of 64-lane reference workgroups onto warps, and launch shapes.
#pragma once
#include "common.cuh"
#include "kernels.h"

#include <cstdint>

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

// Whether [start, start + count) lies inside the buffer (a warp checks once, then loads unchecked).
template <typename T>
__device__ __forceinline__ bool covers(const Buf<T> &b, long long start, long long count) {
    return start >= 0 && count >= 0 && start + count <= b.n;
}

// One reference workgroup's strided sum of products over a row of `cols` (thread t of the warp
// owns lanes t and t + 32), then the shared-memory tree: tree64's result. The pointers must
// cover [0, cols). Loads are issued eight at a time ahead of the two rounded accumulation
// chains, which keep the reference's order.
__device__ __forceinline__ float lane_dot(const float *w, const float *x, int cols, int t) {
    float lo = 0.0f, hi = 0.0f;
    int i = t;
    for (; i + 3 * STRATA_LANES + 32 < cols; i += 4 * STRATA_LANES) {
        float wv[8], xv[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            wv[2 * k] = w[i + STRATA_LANES * k];
            xv[2 * k] = x[i + STRATA_LANES * k];
            wv[2 * k + 1] = w[i + STRATA_LANES * k + 32];
            xv[2 * k + 1] = x[i + STRATA_LANES * k + 32];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            lo = __fadd_rn(lo, __fmul_rn(wv[2 * k], xv[2 * k]));
            hi = __fadd_rn(hi, __fmul_rn(wv[2 * k + 1], xv[2 * k + 1]));
        }
    }
    for (; i < cols; i += STRATA_LANES) {
        lo = __fadd_rn(lo, __fmul_rn(w[i], x[i]));
        if (i + 32 < cols) hi = __fadd_rn(hi, __fmul_rn(w[i + 32], x[i + 32]));
    }
    return tree64(lo, hi);
}

// Copy n floats from global memory into shared memory with all threads of the block, 16 bytes
// at a time where both sides allow it.
__device__ __forceinline__ void stage_row(float *dst, const float *src, int n) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const int n4 = n / 4, bd = blockDim.x;
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        // eight 16-byte loads of a thread in flight before their stores (one round trip for
        // rows up to 8 * 16 * blockDim bytes)
        for (int k0 = threadIdx.x; k0 < n4; k0 += 8 * bd) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (k0 + i * bd < n4) v[i] = s4[k0 + i * bd];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (k0 + i * bd < n4) d4[k0 + i * bd] = v[i];
        }
        for (int k = n4 * 4 + threadIdx.x; k < n; k += bd) dst[k] = src[k];
    } else {
        for (int k = threadIdx.x; k < n; k += blockDim.x) dst[k] = src[k];
    }
}

// Programmatic dependent launch of the engine entries. A kernel launched by launch_dep may be
// scheduled while the previous kernel of its stream is still running. Its first statement is
// dep_enter(): wait until that kernel has finished and its writes are visible, then let the next
// kernel of the stream be scheduled. So at most one kernel runs ahead of its predecessor's end,
// and it touches no memory before dep_enter() except L2 prefetches of weights (which no kernel
// writes). Launched without the attribute (STRATA_ENGINE_PDL=0), dep_enter() returns at once.
__device__ __forceinline__ void dep_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// A hint that [p, p + bytes) will be read soon: one bulk L2 prefetch (16-byte aligned start, the
// size rounded down to 16 bytes; nothing is issued for an unaligned start).
__device__ __forceinline__ void prefetch_l2(const void *p, unsigned long long bytes) {
    bytes &= ~15ull;
    if ((reinterpret_cast<uintptr_t>(p) & 15) != 0 || bytes == 0) return;
    while (bytes > 0) {
        const unsigned n = bytes > (1ull << 30) ? (1u << 30) : (unsigned)bytes;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(n) : "memory");
        p = static_cast<const char *>(p) + n;
        bytes -= n;
    }
}
bool engine_pdl();  // STRATA_ENGINE_PDL is not "0" (read once)
// `dep`: launch with the attribute. The one-token (decode) dispatches take it; prompt-chunk
// dispatches run long enough that an early launch gains nothing, and their blocks are then placed
// wherever the previous kernel has freed room instead of evenly over the SMs.
template <typename... KT, typename... AT>
inline cudaError_t launch_k(bool dep, void (*k)(KT...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, AT &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dep && engine_pdl() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<AT &&>(args)...);
}

// 16-byte asynchronous global -> shared copies (cp.async, L2 only) and their group waits.
__device__ __forceinline__ void copy16_async(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void copy_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void copy_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// The same workgroups with y varying fastest: consecutive warps take consecutive tokens of one
// weight row, so a prompt chunk reads each row from HBM once (the rest hit L1/L2).
__device__ __forceinline__ bool my_group_y_first(const Grid g, unsigned &gx, unsigned &gy, unsigned &gz) {
    unsigned long long w = (unsigned long long)blockIdx.x * kWarpsPerBlock + threadIdx.x / 32;
    unsigned long long total = (unsigned long long)g.x * g.y * g.z;
    if (w >= total) return false;
    gy = (unsigned)(w % g.y);
    gx = (unsigned)((w / g.y) % g.x);
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
