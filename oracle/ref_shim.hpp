// TEST INFRASTRUCTURE (oracle/_ref recipe). Force-included in front of the reference's
// unmodified kernels/strata.cu so that g++ can compile it natively as the reference's CPU
// path. It supplies the small CUDA vocabulary the source uses, with the semantics of the
// reference's own CPU runtime (vendor/webcuda/src/wasm/cuda-cpu.hpp:1-20 and
// thread-pool.hpp:18-65):
//   * a workgroup is 64 lanes that run cooperatively on ONE host thread;
//   * __syncthreads() suspends the lane until every live lane of the workgroup has reached
//     the same barrier site (a lane that finishes or waits at another site is a fault, as
//     cw_fault in thread-pool.hpp:42 / compile.mjs:35);
//   * __shared__ arrays are per workgroup (here: per host thread, one workgroup at a time);
//   * independent workgroups run on a pool of 1..8 host threads.
// The reference implements lanes as C++20 coroutines produced by a source rewrite
// (compile.mjs:7-44); this shim implements them as stackful fibers, which needs no rewrite.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

struct StrataRefIndex { unsigned x = 0, y = 0, z = 0; };
struct StrataRefLane;
extern thread_local StrataRefLane *strata_ref_current;
extern thread_local StrataRefIndex blockIdx, blockDim, gridDim;
const StrataRefIndex &strata_ref_thread_index();
void strata_ref_barrier(int site);

inline float __uint_as_float(unsigned int x) { float f; std::memcpy(&f, &x, 4); return f; }
inline float __int_as_float(int x) { float f; std::memcpy(&f, &x, 4); return f; }
inline unsigned int __float_as_uint(float x) { unsigned int u; std::memcpy(&u, &x, 4); return u; }
inline int __float_as_int(float x) { int u; std::memcpy(&u, &x, 4); return u; }

#define __device__
#define __global__
#define __shared__ static thread_local
#define threadIdx (strata_ref_thread_index())
#define __syncthreads() strata_ref_barrier(__COUNTER__)
