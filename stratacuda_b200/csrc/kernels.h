// Internal interface between the C-ABI layer (api.cu) and the kernel files.
#pragma once
#include <string>
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ep_comm.h"

namespace strata {

// Device-side error word bits (set with atomicOr, read by the host at the next sync).
enum : unsigned {
    kErrIndex = 1u,        // a data-dependent index (mapping, gather index, expert id) was out of range
    kErrWaitTimeout = 2u,  // a bounded spin-wait gave up
    kErrRouting = 4u,      // a routed expert id was invalid or repeated (src/engine.js:138)
    kErrPleScale = 8u,     // a gathered PLE row has a non-finite FP16 scale (src/model.js:241)
};

// One resolved argument of a reference-compatible dispatch: a device buffer (ptr, length in
// 4-byte elements) or a scalar.
struct KArg {
    void *ptr;
    long long len;
    int i;
    float f;
};
using Launcher = cudaError_t (*)(const KArg *args, const unsigned groups[3], cudaStream_t s, unsigned *err);
struct KernelSpec {
    const char *name;
    const char *params;  // "Name:kind ..." with kind f/u/i (buffers) or I/F (scalars)
    Launcher launch;
};
extern const KernelSpec kKernels[];  // compat.cu: the mixture-of-experts entries
extern const int kNumKernels;
extern const KernelSpec kEngineKernels[];  // engine_ops.cu: every other entry of the reference
extern const int kNumEngineKernels;

// Device view of one mixture-of-experts layer (see strata_moe_layer in include/strata_cuda.h).
struct MoeLayerDev {
    int width, ff, experts, topK;
    const float *router;       // [experts][width] f32
    const float *bias;         // [experts] f32 or null
    const unsigned *blobs;     // experts x blob_words
    long long blob_words;
    const unsigned *shared_blob;  // blob_words
    const float *shared_gate;     // [width] f32
};

// Scratch for one fused call, carved from the context's workspace.
struct MoeScratch {
    float *logits;      // [tokens][experts]
    float *sg;          // [tokens]
    int *counts;        // [experts]
    int *active;        // [experts]
    int *n_active;      // [1]
    int *begin;         // [experts + 1]
    int *pair_token;    // [tokens * topK]
    int *pair_slot;     // [tokens * topK]
    float *hidden;      // [(tokens * topK + tokens) * ff]
    float *parts;       // [tokens * topK * width]
    float *shared_out;  // [tokens * width]
};
size_t moe_scratch_bytes(int tokens, int width, int ff, int experts, int topK);
MoeScratch moe_scratch_carve(void *base, int tokens, int width, int ff, int experts, int topK);

// Fused layer: y[tokens][width], ids/weights[tokens][topK]. Exact reduction order everywhere.
cudaError_t moe_forward_exact(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights,
                              const MoeScratch &ws, cudaStream_t s, unsigned *err);

// Fast fused layer for decode batches (csrc/moe_fast.cu): one cooperative launch of `grid`
// CTAs (one per SM). `sync` is 4 zero-initialised words reserved for this kernel's grid
// arrivals; the kernel leaves them zero again on exit.
bool moe_fast_supported(int tokens, int width, int ff, int topK, int grid);
size_t moe_fast_scratch_bytes(int tokens, int width, int ff, int experts, int topK);
int moe_fast_pdl_state();  // 1: launched with programmatic dependent launch, 0: refused, -1: not launched yet
cudaError_t moe_forward_fast(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights, void *scratch,
                             unsigned *sync, int grid, cudaStream_t s, unsigned *err);

// One-token decode layer (csrc/moe_decode1.cu): one cooperative launch of `grid` CTAs. `xchg`
// (moe_decode1_xchg_bytes, zeroed once) and `sync` (kDecode1SyncWords words, zeroed once) belong
// to this kernel alone: they carry its tagged cross-CTA exchange and launch count between calls.
constexpr int kDecode1SyncWords = 2;
bool moe_decode1_supported(int tokens, int width, int ff, int experts, int topK, int grid);
size_t moe_decode1_xchg_bytes();
cudaError_t moe_forward_decode1(const MoeLayerDev &L, const float *x, float *y, int *ids, float *weights, void *xchg, unsigned *sync,
                                int grid, cudaStream_t s, unsigned *err);

// TMA maps of the medium-batch layer for a layer's routed experts [0] and shared expert [1],
// cached by blob address (csrc/moe_fast.cu), all boxes of 128 rows: gate/up codes (128 bytes,
// 128-byte swizzle), gate/up scales (8 groups) and down codes (full rows; 128-byte swizzle for
// 128-byte rows).
struct MoeMaps {
    CUtensorMap gu[2], gs[2], dc[2];
    CUtensorMap dn16[2];  // down codes, boxes of 16 full rows (the one-token decode layer)
    CUtensorMap gu16r[2]; // gate/up codes, boxes of 16 full rows in one request (chunk-major, swizzled)
    CUtensorMap dn64[2];  // down codes, boxes of 64 full rows (8 KB, contiguous)
};
bool moe_tensor_maps(const MoeLayerDev &L, MoeMaps *maps);
// the same plus the gate/up code maps in boxes of 16 rows ([0] routed, [1] shared)
bool moe_decode_maps(const MoeLayerDev &L, CUtensorMap *gu16, MoeMaps *maps);

// Medium-batch layer (csrc/moe_medium.cu), 9 .. 64 tokens: the exact router kernels, then one
// cooperative launch of integer tensor-core units on the 2-bit codes (y within 1e-5 relative
// L2). `sync` as for moe_forward_fast (the two kernels never overlap on a stream).
bool moe_medium_supported(int tokens, int width, int ff, int experts, int topK, int grid);
size_t moe_medium_scratch_bytes(int tokens, int width, int ff, int experts, int topK);
cudaError_t moe_forward_medium(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights, void *scratch,
                               unsigned *sync, int grid, cudaStream_t s, unsigned *err);

// Exact router (csrc/prefill.cu): logits [T][E] + shared-gate logits [T] by the persistent
// logits kernel (`tail`: moe_logits_tail_bytes of scratch), then ids/weights [T][topK].
size_t moe_logits_tail_bytes(int width);
cudaError_t moe_route_exact(const MoeLayerDev &L, const float *x, int T, float *logits, float *sg, float *tail, int *ids, float *weights,
                            int grid, cudaStream_t s, unsigned *err);

// src/model.js:164: the lowest index of `count` blobs holding a non-finite FP16 scale into
// *first_bad (device int), or 0x7f7f7f7f when every scale is finite.
cudaError_t check_expert_scales(const unsigned *blobs, long long count, int width, int ff, int *first_bad, cudaStream_t s);

// Prompt / large-batch layer (csrc/prefill.cu): exact routing, expert products on tcgen05
// tensor cores from Q2 weights dequantised to FP16 (y within 2e-3 relative L2). `grid` is
// the GEMMs' persistent grid (one CTA per SM).
bool moe_prefill_supported(int width, int ff, int experts, int topK);
size_t moe_prefill_scratch_bytes(int tokens, int width, int ff, int experts, int topK);
// `marks` (nullable): four events recorded before routing, after routing, after the gate/up
// GEMM and after the down GEMM.
cudaError_t moe_forward_prefill(const MoeLayerDev &L, const float *x, int tokens, float *y, int *ids, float *weights, void *scratch,
                                int grid, cudaStream_t s, unsigned *err, cudaEvent_t *marks = nullptr);

// Expert parallel (csrc/prefill.cu, communicator and transports in csrc/ep_comm.h): forward of
// one layer whose L.blobs holds this rank's L.experts / n experts. Returns 0 or a nonzero
// code with `msg`; a failed exchange marks the communicator failed and aborts it.
int moe_forward_ep(const MoeLayerDev &L, EpComm *c, const float *x, int tokens, float *y, int *ids, float *weights, int grid, cudaStream_t s,
                   unsigned *err, std::string *msg,
                   cudaEvent_t *marks = nullptr);

// Per-layer embedding rows (csrc/compat.cu): rows ids[0 .. rows) of a device-resident IQ4_NL
// table decoded into values[rows * head_dim]; lengths in elements, for the bounds checks.
cudaError_t ple_gather_decode(const unsigned *table, long long table_words, const int *ids, long long ids_len, int rows, int head_dim,
                              float *values, long long values_len, cudaStream_t s, unsigned *err);

// Device synthetic generator (csrc/synth.cu), same bytes as stratacuda_b200/synth.py.
cudaError_t synth_expert_blobs(unsigned *out, unsigned long long seed, int layer, int first_expert, int count, int width, int ff,
                               int shared, cudaStream_t s);
cudaError_t synth_normals_f32(float *out, unsigned long long key, long long start, long long count, double scale, cudaStream_t s);
unsigned long long synth_stream_key(unsigned long long seed, unsigned long long tag, unsigned long long sub);

}  // namespace strata
