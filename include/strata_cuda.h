/*
 * libstrata_cuda — B200 (sm_100a) backend for StrataCuda's mixture-of-experts path.
 *
 * A C ABI (plain pointers, sizes and opaque 64-bit buffer handles; no CUDA or torch types)
 * that a host language binds through its FFI. It replaces the reference's backend object
 * protocol (src/backend.js:58-206: kind, alloc, write, read, copy, zero, run, free, idle,
 * flush, info, dispose) with one context per device, and adds fused entry points for the
 * whole MoE layer so that no routing result crosses to the host.
 *
 * Conventions
 *  - Every call returns a status (STRATA_OK = 0). The message of the last failure on a
 *    context is available from strata_last_error().
 *  - Buffers hold 4-byte elements (src/backend.js:84-92, 128-134): lengths and offsets are
 *    counted in elements, never bytes.
 *  - Calls on one context are stream-ordered and asynchronous; strata_read and strata_idle
 *    synchronise (src/backend.js:94, 117). One thread drives a context at a time.
 *  - Host memory passed in is borrowed only for the duration of the call.
 *  - Kernels never fault on bad indices: a data-dependent index outside its buffer is
 *    skipped and recorded, and the next synchronising call returns STRATA_ERR_DEVICE.
 */
#ifndef STRATA_CUDA_H
#define STRATA_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define STRATA_OK 0
#define STRATA_ERR_RANGE 1   /* argument outside the supported range: RangeError, src/backend.js:6-9 */
#define STRATA_ERR_LAYOUT 2  /* buffer/shape layout violated: Error, src/backend.js:22-36 */
#define STRATA_ERR_UNKNOWN 3 /* unknown kernel or missing argument: src/backend.js:102; wasm/runtime.js:12 */
#define STRATA_ERR_HANDLE 4  /* not a live buffer of this context: src/backend.js:138-143 */
#define STRATA_ERR_ALLOC 5   /* device allocation failed: wasm/runtime.js:7 "WASM allocation failed" */
#define STRATA_ERR_CUDA 6    /* CUDA runtime error (the message names it) */
#define STRATA_ERR_DEVICE 7  /* a kernel recorded an out-of-range index, an invalid routing, a timed-out wait or a non-finite PLE scale */

#define STRATA_F32 0
#define STRATA_I32 1
#define STRATA_U32 2

#define STRATA_ARG_BUF 0
#define STRATA_ARG_I32 1
#define STRATA_ARG_F32 2

typedef struct strata_ctx strata_ctx;
typedef uint64_t strata_buf; /* opaque; 0 is never a valid handle */

/* One named argument of strata_run: the reference passes buffers and numbers in one object
 * keyed by the kernel's parameter names (src/backend.js:101-113). */
typedef struct {
    const char *name;
    int32_t kind; /* STRATA_ARG_* */
    int32_t i32;
    float f32;
    strata_buf buf;
} strata_arg;

/* ---- context (GpuBackend.create / dispose, src/backend.js:59-71, 121) ---- */
int strata_create(int device, strata_ctx **out);
int strata_destroy(strata_ctx *ctx);
/* Copies the last error message (NUL-terminated, truncated to cap). Returns its full length. */
int strata_last_error(strata_ctx *ctx, char *buf, size_t cap);
/* The CUDA stream the context issues work on (a cudaStream_t, as an opaque pointer). */
int strata_stream(strata_ctx *ctx, void **stream);

/* ---- buffers (src/backend.js:84-100, 114-118) ---- */
/* alloc(length, type, {zero}); length in 4-byte elements, >= 1. */
int strata_alloc(strata_ctx *ctx, uint64_t length, int type, int zero, strata_buf *out);
int strata_free(strata_ctx *ctx, strata_buf buf);
/* write(buffer, data, offset): count elements from host memory at element offset. */
int strata_write(strata_ctx *ctx, strata_buf buf, const void *data, uint64_t count, uint64_t offset);
/* read(buffer): count elements from element offset into host memory; synchronises. */
int strata_read(strata_ctx *ctx, strata_buf buf, void *out, uint64_t count, uint64_t offset);
/* copy(source, destination, count, sourceOffset, destinationOffset), stream-ordered. */
int strata_copy(strata_ctx *ctx, strata_buf src, strata_buf dst, uint64_t count, uint64_t src_offset, uint64_t dst_offset);
/* zero(buffer), stream-ordered (src/backend.js:93). */
int strata_zero(strata_ctx *ctx, strata_buf buf);
/* Length (elements), type and device address of a live buffer. */
int strata_buffer_info(strata_ctx *ctx, strata_buf buf, uint64_t *length, int *type, void **device_ptr);

/* ---- dispatch (run, src/backend.js:101-113; validateDispatch :10-56) ----
 * Runs one reference entry of kernels/strata.cu by name, with the reference's parameter names and
 * its grid of 64-lane workgroups: all 49 entries that src/engine.js, src/ops.js and src/prefill.js
 * dispatch (mixture of experts, projections, norms, embeddings, RoPE, hyper-connections, the gated
 * delta rule, convolution, attention, per-layer embeddings, argmax; their prompt-batch forms).
 * Results are bit-identical to the reference's F32 CPU path; the RoPE table's cosf / sinf and the
 * softplus's logf, which the reference leaves to its C library, agree with it within one ulp.
 * Validation mirrors src/backend.js:10-56. It also rejects zero divisors and loop extents larger
 * than their buffers, which the reference leaves unchecked.
 *
 * Four further names have no counterpart in the reference. They read a token list or a position
 * from device memory instead of a kernel argument, so that one captured CUDA graph can replay
 * every decode step or full prompt chunk:
 *   strata_embed_token  (Table, Token, Residual, width, streams, vocab, tokens)
 *   strata_rope_at      (X, Cos, Sin, Y, Position, dim, heads, rotary, tokens)
 *   strata_kv_append_at (K, V, Keys, Values, Position, width, tokens)
 *   strata_attention_at (Q, Keys, Values, Position, Y, dim, heads, kvHeads, scale; query tokens = groups[2])
 * Each computes what strata_embedding, strata_rope_position, strata_kv_append_batch and
 * strata_attention_batch compute for the same values.
 *
 * Two more have no counterpart either. They run the decode step's hyper-connection block
 * (src/engine.js:78-84) in two launches instead of six, with each value formed by the same
 * operations in the same order:
 *   strata_hc_in  (Residual, NormW, DownW, InjectW, Norm, Down, Inject, width, streams, rank, epsilon):
 *                 strata_norm of the streams rows, then the down and inject projections of the norm
 *   strata_hc_out (Norm, Down, UpW, Mixed, width, streams, rank, scale):
 *                 strata_elementwise mode 1, the up projection and strata_hc_mix
 *
 * Six more serve decode of many independent sequences at once (a serving batch; the reference
 * holds one session per engine, src/engine.js:53-72). Token t of a dispatch belongs to sequence t,
 * which has its own position Positions[t] and its own slice of the cache, history or state
 * buffer; each gives sequence t what the one-sequence entry in brackets gives it alone:
 *   strata_rope_seqs      (X, Cos, Sin, Y, Positions, dim, heads, rotary, tokens)   [strata_rope_position]
 *   strata_kv_append_seqs (K, V, Keys, Values, Positions, width, cells, tokens)     [strata_kv_append;
 *                          sequence t's cache is cells [t cells, (t + 1) cells) of Keys / Values]
 *   strata_attention_seqs (Q, Keys, Values, Positions, Y, dim, heads, kvHeads, cells, scale;
 *                          sequences = groups[2])                                   [strata_attention_batch]
 *   strata_conv_seqs      (History, X, W, Y, channels, taps, dilation, activation, tokens)  [strata_conv]
 *   strata_gdn_seqs       (State, Q, K, V, Decay, Beta, Y, dim, keyHeads, valueHeads, tokens) [strata_gdn_step]
 *   strata_argmax_rows    (Logits, Tokens, count, rows)                             [strata_argmax per row]
 * A position outside [0, cells) is reported as an index error, never written.
 *
 * Two more run parts of the delta-rule layer in one launch each, with the same values as the
 * dispatches they replace:
 *   strata_gdn_prep (History, X, W, Q, K, V, keyDim, valueDim, headDim, qScale, epsilon): one
 *     token's strata_conv (4 taps, dilation 1, SiLU) over the [q | k | v] projection, the three
 *     strata_slice and the two strata_norm mode 1 (q heads times qScale, k heads);
 *   strata_gdn_gates_fused (X, AlphaW, BetaW, A, Dt, Decay, Strength, width, heads, tokens): the
 *     alpha and beta projections of each token, then strata_gdn_gates (src/engine.js; the batch
 *     forms of src/prefill.js for tokens > 1). */
int strata_run(strata_ctx *ctx, const char *name, const strata_arg *args, int nargs, const uint32_t groups[3]);

/* ---- synchronisation and introspection (idle, flush, info: src/backend.js:119-120) ---- */
int strata_idle(strata_ctx *ctx);
int strata_flush(strata_ctx *ctx);
/* JSON object: device, SMs, bytes resident, buffers, dispatches, fused calls. */
int strata_info(strata_ctx *ctx, char *json, size_t cap);

/* ---- fused mixture-of-experts layer ----
 * One layer's weights, as resident buffers. The routed experts are the layer's slice of
 * experts.bin: `experts` consecutive Q2 blobs (vendor/strata/tools/pack_layer.py:54-65 with
 * H = width, FF = ff: gate/up codes with rows interleaved g0,u0,g1,..., down codes,
 * gate/up FP16 scales, down FP16 scales; 3*ff*width*9/32 bytes per blob), read by
 * src/model.js:160-167. Replaces the per-layer sequence of src/engine.js:133-156 (decode)
 * and src/prefill.js:52-78 (prompt batches). */
typedef struct {
    int32_t width;           /* hidden size H; multiple of 64 */
    int32_t ff;              /* expert intermediate size; multiple of 64 */
    int32_t experts;         /* 1..512 */
    int32_t top_k;           /* 1..min(experts, 32) */
    strata_buf router;       /* f32 [experts * width]: blk.L.ffn_gate_inp.weight, row-major */
    strata_buf router_bias;  /* 0, or f32 [experts] added to the logits (strata_elementwise mode 5) */
    strata_buf experts_blob; /* u32 [experts * blob_bytes / 4] */
    strata_buf shared_blob;  /* u32 [blob_bytes / 4]: the shared expert as one Q2 blob */
    strata_buf shared_gate;  /* f32 [width]: blk.L.ffn_gate_inp_shexp.weight */
} strata_moe_layer;

/* Whole layer for `tokens` rows of x (f32 [tokens * width]) into y (f32 [tokens * width]),
 * routed ids (i32 [tokens * top_k]) and weights (f32 [tokens * top_k]). Routing is
 * bit-identical to strata_router_batch; y follows the reference's combine order.
 *   mode 0: exact — every dot product in the reference's reduction order (bit-identical y).
 *   mode 1: fast — at H/F = 2048/512 or 2560/640 (other shapes run the exact mode):
 *           tokens <= 8: one persistent integer tensor-core launch (decode);
 *           9 .. 64: the exact router kernels, then one integer tensor-core launch;
 *           above 64: the tcgen05 prefill path (FP16 operands).
 *           Routing is still bit-identical. y is within 1e-5 relative L2 up to 64 tokens and
 *           the same bits run to run (fixed summation order); within 2e-3 above 64 tokens,
 *           where the GEMM epilogues add with atomics.
 * Stream-ordered; does not synchronise. */
#define STRATA_MOE_EXACT 0
#define STRATA_MOE_FAST 1
int strata_moe_forward(strata_ctx *ctx, const strata_moe_layer *layer, strata_buf x, int32_t tokens, strata_buf y, strata_buf ids,
                       strata_buf weights, int32_t mode);

/* Replaces the per-blob check of PackStore.readExpertBlob (src/model.js:160-167), which the
 * whole-model upload skips: every FP16 scale of `count` consecutive Q2 blobs in `blobs` (gate/up
 * and down scale planes) must be finite. Returns STRATA_ERR_LAYOUT "Non-finite expert scales
 * (blob i)" naming the lowest offending blob. Synchronises. The fused kernels convert scales
 * with the hardware FP16 conversion and rely on this check having passed on upload. */
int strata_validate_experts(strata_ctx *ctx, strata_buf blobs, int32_t count, int32_t width, int32_t ff);

/* ---- allocation-free fused layer ----
 * No counterpart in the reference. For callers that must not allocate device memory: a host
 * engine that has already carved HBM into its own arenas and forbids allocations behind its
 * accounting; code running during CUDA stream capture, where cudaMalloc is not allowed;
 * processes that may not grow their device footprint. strata_moe_forward grows a workspace
 * with cudaMalloc. This variant takes caller-owned device pointers and a stream (a
 * cudaStream_t as void*; NULL = the default stream), computes exactly what
 * strata_moe_forward computes in mode STRATA_MOE_EXACT, and keeps all temporaries in one
 * static device array of STRATA_NOALLOC_SCRATCH_BYTES compiled into the library.
 *  - Calls needing more scratch are rejected with STRATA_ERR_RANGE (up to 73 tokens at
 *    H 2048 / E 512 / k 10 / F 512).
 *  - The first call on each device looks the array's address up, so make it before any
 *    stream capture.
 *  - Calls share the array: calls that overlap on the GPU race, so order them on one stream.
 *  - The calling thread's current device must own `stream`, the pointers and the layer, in
 *    the runtime's primary context (the array's address is cached per device ordinal); a
 *    stream of another device is rejected with STRATA_ERR_RANGE.
 *  - A token whose routing fails (NaN probabilities) gets id -1; that pair adds nothing to y.
 *    strata_moe_forward reports it as an error at the next synchronising call; this entry
 *    cannot without synchronising, so check `ids` for -1.
 *  - Never allocates or frees. `msg` (optional) receives the reason for a non-zero status. */
#define STRATA_NOALLOC_SCRATCH_BYTES (8u << 20)
typedef struct {
    int32_t width, ff, experts, top_k;   /* as in strata_moe_layer */
    const float *router;                 /* device f32 [experts * width] */
    const float *router_bias;            /* device f32 [experts], or NULL */
    const uint32_t *experts_blob;        /* device u32: experts Q2 blobs */
    const uint32_t *shared_blob;         /* device u32: one Q2 blob */
    const float *shared_gate;            /* device f32 [width] */
} strata_moe_layer_dev;
int strata_moe_forward_noalloc(const strata_moe_layer_dev *layer, const float *x, int32_t tokens, float *y, int32_t *ids,
                               float *weights, void *stream, char *msg, size_t msg_cap);

/* ---- expert-parallel layer over NCCL (one process per GPU) ----
 * The fused entry point strata_moe_ep (the expert-parallel path of BASELINE's north star; the
 * reference has no multi-GPU path). The 512 (layer.experts) routed experts are sharded evenly:
 * rank r owns the experts its placement gives it (strata_ep_set_placement; by default
 * [r E/n, (r + 1) E/n)), and its layer.experts_blob holds exactly those blobs in ascending id;
 * router, shared gate and shared expert are replicated. A rank passes its own tokens and
 * receives their y, ids and weights (routing over all E experts, bit-exact; y within 2e-3
 * relative L2, the tensor-core path's tolerance).
 * Setup: rank 0 calls strata_ep_unique_id, the 128 bytes are shared by the caller (e.g. a
 * torch.distributed broadcast), every rank calls strata_ep_init. NCCL (libnccl.so.2) is bound
 * at run time. Each forward reads the per-peer row counts back to the host once.
 * Failure detection (no reference counterpart; the reference's nearest is its failed-session
 * state, src/engine.js:147-151, and worker-crash rejection, src/backend.js:165-168): the
 * communicator is non-blocking, and every host wait on the peers (the forward's count read,
 * strata_sync/strata_read and friends, strata_destroy) is bounded by strata_ep_set_timeout
 * (default 60 s). A wait that runs out, or an NCCL asynchronous error, aborts the communicator
 * (ncclCommAbort) and returns STRATA_ERR_CUDA naming the cause; later expert-parallel calls
 * fail until strata_ep_init is called again. The context itself stays usable. */
#define STRATA_EP_ID_BYTES 128
int strata_ep_unique_id(strata_ctx *ctx, uint8_t *id, size_t cap);
int strata_ep_init(strata_ctx *ctx, int32_t rank, int32_t n_ranks, const uint8_t *id);
int strata_ep_set_timeout(strata_ctx *ctx, int32_t milliseconds);
/* Expert placement (no reference counterpart): owner[e] is the rank that holds expert e, for
 * e < experts; every rank must own at least one expert, and every rank must set the same
 * placement. A rank's layer.experts_blob then holds the experts it owns in ascending id order.
 * Without a call (or with owner = NULL) rank r owns experts [r E/n, (r + 1) E/n). A placement
 * balanced by the experts' routed rows keeps a skewed router from loading one rank with the
 * popular experts. Synchronises. strata_ep_local_experts gives this rank's blob count under
 * the placement in force for `experts` (setting the contiguous one if none is). */
int strata_ep_set_placement(strata_ctx *ctx, int32_t experts, const int32_t *owner);
int strata_ep_local_experts(strata_ctx *ctx, int32_t experts, int32_t *count);
int strata_moe_ep_forward(strata_ctx *ctx, const strata_moe_layer *layer, strata_buf x, int32_t tokens, strata_buf y, strata_buf ids,
                          strata_buf weights);
/* Same-device loopback transport (no reference counterpart): n virtual ranks on ONE GPU, one
 * context each, driven by n host threads; the exchanges become device-to-device copies
 * between the ranks' buffers, ordered by stream events (no kernel waits on another rank).
 * Tests the expert-parallel layer at 2, 4 or 8 ranks on a single GPU. The hub's creator calls
 * strata_ep_loopback_create once, every rank's context strata_ep_init_loopback(rank, hub);
 * strata_ep_loopback_release drops the creator's reference (the ranks keep theirs). */
int strata_ep_loopback_create(strata_ctx *ctx, int32_t n_ranks, uint64_t *hub);
int strata_ep_init_loopback(strata_ctx *ctx, int32_t rank, uint64_t hub);
int strata_ep_loopback_release(strata_ctx *ctx, uint64_t hub);

/* ---- per-layer embeddings (PLE) on the device ----
 * Replaces the host-side row gather of src/model.js:230-242 (plePackedRows) followed by the
 * strata_ple_decode dispatch of src/ops.js:79-83. The IQ4_NL table (rows of head_dim values,
 * head_dim / 32 * 18 bytes each: per 32 values an FP16 scale and 16 code bytes) stays resident
 * in `table` (u32 words); the host still computes the n-gram row ids (src/model.js ngramRows)
 * and writes them to `ids` (i32). Values[h * head_dim + j] receive exactly what
 * strata_ple_decode gives for the same rows packed one after another. head_dim must be a
 * multiple of 32 ("Invalid packed PLE layout"). A row outside the table reads zeros and a
 * non-finite scale ("Non-finite PLE scales", src/model.js:241) are reported by the next
 * synchronising call. Stream-ordered. */
int strata_ple_gather_decode(strata_ctx *ctx, strata_buf table, strata_buf ids, int32_t rows, int32_t head_dim, strata_buf values);

/* ---- CUDA graphs of the context's stream (no reference counterpart: the B200 runtime replays
 * captured work instead of relaunching it from the host) ----
 * strata_capture_begin starts capturing the context's stream (thread-local mode): the calls
 * that follow on this thread are recorded, not run. Calls that synchronise (read, idle, free)
 * or that would grow the layer workspace fail while capturing, so run a layer once before
 * capturing it. strata_capture_end instantiates the recorded work and returns a graph handle;
 * strata_graph_launch replays it on the stream (stream-ordered, asynchronous);
 * strata_graph_free synchronises and releases it. The graph keeps the buffers it was captured
 * with: free a graph before freeing its buffers. */
int strata_capture_begin(strata_ctx *ctx);
int strata_capture_end(strata_ctx *ctx, uint64_t *graph);
int strata_graph_launch(strata_ctx *ctx, uint64_t graph);
int strata_graph_free(strata_ctx *ctx, uint64_t graph);

/* ---- device-time profile of the fused layer (diagnostics; no reference counterpart) ----
 * While enabled, strata_moe_forward records CUDA events around its phases on the context's
 * stream. strata_profile_read synchronises, adds the phase times (milliseconds) of every call
 * since the last read into ms[0..n) and resets them; *calls receives the number of calls.
 * Phases: 0 routing (prefill path: router logits, top-k, permutation, activation rows),
 * 1 gate/up tensor-core GEMM, 2 down tensor-core GEMM (prefill and expert-parallel paths),
 * 3 fused decode kernel (decode path), 4 expert-parallel dispatch (counts and rows exchange,
 * regrouping by local expert), 5 expert-parallel return (outputs back to their ranks, combine).
 * strata_moe_ep_forward records phases 0, 4, 1, 2, 5. */
#define STRATA_PHASES 6
int strata_profile(strata_ctx *ctx, int32_t enable);
int strata_profile_read(strata_ctx *ctx, double *ms, int32_t n, uint64_t *calls);

/* ---- seeded synthetic workload (device generator; same bytes as stratacuda_b200/synth.py) ---- */
/* `count` expert blobs of one layer starting at `first_expert` into buf at element offset.
 * `shared` is a flag word: 1 = the shared expert's random streams, 2 = signed FP16 scales
 * N(0, 0.02) instead of |N(0, 0.02)|. */
int strata_synth_blobs(strata_ctx *ctx, strata_buf buf, uint64_t offset, uint64_t seed, int32_t layer, int32_t first_expert,
                       int32_t count, int32_t width, int32_t ff, int32_t shared);
/* `count` normals N(0,1)*scale of stream (seed, tag, sub) from draw `start` into buf at offset. */
int strata_synth_normals(strata_ctx *ctx, strata_buf buf, uint64_t offset, uint64_t seed, uint64_t tag, uint64_t sub, uint64_t start,
                         uint64_t count, double scale);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
