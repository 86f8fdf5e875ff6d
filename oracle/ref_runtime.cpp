// TEST INFRASTRUCTURE (oracle/_ref recipe). Compiles the reference's kernels/strata.cu in
// place (its path arrives as STRATA_REF_SOURCE from oracle/build_ref.py) together with a
// fiber runtime that gives each 64-lane workgroup the semantics of the reference's CPU
// runtime (vendor/webcuda/src/wasm/thread-pool.hpp:18-65, compile.mjs:30-37), and exports
// ref_<entry>(gx, gy, gz, params...) for the mixture-of-experts entries, mirroring the
// cw_<entry> wrappers of compile.mjs:39. Output goes to oracle/_ref/ only.
#include "ref_shim.hpp"
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>
#include <cstdlib>
#include <xmmintrin.h>

struct StrataRefLane {
    void *sp = nullptr;
    StrataRefIndex idx;
    int site = -1;
    bool done = false;
};
thread_local StrataRefLane *strata_ref_current = nullptr;
thread_local StrataRefIndex blockIdx, blockDim, gridDim;
const StrataRefIndex &strata_ref_thread_index() { return strata_ref_current->idx; }

// Minimal x86-64 SysV context switch: save callee-saved registers, MXCSR and the x87 control
// word on the current stack, store the stack pointer, load the other one, restore, return.
extern "C" void strata_ref_switch(void **save, void *load);
asm(R"(
.text
.globl strata_ref_switch
.type strata_ref_switch,@function
strata_ref_switch:
    pushq %rbp
    pushq %rbx
    pushq %r12
    pushq %r13
    pushq %r14
    pushq %r15
    subq $8, %rsp
    stmxcsr (%rsp)
    fnstcw 4(%rsp)
    movq %rsp, (%rdi)
    movq %rsi, %rsp
    ldmxcsr (%rsp)
    fldcw 4(%rsp)
    addq $8, %rsp
    popq %r15
    popq %r14
    popq %r13
    popq %r12
    popq %rbx
    popq %rbp
    ret
.size strata_ref_switch,.-strata_ref_switch
)");

namespace {
constexpr int kLanes = 64;
constexpr size_t kStack = 64 * 1024;

struct Worker {
    void *sched_sp = nullptr;
    StrataRefLane lanes[kLanes];
    unsigned char *stacks = nullptr;
    const std::function<void()> *body = nullptr;
};
thread_local Worker *tl_worker = nullptr;

[[noreturn]] void lane_entry() {
    Worker *w = tl_worker;
    (*w->body)();
    strata_ref_current->done = true;
    for (;;) strata_ref_switch(&strata_ref_current->sp, w->sched_sp);
}

void prepare_lane(Worker *w, int lane) {
    unsigned char *top = w->stacks + (size_t)(lane + 1) * kStack;
    uintptr_t t = reinterpret_cast<uintptr_t>(top) & ~uintptr_t(15);
    uintptr_t sp = t - 64 - 8;  // after the 56-byte restore and `ret`, rsp == t - 8 (entry alignment)
    uint64_t *frame = reinterpret_cast<uint64_t *>(sp);
    uint32_t csr = _mm_getcsr();
    uint16_t cw;
    asm volatile("fnstcw %0" : "=m"(cw));
    std::memcpy(reinterpret_cast<unsigned char *>(frame), &csr, 4);
    std::memcpy(reinterpret_cast<unsigned char *>(frame) + 4, &cw, 2);
    for (int i = 1; i <= 6; ++i) frame[i] = 0;
    frame[7] = reinterpret_cast<uint64_t>(&lane_entry);
    StrataRefLane &l = w->lanes[lane];
    l.sp = reinterpret_cast<void *>(sp);
    l.idx = StrataRefIndex{(unsigned)lane, 0, 0};
    l.site = -1;
    l.done = false;
}

// Runs one workgroup: resume every live lane until all have finished; all live lanes must
// stop at the same barrier site each round (else: divergent barrier, as cw_fault).
bool run_group(Worker *w) {
    for (int lane = 0; lane < kLanes; ++lane) prepare_lane(w, lane);
    for (;;) {
        int finished = 0, site = -1;
        bool mismatch = false;
        for (int lane = 0; lane < kLanes; ++lane) {
            StrataRefLane &l = w->lanes[lane];
            if (!l.done) {
                strata_ref_current = &l;
                strata_ref_switch(&w->sched_sp, l.sp);
            }
            if (l.done) ++finished;
            else if (site < 0) site = l.site;
            else if (site != l.site) mismatch = true;
        }
        if (finished == kLanes) return true;
        if (finished || mismatch) return false;
    }
}

// Pool state lives for the whole process (never destroyed), so that exit() with parked
// workers neither runs std::thread destructors on joinable threads nor destroys a
// condition variable that workers wait on.
struct Pool {
    std::mutex mutex;
    std::condition_variable work, done;
    std::vector<std::thread> threads;
    unsigned epoch = 0, finished = 0, count = 0;
    bool stop = false;
    std::atomic<unsigned> next{0};
    std::atomic<int> fault{0};
    std::function<void(unsigned)> job;
};
Pool &pool = *new Pool();

Worker *worker_for_thread() {
    if (!tl_worker) {
        tl_worker = new Worker();
        tl_worker->stacks = static_cast<unsigned char *>(std::aligned_alloc(64, kStack * kLanes));
    }
    return tl_worker;
}
void consume(const std::function<void(unsigned)> &job) {
    for (;;) {
        unsigned i = pool.next.fetch_add(1, std::memory_order_relaxed);
        if (i >= pool.count) break;
        job(i);
    }
}
}  // namespace

void strata_ref_barrier(int site) {
    strata_ref_current->site = site;
    strata_ref_switch(&strata_ref_current->sp, tl_worker->sched_sp);
}

extern "C" int ref_init(int count) {
    if (!pool.threads.empty() || count < 1 || count > 8) return -1;  // thread-pool.hpp:49 limit
    pool.stop = false;
    for (int i = 1; i < count; ++i)
        pool.threads.emplace_back([] {
            unsigned epoch = 0;
            for (;;) {
                std::unique_lock<std::mutex> lock(pool.mutex);
                pool.work.wait(lock, [&] { return pool.stop || pool.epoch != epoch; });
                if (pool.stop) return;
                epoch = pool.epoch;
                auto job = pool.job;
                lock.unlock();
                consume(job);
                lock.lock();
                ++pool.finished;
                pool.done.notify_one();
            }
        });
    return count;
}
extern "C" int ref_threads() { return (int)pool.threads.size() + 1; }
extern "C" void ref_shutdown() {
    {
        std::lock_guard<std::mutex> lock(pool.mutex);
        pool.stop = true;
    }
    pool.work.notify_all();
    for (auto &t : pool.threads) t.join();
    pool.threads.clear();
}

static int ref_parallel(unsigned gx, unsigned gy, unsigned gz, const std::function<void()> &body) {
    unsigned count = gx * gy * gz;
    std::function<void(unsigned)> job = [=, &body](unsigned index) {
        Worker *w = worker_for_thread();
        w->body = &body;
        blockDim = StrataRefIndex{(unsigned)kLanes, 1, 1};
        gridDim = StrataRefIndex{gx, gy, gz};
        blockIdx = StrataRefIndex{index % gx, (index / gx) % gy, index / (gx * gy)};
        if (!run_group(w)) pool.fault = 1;
    };
    {
        std::lock_guard<std::mutex> lock(pool.mutex);
        pool.job = job;
        pool.count = count;
        pool.finished = 0;
        pool.next = 0;
        pool.fault = 0;
        ++pool.epoch;
    }
    pool.work.notify_all();
    consume(job);
    std::unique_lock<std::mutex> lock(pool.mutex);
    pool.done.wait(lock, [] { return pool.finished == pool.threads.size(); });
    pool.job = {};
    return pool.fault.load();
}

// ---- the reference's kernels, compiled unmodified ----
#include STRATA_REF_SOURCE

#define P(...) __VA_ARGS__
#define REF_ENTRY(name, params, args) \
    extern "C" int ref_##name(unsigned gx, unsigned gy, unsigned gz, params) { return ref_parallel(gx, gy, gz, [=] { name(args); }); }

REF_ENTRY(strata_unpack_half, P(const unsigned int *Packed, float *Values, int count), P(Packed, Values, count))
REF_ENTRY(strata_expert_scales, P(const unsigned int *Blob, float *Scales, int offset, int count), P(Blob, Scales, offset, count))
REF_ENTRY(strata_ple_decode, P(const unsigned int *Packed, float *Values, int count), P(Packed, Values, count))
REF_ENTRY(strata_q2_gate_up,
          P(const float *X, const unsigned int *Blob, const float *Scales, const int *Mapping, float *Hidden, int width, int ff,
            int tokens, int mapped, int expanded, int codeOffset, int scaleOffset),
          P(X, Blob, Scales, Mapping, Hidden, width, ff, tokens, mapped, expanded, codeOffset, scaleOffset))
REF_ENTRY(strata_q2_down,
          P(const float *Hidden, const unsigned int *Blob, const float *Scales, const int *Mapping, float *Y, int width, int ff,
            int tokens, int mapped, int expanded, int outputOffset, int codeOffset, int scaleOffset),
          P(Hidden, Blob, Scales, Mapping, Y, width, ff, tokens, mapped, expanded, outputOffset, codeOffset, scaleOffset))
REF_ENTRY(strata_project,
          P(const float *X, const float *W, float *Y, int cols, int rows, int tokens, int outputStride, int outputOffset),
          P(X, W, Y, cols, rows, tokens, outputStride, outputOffset))
REF_ENTRY(strata_bf16_project,
          P(const float *X, const unsigned int *Codes, float *Y, int cols, int rows, int tokens, int outputStride, int outputOffset),
          P(X, Codes, Y, cols, rows, tokens, outputStride, outputOffset))
REF_ENTRY(strata_q2_project,
          P(const float *X, const unsigned int *Blob, float *Y, int cols, int rows, int tokens, int outputStride, int outputOffset,
            int codeOffset, int scaleOffset, int weightRow, int rowStride),
          P(X, Blob, Y, cols, rows, tokens, outputStride, outputOffset, codeOffset, scaleOffset, weightRow, rowStride))
REF_ENTRY(strata_quant_project,
          P(const float *X, const unsigned int *Codes, const float *Scales, const float *Offsets, float *Y, int cols, int rows,
            int tokens, int outputStride, int outputOffset, int bits, int groupSize, int bias, int codebook, int hasOffset),
          P(X, Codes, Scales, Offsets, Y, cols, rows, tokens, outputStride, outputOffset, bits, groupSize, bias, codebook,
            hasOffset))
REF_ENTRY(strata_elementwise, P(const float *A, const float *B, float *Y, int n, int mode, float scale), P(A, B, Y, n, mode, scale))
REF_ENTRY(strata_router, P(const float *Logits, int *Ids, float *Weights, int experts, int topK), P(Logits, Ids, Weights, experts, topK))
REF_ENTRY(strata_router_batch, P(const float *Logits, int *Ids, float *Weights, int experts, int topK),
          P(Logits, Ids, Weights, experts, topK))
REF_ENTRY(strata_moe_combine,
          P(const float *Parts, const float *Weights, const float *Shared, const float *SharedGate, float *Y, int width, int count),
          P(Parts, Weights, Shared, SharedGate, Y, width, count))
REF_ENTRY(strata_moe_combine_batch,
          P(const float *Parts, const float *Weights, const float *Shared, const float *SharedGate, float *Y, int width, int count,
            int tokens),
          P(Parts, Weights, Shared, SharedGate, Y, width, count, tokens))
REF_ENTRY(strata_gather_rows, P(const float *X, const int *Indices, float *Y, int width, int rows), P(X, Indices, Y, width, rows))
REF_ENTRY(strata_scatter_rows, P(const float *X, const int *Indices, float *Y, int width, int rows), P(X, Indices, Y, width, rows))

// The remaining entries (kernels/strata.cu:72-534).
REF_ENTRY(strata_embedding, P(float *Values, unsigned int *Codes, float *Scales, float *Offsets, float *Residual, int width, int streams, int outputOffset, int format, int bits, int groupSize, int bias, int codebook, int hasOffset),
          P(Values, Codes, Scales, Offsets, Residual, width, streams, outputOffset, format, bits, groupSize, bias, codebook, hasOffset))
REF_ENTRY(strata_embed, P(float *Row, float *Residual, int width, int streams),
          P(Row, Residual, width, streams))
REF_ENTRY(strata_embed_batch, P(float *Rows, float *Residual, int width, int streams, int tokens),
          P(Rows, Residual, width, streams, tokens))
REF_ENTRY(strata_rope_frequencies, P(float *High, float *Low, int rotary, float base),
          P(High, Low, rotary, base))
REF_ENTRY(strata_rope_table, P(float *High, float *Low, float *Cos, float *Sin, int rotary, int context),
          P(High, Low, Cos, Sin, rotary, context))
REF_ENTRY(strata_rope_position, P(float *X, float *Cos, float *Sin, float *Y, int dim, int heads, int rotary, int position, int tokens),
          P(X, Cos, Sin, Y, dim, heads, rotary, position, tokens))
REF_ENTRY(strata_rope, P(float *X, float *Cos, float *Sin, float *Y, int dim, int heads, int rotary),
          P(X, Cos, Sin, Y, dim, heads, rotary))
REF_ENTRY(strata_rope_batch, P(float *X, float *Cos, float *Sin, float *Y, int dim, int heads, int rotary, int tokens),
          P(X, Cos, Sin, Y, dim, heads, rotary, tokens))
REF_ENTRY(strata_gemv, P(float *X, float *W, float *Y, int cols, int rows, int tokens),
          P(X, W, Y, cols, rows, tokens))
REF_ENTRY(strata_quant_gemv, P(float *X, unsigned int *Codes, float *Scales, float *Offsets, float *Y, int cols, int rows, int bits, int groupSize, int bias, int codebook, int hasOffset),
          P(X, Codes, Scales, Offsets, Y, cols, rows, bits, groupSize, bias, codebook, hasOffset))
REF_ENTRY(strata_norm, P(float *X, float *W, float *Y, int cols, int rows, int weightRows, int mode, float epsilon, float scale),
          P(X, W, Y, cols, rows, weightRows, mode, epsilon, scale))
REF_ENTRY(strata_ple_gate, P(float *Key, float *Query, float *Gate, int width, int streams),
          P(Key, Query, Gate, width, streams))
REF_ENTRY(strata_argmax, P(float *Logits, int *Token, int count),
          P(Logits, Token, count))
REF_ENTRY(strata_attention, P(float *Q, float *Keys, float *Values, int *Cells, float *Y, int dim, int heads, int kvHeads, int count, float scale),
          P(Q, Keys, Values, Cells, Y, dim, heads, kvHeads, count, scale))
REF_ENTRY(strata_attention_batch, P(float *Q, float *Keys, float *Values, float *Y, int dim, int heads, int kvHeads, int position, float scale),
          P(Q, Keys, Values, Y, dim, heads, kvHeads, position, scale))
REF_ENTRY(strata_kv_append, P(float *K, float *V, float *Keys, float *Values, int width, int position),
          P(K, V, Keys, Values, width, position))
REF_ENTRY(strata_kv_append_batch, P(float *K, float *V, float *Keys, float *Values, int width, int position, int tokens),
          P(K, V, Keys, Values, width, position, tokens))
REF_ENTRY(strata_attention_gate, P(float *Attention, float *FullQ, float *Y, int dim, int heads),
          P(Attention, FullQ, Y, dim, heads))
REF_ENTRY(strata_attention_gate_batch, P(float *Attention, float *FullQ, float *Y, int dim, int heads, int tokens),
          P(Attention, FullQ, Y, dim, heads, tokens))
REF_ENTRY(strata_slice, P(float *X, float *Y, int width, int rows, int stride, int offset),
          P(X, Y, width, rows, stride, offset))
REF_ENTRY(strata_hc_mix, P(float *Norm, float *Gate, float *Mixed, int width, int streams),
          P(Norm, Gate, Mixed, width, streams))
REF_ENTRY(strata_hc_mix_batch, P(float *Norm, float *Gate, float *Mixed, int width, int streams, int tokens),
          P(Norm, Gate, Mixed, width, streams, tokens))
REF_ENTRY(strata_hc_write, P(float *Residual, float *Output, float *Inject, int width, int streams),
          P(Residual, Output, Inject, width, streams))
REF_ENTRY(strata_hc_write_batch, P(float *Residual, float *Output, float *Inject, int width, int streams, int tokens),
          P(Residual, Output, Inject, width, streams, tokens))
REF_ENTRY(strata_ple_broadcast, P(float *Value, float *Gate, float *Y, int width, int streams),
          P(Value, Gate, Y, width, streams))
REF_ENTRY(strata_ple_broadcast_batch, P(float *Value, float *Gate, float *Y, int width, int streams, int tokens),
          P(Value, Gate, Y, width, streams, tokens))
REF_ENTRY(strata_ple_add, P(float *Residual, float *Gated, float *Conv, int n),
          P(Residual, Gated, Conv, n))
REF_ENTRY(strata_conv, P(float *History, float *X, float *W, float *Y, int channels, int taps, int dilation, int activation),
          P(History, X, W, Y, channels, taps, dilation, activation))
REF_ENTRY(strata_conv_batch, P(float *History, float *X, float *W, float *Y, int channels, int taps, int dilation, int activation, int tokens),
          P(History, X, W, Y, channels, taps, dilation, activation, tokens))
REF_ENTRY(strata_gdn_gates, P(float *Alpha, float *Beta, float *A, float *Dt, float *Decay, float *Strength, int heads),
          P(Alpha, Beta, A, Dt, Decay, Strength, heads))
REF_ENTRY(strata_gdn_gates_batch, P(float *Alpha, float *Beta, float *A, float *Dt, float *Decay, float *Strength, int heads, int tokens),
          P(Alpha, Beta, A, Dt, Decay, Strength, heads, tokens))
REF_ENTRY(strata_gdn_step, P(float *State, float *Q, float *K, float *V, float *Decay, float *Beta, float *Y, int dim, int keyHeads, int valueHeads),
          P(State, Q, K, V, Decay, Beta, Y, dim, keyHeads, valueHeads))
REF_ENTRY(strata_gdn_batch, P(float *State, float *Q, float *K, float *V, float *Decay, float *Beta, float *Y, int dim, int keyHeads, int valueHeads, int tokens),
          P(State, Q, K, V, Decay, Beta, Y, dim, keyHeads, valueHeads, tokens))
