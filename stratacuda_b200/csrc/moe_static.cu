// Allocation-free variant of the fused mixture-of-experts layer.
//
// Who needs it: some callers of this library must not allocate device memory. Examples
// are a host engine that has already reserved and carved up all of HBM for resident
// weights and will not let a plugin call cudaMalloc behind its accounting, code running
// while a CUDA stream is being captured (cudaMalloc is not allowed there), and a process
// without permission to grow its device footprint after start-up. The handle-based
// strata_moe_forward grows a per-context workspace with cudaMalloc, so those callers
// cannot use it. This entry takes caller-owned device pointers and a stream, and does all
// of its temporary work in one fixed scratch array compiled into the library. It allocates
// nothing.
//
// Cost and limits:
//   * The scratch is a file-scope static device array of STRATA_NOALLOC_SCRATCH_BYTES
//     (8 MiB). Every GPU that loads the library holds it until the process exits.
//   * A call whose scratch need exceeds it is rejected with STRATA_ERR_RANGE and a message.
//     At H 2048 / E 512 / k 10 / F 512 that means up to 73 tokens.
//   * Every call shares the one array, and it keeps the previous call's contents. Each call
//     writes every scratch byte it later reads (the counting sort, hidden rows and shared
//     outputs), so nothing has to start at zero. The one exception is a token whose routing
//     failed (its probabilities are NaN, so an id is -1): that pair has no parts row, and the
//     combine skips it rather than read an older call's row. The reference rejects such a
//     routing ("Invalid expert routing result", src/engine.js:138); this entry cannot report
//     it without synchronising, so the -1 in `ids` is the caller's signal.
//     Two calls that overlap on the GPU (different streams, or different host threads
//     without ordering) race on the array and produce wrong results. Order them on one
//     stream.
//   * In host code the symbol below is only a host-side stand-in for the device array;
//     passing it to a kernel would fault. The device address is therefore looked up once per
//     device, with that device current, by cudaGetSymbolAddress on the first call made on
//     that device. Make that first call before starting any stream capture.
//   * The calling thread's current device must be the device of `stream`, of every pointer
//     and of the layer, in the runtime's primary context of that device (the address cache is
//     keyed by device ordinal). A stream of another device is rejected.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/strata_cuda.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = STRATA_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes == (8u << 20), "the documented limit is 8 MiB");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lookup_mutex;
void *g_scratch_on_device[kMaxDevices] = {};

int say(char *msg, size_t cap, int code, const char *text) {
    if (msg && cap) snprintf(msg, cap, "%s", text);
    return code;
}

}  // namespace

extern "C" int strata_moe_forward_noalloc(const strata_moe_layer_dev *layer, const float *x, int32_t tokens, float *y, int32_t *ids,
                                          float *weights, void *stream, char *msg, size_t msg_cap) {
    if (msg && msg_cap) msg[0] = 0;
    if (!layer) return say(msg, msg_cap, STRATA_ERR_RANGE, "null layer");
    const strata_moe_layer_dev &l = *layer;
    if (l.width <= 0 || l.ff <= 0 || l.width % 64 || l.ff % 64)
        return say(msg, msg_cap, STRATA_ERR_LAYOUT, "Packed expert dimensions must contain complete groups");
    if (l.experts < 1 || l.experts > 512 || l.top_k < 1 || l.top_k > (l.experts < 32 ? l.experts : 32))
        return say(msg, msg_cap, STRATA_ERR_RANGE, "Router supports 1-512 experts and topK <= min(experts,32)");
    if (tokens < 1) return say(msg, msg_cap, STRATA_ERR_RANGE, "tokens must be an integer >= 1");
    if (!l.router || !l.experts_blob || !l.shared_blob || !l.shared_gate || !x || !y || !ids || !weights)
        return say(msg, msg_cap, STRATA_ERR_RANGE, "null device pointer");
    const size_t need = strata::moe_scratch_bytes(tokens, l.width, l.ff, l.experts, l.top_k);
    if (need > kScratchBytes) {
        char text[256];
        snprintf(text, sizeof text,
                 "strata_moe_forward_noalloc: this call needs %zu bytes of scratch, which exceeds the fixed %zu-byte array; "
                 "use fewer tokens per call or strata_moe_forward",
                 need, kScratchBytes);
        return say(msg, msg_cap, STRATA_ERR_RANGE, text);
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return say(msg, msg_cap, STRATA_ERR_CUDA, cudaGetErrorString(e));
    if (device < 0 || device >= kMaxDevices) return say(msg, msg_cap, STRATA_ERR_RANGE, "device ordinal out of range");
    if (stream) {
        int stream_device = -1;
        e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_device);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return say(msg, msg_cap, STRATA_ERR_CUDA, cudaGetErrorString(e));
        }
        if (stream_device != device)
            return say(msg, msg_cap, STRATA_ERR_RANGE,
                       "strata_moe_forward_noalloc: the stream belongs to another device than the calling thread's current device");
    }
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_lookup_mutex);
        if (!g_scratch_on_device[device]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // the calling thread's current device is `device`
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                return say(msg, msg_cap, STRATA_ERR_CUDA, e != cudaSuccess ? cudaGetErrorString(e) : "null scratch address");
            }
            g_scratch_on_device[device] = p;
        }
        scratch = g_scratch_on_device[device];
    }
    const long long blob_words = 3LL * l.ff * l.width / 16 + 3LL * l.ff * l.width / 128;
    strata::MoeLayerDev L{l.width, l.ff, l.experts, l.top_k, l.router, l.router_bias, l.experts_blob, blob_words, l.shared_blob,
                          l.shared_gate};
    strata::MoeScratch s = strata::moe_scratch_carve(scratch, tokens, l.width, l.ff, l.experts, l.top_k);
    e = strata::moe_forward_exact(L, x, tokens, y, ids, weights, s, static_cast<cudaStream_t>(stream), nullptr);
    if (e != cudaSuccess) return say(msg, msg_cap, STRATA_ERR_CUDA, cudaGetErrorString(e));
    return STRATA_OK;
}
