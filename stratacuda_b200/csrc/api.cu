// C-ABI of libstrata_cuda (include/strata_cuda.h): contexts, stream-ordered buffers,
// by-name dispatch of the reference entries with the reference's argument validation, the
// fused mixture-of-experts layer and the synthetic-workload generator.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <cmath>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/strata_cuda.h"
#include "kernels.h"

using namespace strata;

constexpr int kFastSyncWords = 4 + kDecode1SyncWords;

struct Buffer {
    void *ptr;
    uint64_t length;  // elements of 4 bytes
    int type;
};

struct strata_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::unordered_map<uint64_t, Buffer> buffers;
    uint64_t next_handle = 1;
    uint64_t bytes_resident = 0;
    unsigned *err_dev = nullptr;   // device error word (kErr* bits)
    unsigned *err_host = nullptr;  // pinned mirror
    unsigned *fast_sync = nullptr; // grid-arrival words of the fast kernels (self-resetting): [0, 4) batch decode and
                                   // medium layers, [4, 4 + kDecode1SyncWords) the one-token decode layer
    int *check_dev = nullptr;      // strata_validate_experts result
    void *decode1_xchg = nullptr;  // the one-token decode layer's exchange words (zeroed at creation)
    void *workspace = nullptr;
    size_t workspace_bytes = 0;
    uint64_t dispatches = 0, fused_calls = 0;
    // strata_profile: event pairs (phase, start, end) awaiting strata_profile_read
    bool profile = false;
    struct Mark {
        int phase;
        cudaEvent_t a, b;
    };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> spare_events;
    uint64_t profiled_calls = 0;
    EpComm *ep = nullptr;  // strata_ep_init / strata_ep_init_loopback
    long long ep_timeout_ms = 60000;  // strata_ep_set_timeout
    // strata_capture_*: the stream is being captured; instantiated graphs by handle
    bool capturing = false;
    struct Graph {
        cudaGraph_t g;
        cudaGraphExec_t exec;
    };
    std::unordered_map<uint64_t, Graph> graphs;
    uint64_t next_graph = 1;
    std::string last_error;
    char device_name[256] = {0};
    int sms = 0;
};

namespace {

int fail(strata_ctx *ctx, int code, const char *fmt, ...) {
    char msg[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof msg, fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = msg;
    return code;
}

int cuda_fail(strata_ctx *ctx, cudaError_t e, const char *what) {
    return fail(ctx, STRATA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define CUDA_OR_FAIL(ctx, expr, what)                           \
    do {                                                        \
        cudaError_t _e = (expr);                                \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, what); \
    } while (0)

int use_device(strata_ctx *ctx) {
    cudaError_t e = cudaSetDevice(ctx->device);
    return e == cudaSuccess ? STRATA_OK : cuda_fail(ctx, e, "cudaSetDevice");
}

Buffer *find(strata_ctx *ctx, strata_buf h) {
    auto it = ctx->buffers.find(h);
    return it == ctx->buffers.end() ? nullptr : &it->second;
}

// Reads back and clears the device error word; the stream must already be synchronised.
int check_device_errors(strata_ctx *ctx) {
    unsigned e = *ctx->err_host;
    if (!e) return STRATA_OK;
    *ctx->err_host = 0;
    cudaMemsetAsync(ctx->err_dev, 0, sizeof(unsigned), ctx->stream);
    std::string what;
    if (e & kErrIndex) what += "an index outside its buffer was skipped; ";
    if (e & kErrRouting) what += "invalid expert routing result; ";
    if (e & kErrWaitTimeout) what += "a bounded device wait timed out; ";
    if (e & kErrPleScale) what += "Non-finite PLE scales; ";
    return fail(ctx, STRATA_ERR_DEVICE, "device check failed: %s", what.c_str());
}

int sync(strata_ctx *ctx) {
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "synchronising calls are not allowed while the stream is captured");
    CUDA_OR_FAIL(ctx, cudaMemcpyAsync(ctx->err_host, ctx->err_dev, sizeof(unsigned), cudaMemcpyDeviceToHost, ctx->stream),
                 "error word readback");
    if (ctx->ep) {  // the stream may hold exchanges with the peers: a bounded wait, never a hang
        std::string msg;
        if (ep_wait(ctx->ep, ctx->stream, &msg)) return fail(ctx, STRATA_ERR_CUDA, "expert-parallel peers: %s", msg.c_str());
    } else {
        CUDA_OR_FAIL(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    }
    return check_device_errors(ctx);
}

// ---- reference dispatch table (parsed once from kernels.h specs)
struct Param {
    std::string name;
    char kind;
};
struct Entry {
    const KernelSpec *spec;
    std::vector<Param> params;
};
std::vector<Entry> &entries() {
    static std::vector<Entry> table;
    static std::once_flag once;
    std::call_once(once, [] {
        std::vector<const KernelSpec *> specs;
        for (int k = 0; k < kNumKernels; ++k) specs.push_back(&kKernels[k]);
        for (int k = 0; k < kNumEngineKernels; ++k) specs.push_back(&kEngineKernels[k]);
        for (const KernelSpec *spec : specs) {
            Entry e{spec, {}};
            const char *p = spec->params;
            while (*p) {
                while (*p == ' ') ++p;
                const char *c = strchr(p, ':');
                if (!c) break;
                e.params.push_back(Param{std::string(p, c - p), c[1]});
                p = c + 2;
            }
            table.push_back(std::move(e));
        }
    });
    return table;
}

// src/backend.js:5-8 requireInteger(n, label, min=1, max=2^31-1)
bool int_in(long long v, long long lo = 1, long long hi = 0x7fffffff) { return v >= lo && v <= hi; }

// src/backend.js:10-56 for the entries this library serves. Returns 0 or an error code.
int validate(strata_ctx *ctx, const char *name, const std::vector<Param> &params, const std::vector<KArg> &a, const uint32_t groups[3]) {
    auto idx = [&](const char *p) {
        for (size_t i = 0; i < params.size(); ++i)
            if (params[i].name == p) return (int)i;
        return -1;
    };
    auto I = [&](const char *p) { return (long long)a[idx(p)].i; };
    auto len = [&](const char *p) { return a[idx(p)].len; };
    const std::string n(name);
    if (n == "strata_router" || n == "strata_router_batch") {
        if (!int_in(I("experts")) || !int_in(I("topK")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.experts and %s.topK must be integers in [1, 2147483647]", name, name);
        if (I("experts") > 512 || I("topK") > std::min(I("experts"), 32LL))
            return fail(ctx, STRATA_ERR_RANGE, "Router supports 1-512 experts and topK <= min(experts,32)");
    }
    if (n == "strata_quant_project" || n == "strata_quant_gemv") {
        long long bits = I("bits");
        if (bits != 2 && bits != 4 && bits != 8) return fail(ctx, STRATA_ERR_RANGE, "Canonical code width must be 2, 4 or 8");
        if (!int_in(I("cols")) || !int_in(I("groupSize")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.cols and groupSize must be positive integers", name);
        if (I("cols") % I("groupSize") || I("cols") * I("rows") * bits > 0x7fffffffLL)
            return fail(ctx, STRATA_ERR_RANGE, "Quantized rows must contain whole groups and fit 31-bit indexing");
    }
    if (n == "strata_project" || n == "strata_quant_project" || n == "strata_bf16_project" || n == "strata_q2_project") {
        for (const char *p : {"tokens", "rows", "cols", "outputStride"})
            if (!int_in(I(p))) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p);
        if (!int_in(I("outputOffset"), 0)) return fail(ctx, STRATA_ERR_RANGE, "projection output offset must be an integer >= 0");
        if (I("outputOffset") + I("rows") > I("outputStride") || I("tokens") * I("outputStride") > len("Y") ||
            I("tokens") * I("cols") > len("X"))
            return fail(ctx, STRATA_ERR_LAYOUT, "Projection batch exceeds buffer layout");
    }
    if (n == "strata_q2_project") {
        if (I("cols") % 64) return fail(ctx, STRATA_ERR_LAYOUT, "Q2 expert columns must contain complete groups");
        for (const char *p : {"codeOffset", "scaleOffset", "weightRow"})
            if (!int_in(I(p), 0)) return fail(ctx, STRATA_ERR_RANGE, "%s must be an integer >= 0", p);
        if (!int_in(I("rowStride"), 1, 2)) return fail(ctx, STRATA_ERR_RANGE, "expert row stride must be an integer in [1, 2]");
    }
    if (n == "strata_ple_decode") {  // src/backend.js:29
        if (!int_in(I("count"))) return fail(ctx, STRATA_ERR_RANGE, "%s.count must be an integer in [1, 2147483647]", name);
        if (I("count") % 32 || (I("count") / 32 * 18 + 3) / 4 > len("Packed") || I("count") > len("Values"))
            return fail(ctx, STRATA_ERR_LAYOUT, "Invalid packed PLE layout");
    }
    if (n == "strata_q2_gate_up" || n == "strata_q2_down") {
        if (!int_in(I("width")) || !int_in(I("ff")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.width and ff must be positive integers", name);
        if (I("width") % 64 || I("ff") % 64) return fail(ctx, STRATA_ERR_LAYOUT, "Packed expert dimensions must contain complete groups");
        if (!int_in(I("tokens"))) return fail(ctx, STRATA_ERR_RANGE, "%s.tokens must be an integer in [1, 2147483647]", name);
        if (len("Hidden") < I("tokens") * I("ff") || (I("mapped") && len("Mapping") < I("tokens") * 2))
            return fail(ctx, STRATA_ERR_LAYOUT, "Packed expert batch exceeds buffer layout");
        if (n == "strata_q2_down" && !int_in(I("outputOffset"), 0))
            return fail(ctx, STRATA_ERR_RANGE, "expert output offset must be an integer >= 0");
    }
    if (n == "strata_embedding") {
        if (!int_in(I("width")) || !int_in(I("streams")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.width and streams must be integers in [1, 2147483647]", name);
        if (!int_in(I("outputOffset"), 0)) return fail(ctx, STRATA_ERR_RANGE, "embedding output offset must be an integer >= 0");
        const long long format = I("format");
        if (I("outputOffset") + I("width") * I("streams") > len("Residual") || format < 0 || format > 2)
            return fail(ctx, STRATA_ERR_LAYOUT, "Embedding exceeds buffer layout");
        if (format == 2) {
            const long long bits = I("bits");
            if (!int_in(I("groupSize"))) return fail(ctx, STRATA_ERR_RANGE, "%s.groupSize must be an integer in [1, 2147483647]", name);
            if ((bits != 2 && bits != 4 && bits != 8) || I("width") % I("groupSize"))
                return fail(ctx, STRATA_ERR_LAYOUT, "Invalid packed embedding layout");
        }
    }
    if (n == "strata_rope_position") {
        if (!int_in(I("position"), 0, 2047)) return fail(ctx, STRATA_ERR_RANGE, "RoPE position must be an integer in [0, 2047]");
        for (const char *p : {"rotary", "dim", "heads", "tokens"})
            if (!int_in(I(p))) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p);
        if (I("rotary") % 2 || I("rotary") > I("dim") || I("position") + I("tokens") > 2048 ||
            len("Cos") < (I("position") + I("tokens")) * I("rotary") / 2 || len("Sin") != len("Cos") ||
            len("X") != I("dim") * I("heads") * I("tokens") || len("Y") != len("X"))
            return fail(ctx, STRATA_ERR_LAYOUT, "Invalid RoPE layout");
    }
    if (n == "strata_rope_frequencies") {
        const float base = a[idx("base")].f;
        if (!int_in(I("rotary"))) return fail(ctx, STRATA_ERR_RANGE, "%s.rotary must be an integer in [1, 2147483647]", name);
        if (!std::isfinite(base) || base <= 1.0f || I("rotary") % 2) return fail(ctx, STRATA_ERR_LAYOUT, "Invalid RoPE frequencies");
    }
    if (n == "strata_attention" || n == "strata_attention_batch") {
        for (const char *p : {"heads", "kvHeads", "dim"})
            if (!int_in(I(p))) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p);
        if (I("heads") % I("kvHeads"))  // a RangeError for decode, an Error for prompts (src/backend.js:37,41)
            return fail(ctx, n == "strata_attention" ? STRATA_ERR_RANGE : STRATA_ERR_LAYOUT, "Attention heads must be divisible by KV heads");
        if (n == "strata_attention" && !int_in(I("count"), 1, 2048))
            return fail(ctx, STRATA_ERR_RANGE, "attention selected cells must be an integer in [1, 2048]");
        if (n == "strata_attention_batch") {
            if (!int_in(I("position"), 0, 2047)) return fail(ctx, STRATA_ERR_RANGE, "attention position must be an integer in [0, 2047]");
            const long long row = I("heads") * I("dim");
            if (len("Q") % row || I("position") + len("Q") / row > 2048)
                return fail(ctx, STRATA_ERR_LAYOUT, "Batched attention exceeds 2048 cells");
        }
    }
    if (n == "strata_rope") {
        if (!int_in(I("rotary")) || !int_in(I("dim")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.rotary and dim must be integers in [1, 2147483647]", name);
        if (I("rotary") % 2 || I("rotary") > I("dim")) return fail(ctx, STRATA_ERR_RANGE, "Rotary width must be even and <= head dimension");
    }
    if (n == "strata_norm") {
        if (!int_in(I("rows")) || !int_in(I("weightRows")))
            return fail(ctx, STRATA_ERR_RANGE, "%s.rows and weightRows must be integers in [1, 2147483647]", name);
        if (I("rows") % I("weightRows")) return fail(ctx, STRATA_ERR_RANGE, "Normalization weight rows must divide input rows");
    }
    // Beyond the reference: parameters that these entries divide by must be positive. The
    // reference does not check them; its CPU build traps on an integer division by zero.
    static const struct {
        const char *entry, *params;
    } kDivisors[] = {
        {"strata_embed", "width"},           {"strata_embed_batch", "width streams"}, {"strata_hc_mix_batch", "width"},
        {"strata_hc_write", "width"},        {"strata_hc_write_batch", "width streams"},
        {"strata_ple_broadcast", "width"},   {"strata_ple_broadcast_batch", "width streams"},
        {"strata_slice", "width"},           {"strata_rope_batch", "dim rotary"},  {"strata_rope_table", "rotary"},
        {"strata_attention_gate", "dim"},    {"strata_attention_gate_batch", "dim"}, {"strata_gdn_gates_batch", "heads"},
        {"strata_gdn_step", "dim keyHeads valueHeads"}, {"strata_gdn_batch", "dim keyHeads valueHeads"},
    };
    for (const auto &d : kDivisors) {
        if (n != d.entry) continue;
        std::string list(d.params), p;
        for (size_t at = 0; at <= list.size(); ++at) {
            if (at < list.size() && list[at] != ' ') {
                p += list[at];
                continue;
            }
            if (p.empty()) continue;
            const long long v = I(p.c_str());
            if (!int_in(v) || (p == "rotary" && v < 2))
                return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [%d, 2147483647]", name, p.c_str(), p == "rotary" ? 2 : 1);
            p.clear();
        }
    }
    // Beyond the reference: every loop extent must fit the buffer it walks, so a malformed
    // dispatch is rejected instead of spinning over skipped out-of-range reads.
    auto fits = [&](long long need, const char *buf) { return need >= 0 && need <= len(buf); };
    bool ok = true;
    if (n == "strata_conv" || n == "strata_conv_batch") {
        const long long c = I("channels"), taps = I("taps"), dil = I("dilation"), t = n == "strata_conv" ? 1 : I("tokens");
        ok = int_in(c) && int_in(taps) && int_in(dil) && int_in(t) && fits(c * (taps - 1) * dil, "History") && fits(c * taps, "W") &&
             fits(t * c, "X") && fits(t * c, "Y");
    } else if (n == "strata_gdn_step" || n == "strata_gdn_batch") {
        const long long d = I("dim"), vh = I("valueHeads"), kh = I("keyHeads"), t = n == "strata_gdn_step" ? 1 : I("tokens");
        ok = int_in(d) && int_in(vh) && int_in(kh) && int_in(t) && fits(d * vh * d, "State") && fits(t * kh * d, "Q") &&
             fits(t * kh * d, "K") && fits(t * vh * d, "V") && fits(t * vh * d, "Y");
    } else if (n == "strata_norm") {
        ok = int_in(I("cols")) && fits(I("rows") * I("cols"), "X") && fits(I("rows") * I("cols"), "Y");
    } else if (n == "strata_gemv") {
        ok = int_in(I("cols")) && int_in(I("rows")) && int_in(I("tokens")) && fits(I("rows") * I("cols"), "W") &&
             fits(I("tokens") * I("cols"), "X");
    } else if (n == "strata_quant_gemv") {
        ok = fits(I("cols"), "X");
    } else if (n == "strata_ple_gate") {
        ok = int_in(I("width")) && int_in(I("streams")) && fits(I("streams") * I("width"), "Key") &&
             fits(I("streams") * I("width"), "Query");
    } else if (n == "strata_argmax") {
        ok = int_in(I("count")) && fits(I("count"), "Logits");
    } else if (n == "strata_attention") {
        ok = fits(I("heads") * I("dim"), "Q") && fits(I("count"), "Cells");
    } else if (n == "strata_hc_mix" || n == "strata_hc_mix_batch") {
        ok = int_in(I("width")) && int_in(I("streams")) &&
             fits((n == "strata_hc_mix" ? 1 : I("tokens")) * I("streams") * I("width"), "Norm");
    } else if (n == "strata_embed_token") {
        ok = int_in(I("width")) && int_in(I("streams")) && int_in(I("vocab")) && int_in(I("tokens")) &&
             fits(I("tokens") * I("width") * I("streams"), "Residual") && fits(I("vocab") * I("width"), "Table") && fits(I("tokens"), "Token");
    } else if (n == "strata_rope_at") {
        for (const char *p : {"rotary", "dim", "heads", "tokens"})
            if (!int_in(I(p))) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p);
        if (I("rotary") % 2 || I("rotary") > I("dim") || len("X") != I("dim") * I("heads") * I("tokens") || len("Y") != len("X"))
            return fail(ctx, STRATA_ERR_LAYOUT, "Invalid RoPE layout");
        ok = fits(1, "Position");
    } else if (n == "strata_kv_append_at") {
        ok = int_in(I("width")) && int_in(I("tokens")) && fits(1, "Position");
    } else if (n == "strata_attention_at") {
        for (const char *p : {"heads", "kvHeads", "dim"})
            if (!int_in(I(p))) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p);
        if (I("heads") % I("kvHeads")) return fail(ctx, STRATA_ERR_RANGE, "Attention heads must be divisible by KV heads");
        ok = fits(I("heads") * I("dim"), "Q") && fits(1, "Position");
    }
    // Sequence-batch decode entries: one token per sequence, each sequence with its own position,
    // cache, history or state; every per-sequence region must lie inside its buffer.
    if (n == "strata_rope_seqs" || n == "strata_kv_append_seqs" || n == "strata_attention_seqs" || n == "strata_conv_seqs" ||
        n == "strata_gdn_seqs" || n == "strata_argmax_rows") {
        static const struct {
            const char *entry, *params;
        } kPositive[] = {
            {"strata_rope_seqs", "dim heads rotary tokens"},     {"strata_kv_append_seqs", "width cells tokens"},
            {"strata_attention_seqs", "dim heads kvHeads cells"}, {"strata_conv_seqs", "channels taps dilation tokens"},
            {"strata_gdn_seqs", "dim keyHeads valueHeads tokens"}, {"strata_argmax_rows", "count rows"},
        };
        for (const auto &d : kPositive) {
            if (n != d.entry) continue;
            std::string list(d.params), p;
            for (size_t at = 0; at <= list.size(); ++at) {
                if (at < list.size() && list[at] != ' ') {
                    p += list[at];
                    continue;
                }
                if (!p.empty() && !int_in(I(p.c_str())))
                    return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer in [1, 2147483647]", name, p.c_str());
                p.clear();
            }
        }
        if (n == "strata_rope_seqs") {
            if (I("rotary") % 2 || I("rotary") > I("dim") || len("X") != I("dim") * I("heads") * I("tokens") || len("Y") != len("X"))
                return fail(ctx, STRATA_ERR_LAYOUT, "Invalid RoPE layout");
            ok = fits(I("tokens"), "Positions");
        } else if (n == "strata_kv_append_seqs") {
            const long long t = I("tokens"), w = I("width"), cache = t * I("cells") * w;
            ok = fits(t * w, "K") && fits(t * w, "V") && fits(cache, "Keys") && fits(cache, "Values") && fits(t, "Positions");
        } else if (n == "strata_attention_seqs") {
            if (I("heads") % I("kvHeads")) return fail(ctx, STRATA_ERR_RANGE, "Attention heads must be divisible by KV heads");
            if (I("cells") > 2048) return fail(ctx, STRATA_ERR_RANGE, "attention cells must be an integer in [1, 2048]");
            const long long t = groups[2], cache = t * I("cells") * I("kvHeads") * I("dim");
            ok = fits(t * I("heads") * I("dim"), "Q") && fits(t * I("heads") * I("dim"), "Y") && fits(cache, "Keys") &&
                 fits(cache, "Values") && fits(t, "Positions");
        } else if (n == "strata_conv_seqs") {
            const long long c = I("channels"), t = I("tokens");
            ok = fits(t * c * (I("taps") - 1) * I("dilation"), "History") && fits(c * I("taps"), "W") && fits(t * c, "X") &&
                 fits(t * c, "Y");
        } else if (n == "strata_gdn_seqs") {
            const long long d = I("dim"), vh = I("valueHeads"), kh = I("keyHeads"), t = I("tokens");
            ok = fits(t * d * vh * d, "State") && fits(t * kh * d, "Q") && fits(t * kh * d, "K") && fits(t * vh * d, "V") &&
                 fits(t * vh * d, "Y") && fits(t * vh, "Decay") && fits(t * vh, "Beta");
        } else {
            ok = fits(I("rows") * I("count"), "Logits") && fits(I("rows"), "Tokens");
        }
    }
    if (n == "strata_hc_in" || n == "strata_hc_out") {  // every index the kernels read or write lies inside its buffer
        const long long w = I("width"), st = I("streams"), r = I("rank"), hc = w * st;
        if (!int_in(w) || !int_in(st, 1, 64) || !int_in(r))
            return fail(ctx, STRATA_ERR_RANGE, "%s: width, rank >= 1 and streams in [1, 64] required", name);
        if (n == "strata_hc_in")
            ok = hc * 8 <= 200 * 1024 && fits(hc, "Residual") && fits(hc, "NormW") && fits(r * hc, "DownW") && fits(st * hc, "InjectW") &&
                 fits(hc, "Norm") && fits(r, "Down") && fits(st, "Inject");
        else
            ok = r * 4 <= 48 * 1024 && fits(hc, "Norm") && fits(r, "Down") && fits(hc * r, "UpW") && fits(w, "Mixed");
    }
    if (!ok) return fail(ctx, STRATA_ERR_LAYOUT, "%s: a loop extent exceeds its buffer layout", name);
    return STRATA_OK;
}

bool blob_geometry_ok(int width, int ff) { return width > 0 && ff > 0 && width % 64 == 0 && ff % 64 == 0; }
long long blob_words_of(int width, int ff) { return 3LL * ff * width / 16 + 3LL * ff * width / 128; }

}  // namespace

extern "C" {

int strata_create(int device, strata_ctx **out) {
    if (!out) return STRATA_ERR_RANGE;
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) return STRATA_ERR_CUDA;
    if (device < 0 || device >= count) return STRATA_ERR_RANGE;
    auto *ctx = new strata_ctx();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->err_dev, sizeof(unsigned)) != cudaSuccess ||
        cudaHostAlloc(&ctx->err_host, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess ||
        cudaMemset(ctx->err_dev, 0, sizeof(unsigned)) != cudaSuccess || cudaMalloc(&ctx->fast_sync, kFastSyncWords * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(ctx->fast_sync, 0, kFastSyncWords * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&ctx->decode1_xchg, moe_decode1_xchg_bytes()) != cudaSuccess ||
        cudaMemset(ctx->decode1_xchg, 0, moe_decode1_xchg_bytes()) != cudaSuccess) {
        strata_destroy(ctx);
        return STRATA_ERR_CUDA;
    }
    *ctx->err_host = 0;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) {
        snprintf(ctx->device_name, sizeof ctx->device_name, "%s", prop.name);
        ctx->sms = prop.multiProcessorCount;
    }
    *out = ctx;
    return STRATA_OK;
}

int strata_destroy(strata_ctx *ctx) {
    if (!ctx) return STRATA_OK;
    cudaSetDevice(ctx->device);
    if (ctx->ep && ctx->stream) {  // a peer that is gone must not hang the teardown: bounded wait, abort on failure
        std::string msg;
        ep_wait(ctx->ep, ctx->stream, &msg);
    }
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (auto &kv : ctx->buffers) cudaFree(kv.second.ptr);
    ctx->buffers.clear();
    if (ctx->workspace) cudaFree(ctx->workspace);
    for (const auto &m : ctx->marks) {
        ctx->spare_events.push_back(m.a);
        ctx->spare_events.push_back(m.b);
    }
    std::sort(ctx->spare_events.begin(), ctx->spare_events.end());
    ctx->spare_events.erase(std::unique(ctx->spare_events.begin(), ctx->spare_events.end()), ctx->spare_events.end());
    for (cudaEvent_t e : ctx->spare_events) cudaEventDestroy(e);
    if (ctx->ep) ep_destroy(ctx->ep);
    for (auto &kv : ctx->graphs) {
        cudaGraphExecDestroy(kv.second.exec);
        cudaGraphDestroy(kv.second.g);
    }
    ctx->graphs.clear();
    if (ctx->err_dev) cudaFree(ctx->err_dev);
    if (ctx->fast_sync) cudaFree(ctx->fast_sync);
    if (ctx->check_dev) cudaFree(ctx->check_dev);
    if (ctx->decode1_xchg) cudaFree(ctx->decode1_xchg);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return STRATA_OK;
}

int strata_last_error(strata_ctx *ctx, char *buf, size_t cap) {
    if (!ctx) return 0;
    if (buf && cap) snprintf(buf, cap, "%s", ctx->last_error.c_str());
    return (int)ctx->last_error.size();
}

int strata_stream(strata_ctx *ctx, void **stream) {
    if (!ctx || !stream) return STRATA_ERR_RANGE;
    *stream = (void *)ctx->stream;
    return STRATA_OK;
}

int strata_alloc(strata_ctx *ctx, uint64_t length, int type, int zero, strata_buf *out) {
    if (!ctx || !out) return STRATA_ERR_RANGE;
    if (type != STRATA_F32 && type != STRATA_I32 && type != STRATA_U32) return fail(ctx, STRATA_ERR_RANGE, "Unsupported buffer type %d", type);
    if (length < 1 || length > (1ull << 40)) return fail(ctx, STRATA_ERR_RANGE, "allocation must be an integer in [1, 2^40] elements");
    if (int r = use_device(ctx)) return r;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, length * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, STRATA_ERR_ALLOC, "device allocation of %llu bytes failed: %s", (unsigned long long)(length * 4),
                    cudaGetErrorString(e));
    }
    if (zero) CUDA_OR_FAIL(ctx, cudaMemsetAsync(p, 0, length * 4, ctx->stream), "cudaMemsetAsync");
    uint64_t h = ctx->next_handle++;
    ctx->buffers[h] = Buffer{p, length, type};
    ctx->bytes_resident += length * 4;
    *out = h;
    return STRATA_OK;
}

int strata_free(strata_ctx *ctx, strata_buf buf) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return STRATA_OK;  // src/backend.js:115 ignores unknown buffers
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "buffers cannot be freed while the stream is captured");
    if (int r = use_device(ctx)) return r;
    cudaStreamSynchronize(ctx->stream);  // work that still reads the buffer completes first
    cudaFree(b->ptr);
    ctx->bytes_resident -= b->length * 4;
    ctx->buffers.erase(buf);
    return STRATA_OK;
}

int strata_write(strata_ctx *ctx, strata_buf buf, const void *data, uint64_t count, uint64_t offset) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "Invalid write: unknown buffer");
    if (offset + count > b->length || offset + count < offset) return fail(ctx, STRATA_ERR_LAYOUT, "Invalid write: exceeds buffer");
    if (!count) return STRATA_OK;
    if (!data) return fail(ctx, STRATA_ERR_RANGE, "Invalid write: null data");
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "host writes are not allowed while the stream is captured");
    if (int r = use_device(ctx)) return r;
    // Pageable memory is staged before this returns; page-locked memory is read later by the
    // stream and must stay unchanged until the next synchronising call.
    CUDA_OR_FAIL(ctx, cudaMemcpyAsync((char *)b->ptr + offset * 4, data, count * 4, cudaMemcpyHostToDevice, ctx->stream),
                 "host-to-device copy");
    return STRATA_OK;
}

int strata_read(strata_ctx *ctx, strata_buf buf, void *out, uint64_t count, uint64_t offset) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "Invalid read: unknown buffer");
    if (offset + count > b->length || offset + count < offset) return fail(ctx, STRATA_ERR_LAYOUT, "Invalid read: exceeds buffer");
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "reads are not allowed while the stream is captured");
    if (int r = use_device(ctx)) return r;
    if (count) {
        if (!out) return fail(ctx, STRATA_ERR_RANGE, "Invalid read: null destination");
        CUDA_OR_FAIL(ctx, cudaMemcpyAsync(out, (const char *)b->ptr + offset * 4, count * 4, cudaMemcpyDeviceToHost, ctx->stream),
                     "device-to-host copy");
    }
    return sync(ctx);
}

int strata_copy(strata_ctx *ctx, strata_buf src, strata_buf dst, uint64_t count, uint64_t src_offset, uint64_t dst_offset) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *a = find(ctx, src), *b = find(ctx, dst);
    if (!a || !b) return fail(ctx, STRATA_ERR_HANDLE, "Invalid copy: unknown buffer");
    if (count + src_offset > a->length || count + dst_offset > b->length) return fail(ctx, STRATA_ERR_LAYOUT, "Invalid copy: exceeds buffer");
    if (!count) return STRATA_OK;
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaMemcpyAsync((char *)b->ptr + dst_offset * 4, (const char *)a->ptr + src_offset * 4, count * 4,
                                      cudaMemcpyDeviceToDevice, ctx->stream),
                 "device copy");
    return STRATA_OK;
}

int strata_zero(strata_ctx *ctx, strata_buf buf) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "Invalid zero: unknown buffer");
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaMemsetAsync(b->ptr, 0, b->length * 4, ctx->stream), "cudaMemsetAsync");
    return STRATA_OK;
}

int strata_buffer_info(strata_ctx *ctx, strata_buf buf, uint64_t *length, int *type, void **device_ptr) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "unknown buffer");
    if (length) *length = b->length;
    if (type) *type = b->type;
    if (device_ptr) *device_ptr = b->ptr;
    return STRATA_OK;
}

int strata_run(strata_ctx *ctx, const char *name, const strata_arg *args, int nargs, const uint32_t groups[3]) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!name) return fail(ctx, STRATA_ERR_UNKNOWN, "Unknown kernel (null)");
    const Entry *entry = nullptr;
    for (const Entry &e : entries())
        if (!strcmp(e.spec->name, name)) entry = &e;
    if (!entry) return fail(ctx, STRATA_ERR_UNKNOWN, "Unknown kernel %s", name);
    // vendor/webcuda/src/wasm/runtime.js:11: three positive integers, at most 1e8 workgroups.
    if (!groups || !groups[0] || !groups[1] || !groups[2] || (double)groups[0] * groups[1] * groups[2] > 1e8)
        return fail(ctx, STRATA_ERR_RANGE, "Invalid dispatch size");
    std::vector<KArg> vals(entry->params.size());
    for (size_t i = 0; i < entry->params.size(); ++i) {
        const Param &p = entry->params[i];
        const strata_arg *found = nullptr;
        for (int j = 0; j < nargs; ++j)
            if (args[j].name && p.name == args[j].name) found = &args[j];
        if (!found) return fail(ctx, STRATA_ERR_UNKNOWN, "Missing %s.%s", name, p.name.c_str());
        KArg v{nullptr, 0, 0, 0.0f};
        if (p.kind == 'f' || p.kind == 'u' || p.kind == 'i') {
            if (found->kind != STRATA_ARG_BUF) return fail(ctx, STRATA_ERR_LAYOUT, "%s.%s must be a buffer", name, p.name.c_str());
            Buffer *b = find(ctx, found->buf);
            if (!b) return fail(ctx, STRATA_ERR_HANDLE, "%s.%s is not a live buffer", name, p.name.c_str());
            v.ptr = b->ptr;
            v.len = (long long)b->length;
        } else if (p.kind == 'I') {
            if (found->kind != STRATA_ARG_I32) return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be an integer", name, p.name.c_str());
            v.i = found->i32;
        } else {
            if (found->kind == STRATA_ARG_F32) v.f = found->f32;
            else if (found->kind == STRATA_ARG_I32) v.f = (float)found->i32;
            else return fail(ctx, STRATA_ERR_RANGE, "%s.%s must be a number", name, p.name.c_str());
        }
        vals[i] = v;
    }
    if (int r = validate(ctx, name, entry->params, vals, groups)) return r;
    if (int r = use_device(ctx)) return r;
    const unsigned g[3] = {groups[0], groups[1], groups[2]};
    cudaError_t e = entry->spec->launch(vals.data(), g, ctx->stream, ctx->err_dev);
    if (e != cudaSuccess) return cuda_fail(ctx, e, name);
    ++ctx->dispatches;
    return STRATA_OK;
}

int strata_idle(strata_ctx *ctx) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (int r = use_device(ctx)) return r;
    return sync(ctx);
}

int strata_flush(strata_ctx *ctx) { return ctx ? STRATA_OK : STRATA_ERR_RANGE; }

int strata_info(strata_ctx *ctx, char *json, size_t cap) {
    if (!ctx) return STRATA_ERR_RANGE;
    char buf[1024];
    int n = snprintf(buf, sizeof buf,
                     "{\"backend\":\"cuda\",\"device\":\"%s\",\"ordinal\":%d,\"sms\":%d,\"buffers\":%zu,\"bytesResident\":%llu,"
                     "\"workspaceBytes\":%zu,\"dispatches\":%llu,\"fusedCalls\":%llu,\"fastPdl\":%d}",
                     ctx->device_name, ctx->device, ctx->sms, ctx->buffers.size(), (unsigned long long)ctx->bytes_resident,
                     ctx->workspace_bytes, (unsigned long long)ctx->dispatches, (unsigned long long)ctx->fused_calls, moe_fast_pdl_state());
    if (json && cap) snprintf(json, cap, "%s", buf);
    return n;
}

int strata_ple_gather_decode(strata_ctx *ctx, strata_buf table, strata_buf ids, int32_t rows, int32_t head_dim, strata_buf values) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (rows < 1) return fail(ctx, STRATA_ERR_RANGE, "rows must be an integer >= 1");
    if (head_dim < 32 || head_dim % 32) return fail(ctx, STRATA_ERR_LAYOUT, "Invalid packed PLE layout");
    Buffer *t = find(ctx, table), *d = find(ctx, ids), *v = find(ctx, values);
    if (!t || !d || !v) return fail(ctx, STRATA_ERR_HANDLE, "strata_ple_gather_decode: unknown buffer");
    if ((long long)d->length < rows || (long long)v->length < (long long)rows * head_dim)
        return fail(ctx, STRATA_ERR_LAYOUT, "Invalid packed PLE layout");
    if (int r = use_device(ctx)) return r;
    cudaError_t e = ple_gather_decode((const unsigned *)t->ptr, (long long)t->length, (const int *)d->ptr, (long long)d->length, rows, head_dim,
                                      (float *)v->ptr, (long long)v->length, ctx->stream, ctx->err_dev);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "strata_ple_gather_decode");
    return STRATA_OK;
}

int strata_capture_begin(strata_ctx *ctx) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "the stream is already being captured");
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    ctx->capturing = true;
    return STRATA_OK;
}

int strata_capture_end(strata_ctx *ctx, uint64_t *graph) {
    if (!ctx || !graph) return STRATA_ERR_RANGE;
    if (!ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "the stream is not being captured");
    if (int r = use_device(ctx)) return r;
    ctx->capturing = false;
    cudaGraph_t g = nullptr;
    CUDA_OR_FAIL(ctx, cudaStreamEndCapture(ctx->stream, &g), "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
    if (e == cudaSuccess) e = cudaGraphUpload(exec, ctx->stream);  // the first replay needs no upload
    if (e != cudaSuccess) {
        if (exec) cudaGraphExecDestroy(exec);
        cudaGraphDestroy(g);
        return cuda_fail(ctx, e, "cudaGraphInstantiate");
    }
    const uint64_t h = ctx->next_graph++;
    ctx->graphs[h] = {g, exec};
    *graph = h;
    return STRATA_OK;
}

int strata_graph_launch(strata_ctx *ctx, uint64_t graph) {
    if (!ctx) return STRATA_ERR_RANGE;
    auto it = ctx->graphs.find(graph);
    if (it == ctx->graphs.end()) return fail(ctx, STRATA_ERR_HANDLE, "graph %llu is not live", (unsigned long long)graph);
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaGraphLaunch(it->second.exec, ctx->stream), "cudaGraphLaunch");
    return STRATA_OK;
}

int strata_graph_free(strata_ctx *ctx, uint64_t graph) {
    if (!ctx) return STRATA_ERR_RANGE;
    auto it = ctx->graphs.find(graph);
    if (it == ctx->graphs.end()) return fail(ctx, STRATA_ERR_HANDLE, "graph %llu is not live", (unsigned long long)graph);
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    cudaGraphExecDestroy(it->second.exec);
    cudaGraphDestroy(it->second.g);
    ctx->graphs.erase(it);
    return STRATA_OK;
}

int strata_profile(strata_ctx *ctx, int32_t enable) {
    if (!ctx) return STRATA_ERR_RANGE;
    ctx->profile = enable != 0;
    return STRATA_OK;
}

int strata_profile_read(strata_ctx *ctx, double *ms, int32_t n, uint64_t *calls) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (int r = use_device(ctx)) return r;
    CUDA_OR_FAIL(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    for (int i = 0; i < n && ms; ++i) ms[i] = 0.0;
    std::vector<cudaEvent_t> seen;
    for (const auto &m : ctx->marks) {
        float t = 0.0f;
        CUDA_OR_FAIL(ctx, cudaEventElapsedTime(&t, m.a, m.b), "cudaEventElapsedTime");
        if (ms && m.phase < n) ms[m.phase] += t;
        seen.push_back(m.a);
        seen.push_back(m.b);
    }
    std::sort(seen.begin(), seen.end());
    seen.erase(std::unique(seen.begin(), seen.end()), seen.end());
    for (cudaEvent_t e : seen) ctx->spare_events.push_back(e);
    ctx->marks.clear();
    if (calls) *calls = ctx->profiled_calls;
    ctx->profiled_calls = 0;
    return STRATA_OK;
}

int strata_ep_unique_id(strata_ctx *ctx, uint8_t *id, size_t cap) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!id || cap < STRATA_EP_ID_BYTES) return fail(ctx, STRATA_ERR_RANGE, "unique id buffer needs %d bytes", STRATA_EP_ID_BYTES);
    std::string err;
    if (ep_unique_id(reinterpret_cast<char *>(id), &err)) return fail(ctx, STRATA_ERR_CUDA, "%s", err.c_str());
    return STRATA_OK;
}

int strata_ep_init(strata_ctx *ctx, int32_t rank, int32_t n_ranks, const uint8_t *id) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!id || n_ranks < 1 || rank < 0 || rank >= n_ranks) return fail(ctx, STRATA_ERR_RANGE, "invalid rank %d of %d", rank, n_ranks);
    if (int r = use_device(ctx)) return r;
    if (ctx->ep) {
        ep_destroy(ctx->ep);
        ctx->ep = nullptr;
    }
    std::string err;
    ctx->ep = ep_create(rank, n_ranks, reinterpret_cast<const char *>(id), ctx->ep_timeout_ms, &err);
    if (!ctx->ep) return fail(ctx, STRATA_ERR_CUDA, "%s", err.c_str());
    return STRATA_OK;
}

int strata_ep_loopback_create(strata_ctx *ctx, int32_t n_ranks, uint64_t *hub) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!hub) return fail(ctx, STRATA_ERR_RANGE, "null hub");
    std::string err;
    unsigned long long h = 0;
    if (ep_loopback_hub_create(n_ranks, &h, &err)) return fail(ctx, STRATA_ERR_RANGE, "%s", err.c_str());
    *hub = h;
    return STRATA_OK;
}

int strata_ep_loopback_release(strata_ctx *ctx, uint64_t hub) {
    if (!ctx) return STRATA_ERR_RANGE;
    std::string err;
    if (ep_loopback_hub_release(hub, &err)) return fail(ctx, STRATA_ERR_HANDLE, "%s", err.c_str());
    return STRATA_OK;
}

int strata_ep_init_loopback(strata_ctx *ctx, int32_t rank, uint64_t hub) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (int r = use_device(ctx)) return r;
    if (ctx->ep) {
        ep_destroy(ctx->ep);
        ctx->ep = nullptr;
    }
    std::string err;
    ctx->ep = ep_create_loopback(hub, rank, ctx->ep_timeout_ms, &err);
    if (!ctx->ep) return fail(ctx, STRATA_ERR_RANGE, "%s", err.c_str());
    return STRATA_OK;
}

int strata_ep_set_timeout(strata_ctx *ctx, int32_t milliseconds) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (milliseconds < 1) return fail(ctx, STRATA_ERR_RANGE, "timeout must be >= 1 ms");
    ctx->ep_timeout_ms = milliseconds;
    if (ctx->ep) ctx->ep->t->timeout_ms = milliseconds;
    return STRATA_OK;
}

namespace {
// Expert placement of the context's communicator: owner[e] (nullptr: contiguous, experts / n
// per rank); every rank must own at least one expert. Synchronises.
int set_placement(strata_ctx *ctx, int experts, const int32_t *owner) {
    EpComm &c = *ctx->ep;
    const int n = c.n;
    if (experts < 1 || experts > 512) return fail(ctx, STRATA_ERR_RANGE, "placement: experts must be 1 .. 512");
    if (!owner && experts % n) return fail(ctx, STRATA_ERR_RANGE, "experts must be a multiple of the %d ranks", n);
    std::vector<int> h(2 * (size_t)experts), cnt(n, 0);
    for (int e = 0; e < experts; ++e) {
        const int o = owner ? owner[e] : e / (experts / n);
        if (o < 0 || o >= n) return fail(ctx, STRATA_ERR_RANGE, "placement: expert %d on rank %d, outside 0 .. %d", e, o, n - 1);
        h[e] = o;
        h[experts + e] = cnt[o]++;
    }
    for (int r = 0; r < n; ++r)
        if (!cnt[r]) return fail(ctx, STRATA_ERR_RANGE, "placement: rank %d owns no expert", r);
    if (int r = use_device(ctx)) return r;
    const size_t bytes = sizeof(int) * h.size();
    if (c.place_cap < bytes) {
        if (c.d_place) cudaFree(c.d_place);
        c.d_place = nullptr;
        c.place_cap = 0;
        CUDA_OR_FAIL(ctx, cudaMalloc(&c.d_place, bytes), "cudaMalloc");
        c.place_cap = bytes;
    }
    CUDA_OR_FAIL(ctx, cudaMemcpy(c.d_place, h.data(), bytes, cudaMemcpyHostToDevice), "cudaMemcpy");
    c.placed_experts = experts;
    c.n_local = cnt[c.rank];
    return STRATA_OK;
}
}  // namespace

int strata_ep_set_placement(strata_ctx *ctx, int32_t experts, const int32_t *owner) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!ctx->ep) return fail(ctx, STRATA_ERR_RANGE, "strata_ep_init has not been called");
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "synchronising calls are not allowed while the stream is captured");
    return set_placement(ctx, experts, owner);
}

int strata_ep_local_experts(strata_ctx *ctx, int32_t experts, int32_t *count) {
    if (!ctx || !count) return STRATA_ERR_RANGE;
    if (!ctx->ep) return fail(ctx, STRATA_ERR_RANGE, "strata_ep_init has not been called");
    if (ctx->ep->placed_experts != experts) {
        if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "synchronising calls are not allowed while the stream is captured");
        if (int r = set_placement(ctx, experts, nullptr)) return r;
    }
    *count = ctx->ep->n_local;
    return STRATA_OK;
}

int strata_moe_ep_forward(strata_ctx *ctx, const strata_moe_layer *layer, strata_buf x, int32_t tokens, strata_buf y, strata_buf ids,
                          strata_buf weights) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!ctx->ep) return fail(ctx, STRATA_ERR_RANGE, "strata_ep_init has not been called");
    if (!layer) return fail(ctx, STRATA_ERR_RANGE, "null layer");
    const strata_moe_layer &l = *layer;
    if (!moe_prefill_supported(l.width, l.ff, l.experts, l.top_k))
        return fail(ctx, STRATA_ERR_RANGE, "expert-parallel layer supports H 2048/F 512 and H 2560/F 640, <= 512 experts, topK <= 32");
    if (l.top_k < 1 || l.top_k > l.experts) return fail(ctx, STRATA_ERR_RANGE, "topK must be 1 .. experts");
    if (tokens < 1) return fail(ctx, STRATA_ERR_RANGE, "tokens must be an integer >= 1");
    if (ctx->ep->placed_experts != l.experts) {  // no placement for this expert count: contiguous
        if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "synchronising calls are not allowed while the stream is captured");
        if (int r = set_placement(ctx, l.experts, nullptr)) return r;
    }
    const long long bw = blob_words_of(l.width, l.ff);
    struct Need {
        strata_buf h;
        long long n;
        const char *what;
        bool optional;
    } need[] = {{l.router, (long long)l.experts * l.width, "router", false},
                {l.router_bias, l.experts, "router_bias", true},
                {l.experts_blob, bw * ctx->ep->n_local, "experts_blob (this rank's experts)", false},
                {l.shared_blob, bw, "shared_blob", false},
                {l.shared_gate, l.width, "shared_gate", false},
                {x, (long long)tokens * l.width, "x", false},
                {y, (long long)tokens * l.width, "y", false},
                {ids, (long long)tokens * l.top_k, "ids", false},
                {weights, (long long)tokens * l.top_k, "weights", false}};
    void *ptr[9];
    for (int i = 0; i < 9; ++i) {
        ptr[i] = nullptr;
        if (need[i].optional && need[i].h == 0) continue;
        Buffer *b = find(ctx, need[i].h);
        if (!b) return fail(ctx, STRATA_ERR_HANDLE, "ep layer: %s is not a live buffer", need[i].what);
        if ((long long)b->length < need[i].n)
            return fail(ctx, STRATA_ERR_LAYOUT, "ep layer: %s holds %llu elements, needs %lld", need[i].what, (unsigned long long)b->length,
                        need[i].n);
        ptr[i] = b->ptr;
    }
    if (int r = use_device(ctx)) return r;
    MoeLayerDev L{l.width, l.ff, l.experts, l.top_k, (const float *)ptr[0], (const float *)ptr[1], (const unsigned *)ptr[2], bw,
                  (const unsigned *)ptr[3], (const float *)ptr[4]};
    // profile: boundaries start | packed | GEMMs start | gate/up done | down done | combined
    cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    if (ctx->profile) {
        for (cudaEvent_t &e : ev) {
            if (!ctx->spare_events.empty()) {
                e = ctx->spare_events.back();
                ctx->spare_events.pop_back();
            } else {
                CUDA_OR_FAIL(ctx, cudaEventCreate(&e), "cudaEventCreate");
            }
        }
        ++ctx->profiled_calls;
    }
    std::string msg;
    const int rc = moe_forward_ep(L, ctx->ep, (const float *)ptr[5], tokens, (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], ctx->sms,
                                  ctx->stream, ctx->err_dev, &msg, ev[0] ? ev : nullptr);
    if (ev[0]) {
        if (rc) {
            for (cudaEvent_t e : ev) ctx->spare_events.push_back(e);
            --ctx->profiled_calls;
        } else {
            ctx->marks.push_back({0, ev[0], ev[1]});
            ctx->marks.push_back({4, ev[1], ev[2]});
            ctx->marks.push_back({1, ev[2], ev[3]});
            ctx->marks.push_back({2, ev[3], ev[4]});
            ctx->marks.push_back({5, ev[4], ev[5]});
        }
    }
    if (rc) return fail(ctx, STRATA_ERR_CUDA, "strata_moe_ep_forward: %s", msg.c_str());
    ++ctx->fused_calls;
    return STRATA_OK;
}

int strata_validate_experts(strata_ctx *ctx, strata_buf blobs, int32_t count, int32_t width, int32_t ff) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!blob_geometry_ok(width, ff)) return fail(ctx, STRATA_ERR_LAYOUT, "Packed expert dimensions must contain complete groups");
    if (count < 1) return fail(ctx, STRATA_ERR_RANGE, "count must be an integer >= 1");
    Buffer *b = find(ctx, blobs);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "validate experts: not a live buffer");
    const long long bw = blob_words_of(width, ff);
    if ((long long)b->length < bw * count)
        return fail(ctx, STRATA_ERR_LAYOUT, "validate experts: the buffer holds %llu words, %d blobs need %lld", (unsigned long long)b->length,
                    count, bw * count);
    if (ctx->capturing) return fail(ctx, STRATA_ERR_RANGE, "synchronising calls are not allowed while the stream is captured");
    if (int r = use_device(ctx)) return r;
    if (!ctx->check_dev) CUDA_OR_FAIL(ctx, cudaMalloc(&ctx->check_dev, sizeof(int)), "cudaMalloc");
    CUDA_OR_FAIL(ctx, check_expert_scales((const unsigned *)b->ptr, count, width, ff, ctx->check_dev, ctx->stream), "scale check");
    int first_bad = 0;
    CUDA_OR_FAIL(ctx, cudaMemcpyAsync(&first_bad, ctx->check_dev, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream), "readback");
    if (int r = sync(ctx)) return r;
    if (first_bad != 0x7f7f7f7f) return fail(ctx, STRATA_ERR_LAYOUT, "Non-finite expert scales (blob %d)", first_bad);
    return STRATA_OK;
}

int strata_moe_forward(strata_ctx *ctx, const strata_moe_layer *layer, strata_buf x, int32_t tokens, strata_buf y, strata_buf ids,
                       strata_buf weights, int32_t mode) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!layer) return fail(ctx, STRATA_ERR_RANGE, "null layer");
    const strata_moe_layer &l = *layer;
    if (!blob_geometry_ok(l.width, l.ff)) return fail(ctx, STRATA_ERR_LAYOUT, "Packed expert dimensions must contain complete groups");
    if (l.experts < 1 || l.experts > 512 || l.top_k < 1 || l.top_k > std::min(l.experts, 32))
        return fail(ctx, STRATA_ERR_RANGE, "Router supports 1-512 experts and topK <= min(experts,32)");
    if (tokens < 1) return fail(ctx, STRATA_ERR_RANGE, "tokens must be an integer >= 1");
    if (mode != STRATA_MOE_EXACT && mode != STRATA_MOE_FAST) return fail(ctx, STRATA_ERR_RANGE, "unknown mode %d", mode);
    // FAST: the fused decode kernel up to 8 tokens, the medium-batch layer up to 64, the
    // tensor-core prefill path above
    const bool fast = mode == STRATA_MOE_FAST && moe_fast_supported(tokens, l.width, l.ff, l.top_k, ctx->sms);
    // one token: the one-arrival layer (STRATA_DECODE1=0 keeps the batch decode kernel, for comparisons)
    static const bool decode1_on = [] {
        const char *v = std::getenv("STRATA_DECODE1");
        return !(v && v[0] == '0');
    }();
    const bool decode1 = fast && decode1_on && moe_decode1_supported(tokens, l.width, l.ff, l.experts, l.top_k, ctx->sms);
    const bool medium = mode == STRATA_MOE_FAST && !fast && moe_medium_supported(tokens, l.width, l.ff, l.experts, l.top_k, ctx->sms);
    const bool prefill = mode == STRATA_MOE_FAST && !fast && !medium && moe_prefill_supported(l.width, l.ff, l.experts, l.top_k);
    const long long bw = blob_words_of(l.width, l.ff);
    struct Need {
        strata_buf h;
        long long n;
        const char *what;
        bool optional;
    } need[] = {{l.router, (long long)l.experts * l.width, "router", false},
                {l.router_bias, l.experts, "router_bias", true},
                {l.experts_blob, bw * l.experts, "experts_blob", false},
                {l.shared_blob, bw, "shared_blob", false},
                {l.shared_gate, l.width, "shared_gate", false},
                {x, (long long)tokens * l.width, "x", false},
                {y, (long long)tokens * l.width, "y", false},
                {ids, (long long)tokens * l.top_k, "ids", false},
                {weights, (long long)tokens * l.top_k, "weights", false}};
    void *ptr[9];
    for (int i = 0; i < 9; ++i) {
        ptr[i] = nullptr;
        if (need[i].optional && need[i].h == 0) continue;
        Buffer *b = find(ctx, need[i].h);
        if (!b) return fail(ctx, STRATA_ERR_HANDLE, "moe layer: %s is not a live buffer", need[i].what);
        if ((long long)b->length < need[i].n)
            return fail(ctx, STRATA_ERR_LAYOUT, "moe layer: %s holds %llu elements, needs %lld", need[i].what,
                        (unsigned long long)b->length, need[i].n);
        ptr[i] = b->ptr;
    }
    if (int r = use_device(ctx)) return r;
    const size_t ws = fast      ? moe_fast_scratch_bytes(tokens, l.width, l.ff, l.experts, l.top_k)
                      : medium  ? moe_medium_scratch_bytes(tokens, l.width, l.ff, l.experts, l.top_k)
                      : prefill ? moe_prefill_scratch_bytes(tokens, l.width, l.ff, l.experts, l.top_k)
                                : moe_scratch_bytes(tokens, l.width, l.ff, l.experts, l.top_k);
    if (ws > ctx->workspace_bytes) {
        if (ctx->capturing)
            return fail(ctx, STRATA_ERR_RANGE, "the layer's workspace must be sized before capture: run the call once first");
        CUDA_OR_FAIL(ctx, cudaStreamSynchronize(ctx->stream), "workspace resize");
        if (ctx->workspace) cudaFree(ctx->workspace);
        ctx->workspace = nullptr;
        ctx->workspace_bytes = 0;
        cudaError_t e = cudaMalloc(&ctx->workspace, ws);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(ctx, STRATA_ERR_ALLOC, "workspace allocation of %zu bytes failed", ws);
        }
        ctx->workspace_bytes = ws;
    }
    MoeLayerDev L{l.width, l.ff, l.experts, l.top_k, (const float *)ptr[0], (const float *)ptr[1], (const unsigned *)ptr[2], bw,
                  (const unsigned *)ptr[3], (const float *)ptr[4]};
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    if (ctx->profile && (fast || medium || prefill)) {
        for (cudaEvent_t &x : ev) {
            if (!ctx->spare_events.empty()) {
                x = ctx->spare_events.back();
                ctx->spare_events.pop_back();
            } else {
                CUDA_OR_FAIL(ctx, cudaEventCreate(&x), "cudaEventCreate");
            }
        }
        ++ctx->profiled_calls;
    }
    cudaError_t e;
    if (fast || medium) {
        if (ev[0]) CUDA_OR_FAIL(ctx, cudaEventRecord(ev[0], ctx->stream), "cudaEventRecord");
        e = fast && decode1 ? moe_forward_decode1(L, (const float *)ptr[5], (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], ctx->decode1_xchg,
                                                  ctx->fast_sync + 4, ctx->sms, ctx->stream, ctx->err_dev)
            : fast ? moe_forward_fast(L, (const float *)ptr[5], tokens, (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], ctx->workspace,
                                      ctx->fast_sync, ctx->sms, ctx->stream, ctx->err_dev)
                   : moe_forward_medium(L, (const float *)ptr[5], tokens, (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], ctx->workspace,
                                      ctx->fast_sync, ctx->sms, ctx->stream, ctx->err_dev);
        if (ev[0]) {
            CUDA_OR_FAIL(ctx, cudaEventRecord(ev[1], ctx->stream), "cudaEventRecord");
            ctx->marks.push_back({3, ev[0], ev[1]});
            ctx->spare_events.push_back(ev[2]);
            ctx->spare_events.push_back(ev[3]);
        }
    } else if (prefill) {
        e = moe_forward_prefill(L, (const float *)ptr[5], tokens, (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], ctx->workspace,
                                ctx->sms, ctx->stream, ctx->err_dev, ev[0] ? ev : nullptr);
        if (ev[0]) {
            // the three phases share their boundary events: copies of the handles in each pair
            ctx->marks.push_back({0, ev[0], ev[1]});
            ctx->marks.push_back({1, ev[1], ev[2]});
            ctx->marks.push_back({2, ev[2], ev[3]});
        }
    } else {
        MoeScratch s = moe_scratch_carve(ctx->workspace, tokens, l.width, l.ff, l.experts, l.top_k);
        e = moe_forward_exact(L, (const float *)ptr[5], tokens, (float *)ptr[6], (int *)ptr[7], (float *)ptr[8], s, ctx->stream,
                              ctx->err_dev);
    }
    if (e != cudaSuccess) return cuda_fail(ctx, e, "strata_moe_forward");
    ++ctx->fused_calls;
    return STRATA_OK;
}

int strata_synth_blobs(strata_ctx *ctx, strata_buf buf, uint64_t offset, uint64_t seed, int32_t layer, int32_t first_expert,
                       int32_t count, int32_t width, int32_t ff, int32_t shared) {
    if (!ctx) return STRATA_ERR_RANGE;
    if (!blob_geometry_ok(width, ff) || count < 1 || first_expert < 0 || layer < 0)
        return fail(ctx, STRATA_ERR_RANGE, "synth blobs: invalid geometry");
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "synth blobs: unknown buffer");
    const long long n = blob_words_of(width, ff) * count;
    if ((long long)(offset + n) > (long long)b->length) return fail(ctx, STRATA_ERR_LAYOUT, "synth blobs: exceeds buffer");
    if (int r = use_device(ctx)) return r;
    cudaError_t e = synth_expert_blobs((unsigned *)b->ptr + offset, seed, layer, first_expert, count, width, ff, shared, ctx->stream);
    return e == cudaSuccess ? STRATA_OK : cuda_fail(ctx, e, "synth blobs");
}

int strata_synth_normals(strata_ctx *ctx, strata_buf buf, uint64_t offset, uint64_t seed, uint64_t tag, uint64_t sub, uint64_t start,
                         uint64_t count, double scale) {
    if (!ctx) return STRATA_ERR_RANGE;
    Buffer *b = find(ctx, buf);
    if (!b) return fail(ctx, STRATA_ERR_HANDLE, "synth normals: unknown buffer");
    if (offset + count > b->length) return fail(ctx, STRATA_ERR_LAYOUT, "synth normals: exceeds buffer");
    if (!count) return STRATA_OK;
    if (int r = use_device(ctx)) return r;
    cudaError_t e = synth_normals_f32((float *)b->ptr + offset, synth_stream_key(seed, tag, sub), (long long)start, (long long)count, scale,
                                      ctx->stream);
    return e == cudaSuccess ? STRATA_OK : cuda_fail(ctx, e, "synth normals");
}

}  // extern "C"
