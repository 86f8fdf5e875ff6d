// Transports of the expert-parallel layer (csrc/ep_comm.h).
//
// NCCL. Bound at run time (the process's loaded libnccl.so.2 first, e.g. the one torch
// brought, else the system's), so the library has no NCCL link dependency. The communicator
// is created non-blocking (ncclConfig_t.blocking = 0): initialisation and every group end are
// polled with ncclCommGetAsyncError, and every host wait on the stream (the forward's read of
// the receive counts, a synchronising call of the context) polls cudaStreamQuery and the
// communicator's asynchronous error against a deadline. When a peer has died the wait ends
// with an error status after the deadline and the communicator is aborted (ncclCommAbort),
// which also ends NCCL's kernels still waiting on that peer; the context stays usable for
// everything but expert parallelism until strata_ep_init is called again.
//
// Loopback. n virtual ranks on ONE device, each with its own context and stream, driven by n
// host threads (the test harness of the layer at 2, 4 and 8 ranks without 8 GPUs). A group
// end is a three-step rendezvous on the hub: post the group's operations and an event
// recorded after the rank's preceding work; after everyone has posted, each rank copies
// every receive from the matching send (cudaMemcpyAsync on its own stream, after the
// sender's event) and records a second event; after everyone has issued its copies, each
// rank makes its stream wait for the copies out of its send buffers before anything later
// can overwrite them. Nothing on the GPU waits for another rank: the ordering is stream
// events only, and every host rendezvous has the same deadline as the NCCL waits.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>
#include <unordered_map>
#include <vector>

#include "ep_comm.h"

namespace strata {

namespace {

using Clock = std::chrono::steady_clock;

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi &nccl() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](auto &fn, const char *name) { fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name)); };
        sym(a.GetUniqueId, "ncclGetUniqueId");
        sym(a.CommInitRankConfig, "ncclCommInitRankConfig");
        sym(a.CommFinalize, "ncclCommFinalize");
        sym(a.CommDestroy, "ncclCommDestroy");
        sym(a.CommAbort, "ncclCommAbort");
        sym(a.CommGetAsyncError, "ncclCommGetAsyncError");
        sym(a.GroupStart, "ncclGroupStart");
        sym(a.GroupEnd, "ncclGroupEnd");
        sym(a.Send, "ncclSend");
        sym(a.Recv, "ncclRecv");
        sym(a.GetErrorString, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommDestroy && a.CommAbort && a.CommGetAsyncError && a.GroupStart && a.GroupEnd &&
               a.Send && a.Recv && a.GetErrorString;
    });
    return a;
}

struct P2pOp {
    bool send;
    const void *src;
    void *dst;
    size_t bytes;
    int peer;
};

// Polls until pred() is true or the deadline passes: busy for the first 2 ms (a healthy wait
// is usually that short and its latency is on the layer's path), then 50 us sleeps.
template <class Pred>
bool poll_until(Pred pred, long long timeout_ms) {
    const auto start = Clock::now(), deadline = start + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        if (pred()) return true;
        const auto now = Clock::now();
        if (now >= deadline) return false;
        if (now - start > std::chrono::milliseconds(2)) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

class NcclTransport final : public EpTransport {
  public:
    ncclComm_t comm = nullptr;
    bool aborted = false;
    std::vector<P2pOp> ops;

    ~NcclTransport() override {
        if (!comm) return;
        if (aborted) return;  // ncclCommAbort released it
        const NcclApi &a = nccl();
        bool clean = true;
        if (a.CommFinalize) {
            ncclResult_t r = a.CommFinalize(comm);
            if (r == ncclInProgress) r = settle(nullptr);
            clean = r == ncclSuccess;
        }
        if (clean) {
            ncclResult_t r = a.CommDestroy(comm);
            if (r == ncclInProgress) settle(nullptr);
        } else {
            a.CommAbort(comm);
        }
    }
    const char *kind() const override { return "nccl"; }
    void group_start() override { ops.clear(); }
    void send(const void *p, size_t bytes, int peer) override { ops.push_back({true, p, nullptr, bytes, peer}); }
    void recv(void *p, size_t bytes, int peer) override { ops.push_back({false, nullptr, p, bytes, peer}); }

    // Polls the communicator's asynchronous state until it leaves ncclInProgress.
    ncclResult_t settle(std::string *msg) {
        ncclResult_t st = ncclInProgress;
        const bool done = poll_until(
            [&] {
                if (nccl().CommGetAsyncError(comm, &st) != ncclSuccess) st = ncclInternalError;
                return st != ncclInProgress;
            },
            timeout_ms);
        if (!done) {
            if (msg) *msg = "NCCL: an operation did not complete within " + std::to_string(timeout_ms) + " ms (a peer is gone or stalled)";
            return ncclInProgress;
        }
        if (st != ncclSuccess && msg) *msg = std::string("NCCL: ") + nccl().GetErrorString(st);
        return st;
    }
    int group_end(cudaStream_t s, std::string *msg) override {
        const NcclApi &a = nccl();
        ncclResult_t r = a.GroupStart();
        for (const P2pOp &o : ops) {
            if (r != ncclSuccess && r != ncclInProgress) break;
            r = o.send ? a.Send(o.src, o.bytes, ncclInt8, o.peer, comm, s) : a.Recv(o.dst, o.bytes, ncclInt8, o.peer, comm, s);
        }
        const ncclResult_t e = a.GroupEnd();
        if (r == ncclSuccess || r == ncclInProgress) r = e;
        if (r == ncclInProgress) r = settle(msg);
        else if (r != ncclSuccess) *msg = std::string("NCCL: ") + a.GetErrorString(r);
        return r == ncclSuccess ? 0 : 1;
    }
    int wait(cudaStream_t s, std::string *msg) override {
        cudaError_t ce = cudaSuccess;
        ncclResult_t ne = ncclSuccess;
        const bool done = poll_until(
            [&] {
                ce = cudaStreamQuery(s);
                if (ce != cudaErrorNotReady) return true;
                if (nccl().CommGetAsyncError(comm, &ne) != ncclSuccess) ne = ncclInternalError;
                return ne != ncclSuccess && ne != ncclInProgress;
            },
            timeout_ms);
        if (!done) {
            *msg = "expert-parallel exchange did not complete within " + std::to_string(timeout_ms) + " ms (a peer is gone or stalled)";
            return 1;
        }
        if (ce != cudaSuccess && ce != cudaErrorNotReady) {
            *msg = std::string("CUDA: ") + cudaGetErrorString(ce);
            return 1;
        }
        if (ne != ncclSuccess && ne != ncclInProgress) {
            *msg = std::string("NCCL asynchronous error: ") + nccl().GetErrorString(ne);
            return 1;
        }
        return 0;
    }
    void abort() override {
        if (comm && !aborted) {
            nccl().CommAbort(comm);
            aborted = true;
        }
    }
};

// ---------------------------------------------------------------- loopback
struct LoopbackHub {
    int n = 0;
    std::mutex m;
    std::condition_variable cv;
    unsigned long long gen = 0;
    int count = 0;
    bool broken = false;
    std::string why;
    std::vector<std::vector<P2pOp>> ops;       // [rank] the posted group
    std::vector<cudaEvent_t> ready, copied;    // [rank] owned by the rank's transport
    std::vector<bool> joined;

    // Generation barrier with a deadline; a timeout breaks the hub for every rank.
    int barrier(std::unique_lock<std::mutex> &lk, long long timeout_ms, std::string *msg) {
        if (broken) {
            *msg = why;
            return 1;
        }
        const unsigned long long g = gen;
        if (++count == n) {
            count = 0;
            ++gen;
            cv.notify_all();
            return 0;
        }
        const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
        while (gen == g && !broken) {
            if (cv.wait_until(lk, deadline) == std::cv_status::timeout && gen == g && !broken) {
                broken = true;
                why = "loopback exchange: a rank did not reach the exchange within " + std::to_string(timeout_ms) + " ms";
                cv.notify_all();
            }
        }
        if (gen != g) return 0;
        *msg = why;
        return 1;
    }
    void breakdown(const std::string &reason) {
        if (!broken) {
            broken = true;
            why = reason;
        }
        cv.notify_all();
    }
};

std::mutex g_hub_mutex;
std::unordered_map<unsigned long long, std::shared_ptr<LoopbackHub>> g_hubs;
unsigned long long g_next_hub = 1;

class LoopbackTransport final : public EpTransport {
  public:
    std::shared_ptr<LoopbackHub> hub;
    int rank = 0;
    cudaEvent_t ready = nullptr, copied = nullptr;
    std::vector<P2pOp> ops;

    ~LoopbackTransport() override {
        if (hub) {
            std::lock_guard<std::mutex> lk(hub->m);
            hub->ready[rank] = nullptr;
            hub->copied[rank] = nullptr;
            hub->joined[rank] = false;
            hub->breakdown("loopback exchange: a rank left");
        }
        if (ready) cudaEventDestroy(ready);
        if (copied) cudaEventDestroy(copied);
    }
    const char *kind() const override { return "loopback"; }
    void group_start() override { ops.clear(); }
    void send(const void *p, size_t bytes, int peer) override { ops.push_back({true, p, nullptr, bytes, peer}); }
    void recv(void *p, size_t bytes, int peer) override { ops.push_back({false, nullptr, p, bytes, peer}); }

    int group_end(cudaStream_t s, std::string *msg) override {
        LoopbackHub &h = *hub;
        cudaError_t e = cudaEventRecord(ready, s);  // the rank's sends are complete once its preceding work is
        if (e != cudaSuccess) {
            *msg = std::string("cudaEventRecord: ") + cudaGetErrorString(e);
            std::lock_guard<std::mutex> lk(h.m);
            h.breakdown(*msg);
            return 1;
        }
        struct Copy {
            void *dst;
            const void *src;
            size_t bytes;
            int peer;
        };
        std::vector<Copy> copies;
        std::vector<cudaEvent_t> peer_ready(h.n, nullptr);
        {
            std::unique_lock<std::mutex> lk(h.m);
            h.ops[rank] = ops;
            if (h.barrier(lk, timeout_ms, msg)) return 1;
            // the k-th receive of this rank from p matches the k-th send of p to this rank
            std::vector<int> seen(h.n, 0);
            for (const P2pOp &o : ops) {
                if (o.send) continue;
                if (o.peer < 0 || o.peer >= h.n) {
                    h.breakdown("loopback exchange: receive from rank " + std::to_string(o.peer) + " outside the group");
                    *msg = h.why;
                    return 1;
                }
                int k = seen[o.peer]++;
                const P2pOp *match = nullptr;
                for (const P2pOp &q : h.ops[o.peer])
                    if (q.send && q.peer == rank && k-- == 0) {
                        match = &q;
                        break;
                    }
                if (!match || match->bytes != o.bytes) {
                    h.breakdown("loopback exchange: rank " + std::to_string(rank) + " receives from rank " + std::to_string(o.peer) +
                                (match ? " a size other than the one sent" : " more than was sent"));
                    *msg = h.why;
                    return 1;
                }
                copies.push_back({o.dst, match->src, o.bytes, o.peer});
                peer_ready[o.peer] = h.ready[o.peer];
            }
        }
        for (int p = 0; p < h.n; ++p)
            if (peer_ready[p] && (e = cudaStreamWaitEvent(s, peer_ready[p], 0)) != cudaSuccess) break;
        for (const Copy &c : copies) {
            if (e != cudaSuccess) break;
            if (c.bytes) e = cudaMemcpyAsync(c.dst, c.src, c.bytes, cudaMemcpyDeviceToDevice, s);
        }
        if (e == cudaSuccess) e = cudaEventRecord(copied, s);
        std::vector<cudaEvent_t> peer_copied(h.n, nullptr);
        {
            std::unique_lock<std::mutex> lk(h.m);
            if (e != cudaSuccess) {
                *msg = std::string("loopback copy: ") + cudaGetErrorString(e);
                h.breakdown(*msg);
                return 1;
            }
            if (h.barrier(lk, timeout_ms, msg)) return 1;
            for (const P2pOp &o : ops)
                if (o.send) peer_copied[o.peer] = h.copied[o.peer];
        }
        // later work of this rank (which may overwrite its send buffers) waits for the copies
        for (int p = 0; p < h.n; ++p)
            if (peer_copied[p] && (e = cudaStreamWaitEvent(s, peer_copied[p], 0)) != cudaSuccess) {
                *msg = std::string("cudaStreamWaitEvent: ") + cudaGetErrorString(e);
                return 1;
            }
        return 0;
    }
    int wait(cudaStream_t s, std::string *msg) override {
        cudaError_t ce = cudaSuccess;
        if (!poll_until([&] { return (ce = cudaStreamQuery(s)) != cudaErrorNotReady; }, timeout_ms)) {
            *msg = "loopback exchange: the stream did not drain within " + std::to_string(timeout_ms) + " ms";
            return 1;
        }
        if (ce != cudaSuccess) {
            *msg = std::string("CUDA: ") + cudaGetErrorString(ce);
            return 1;
        }
        return 0;
    }
    void abort() override {
        if (!hub) return;
        std::lock_guard<std::mutex> lk(hub->m);
        hub->breakdown("loopback exchange: aborted by rank " + std::to_string(rank));
    }
};

}  // namespace

// ---------------------------------------------------------------- EpComm
EpComm::~EpComm() {
    for (Buf &b : bufs)
        if (b.p) cudaFree(b.p);
    if (h_off) cudaFreeHost(h_off);
    if (d_place) cudaFree(d_place);
    if (t && failed) t->abort();
    t.reset();
}

void *EpComm::get(int i, size_t bytes, cudaError_t &e) {
    if (bufs[i].cap < bytes) {
        if (bufs[i].p) cudaFree(bufs[i].p);
        bufs[i].p = nullptr;
        bufs[i].cap = 0;
        const size_t want = (bytes + bytes / 4 + 255) & ~size_t(255);
        e = cudaMalloc(&bufs[i].p, want);
        if (e != cudaSuccess) return nullptr;
        bufs[i].cap = want;
    }
    return bufs[i].p;
}

void EpComm::fail(const std::string &why) {
    if (!failed) {
        failed = true;
        failure = why;
    }
    if (t) t->abort();
}

int ep_unique_id(char *out, std::string *err) {
    if (!nccl().ok) {
        *err = "libnccl.so.2 could not be loaded (or lacks the non-blocking communicator API)";
        return 1;
    }
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) {
        *err = std::string("ncclGetUniqueId: ") + nccl().GetErrorString(r);
        return 1;
    }
    std::memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return 0;
}

static EpComm *finish_create(EpComm *c, int n, std::string *err) {
    if (cudaMallocHost(&c->h_off, sizeof(int) * (2 * n + 2)) != cudaSuccess) {
        *err = "cudaMallocHost of the count mirror failed";
        delete c;
        return nullptr;
    }
    return c;
}

EpComm *ep_create(int rank, int n, const char *id_bytes, long long timeout_ms, std::string *err) {
    if (!nccl().ok) {
        *err = "libnccl.so.2 could not be loaded (or lacks the non-blocking communicator API)";
        return nullptr;
    }
    ncclUniqueId id;
    std::memcpy(id.internal, id_bytes, NCCL_UNIQUE_ID_BYTES);
    auto *c = new EpComm;
    c->rank = rank;
    c->n = n;
    auto t = std::make_unique<NcclTransport>();
    t->timeout_ms = timeout_ms;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = nccl().CommInitRankConfig(&t->comm, n, id, rank, &cfg);
    if (r == ncclInProgress || (r == ncclSuccess && t->comm)) r = t->comm ? t->settle(err) : r;
    if (r != ncclSuccess) {
        if (err->empty()) *err = std::string("ncclCommInitRankConfig: ") + nccl().GetErrorString(r);
        t->abort();
        delete c;
        return nullptr;
    }
    c->t = std::move(t);
    return finish_create(c, n, err);
}

int ep_loopback_hub_create(int n, unsigned long long *hub, std::string *err) {
    if (n < 1 || n > 32) {
        *err = "loopback exchange supports 1 to 32 ranks";
        return 1;
    }
    auto h = std::make_shared<LoopbackHub>();
    h->n = n;
    h->ops.resize(n);
    h->ready.assign(n, nullptr);
    h->copied.assign(n, nullptr);
    h->joined.assign(n, false);
    std::lock_guard<std::mutex> lk(g_hub_mutex);
    *hub = g_next_hub++;
    g_hubs[*hub] = h;
    return 0;
}

int ep_loopback_hub_release(unsigned long long hub, std::string *err) {
    std::lock_guard<std::mutex> lk(g_hub_mutex);
    if (!g_hubs.erase(hub)) {
        *err = "unknown loopback hub";
        return 1;
    }
    return 0;
}

EpComm *ep_create_loopback(unsigned long long hub, int rank, long long timeout_ms, std::string *err) {
    std::shared_ptr<LoopbackHub> h;
    {
        std::lock_guard<std::mutex> lk(g_hub_mutex);
        auto it = g_hubs.find(hub);
        if (it == g_hubs.end()) {
            *err = "unknown loopback hub";
            return nullptr;
        }
        h = it->second;
    }
    if (rank < 0 || rank >= h->n) {
        *err = "loopback rank outside the hub's ranks";
        return nullptr;
    }
    auto t = std::make_unique<LoopbackTransport>();
    t->rank = rank;
    t->timeout_ms = timeout_ms;
    if (cudaEventCreateWithFlags(&t->ready, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->copied, cudaEventDisableTiming) != cudaSuccess) {
        *err = "cudaEventCreate failed";
        return nullptr;
    }
    {
        std::lock_guard<std::mutex> lk(h->m);
        if (h->joined[rank]) {
            *err = "loopback rank joined twice";
            return nullptr;
        }
        h->joined[rank] = true;
        h->ready[rank] = t->ready;
        h->copied[rank] = t->copied;
    }
    t->hub = h;
    auto *c = new EpComm;
    c->rank = rank;
    c->n = h->n;
    c->t = std::move(t);
    return finish_create(c, c->n, err);
}

void ep_destroy(EpComm *c) { delete c; }
int ep_ranks(const EpComm *c) { return c->n; }

int ep_wait(EpComm *c, cudaStream_t s, std::string *msg) {
    if (c->failed) {
        // the transport is aborted: nothing of it can still wait on a peer
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) *msg = std::string("CUDA: ") + cudaGetErrorString(e);
        return e == cudaSuccess ? 0 : 1;
    }
    if (c->t->wait(s, msg)) {
        c->fail(*msg);
        return 1;
    }
    return 0;
}

}  // namespace strata
