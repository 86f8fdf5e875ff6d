// Communicator of the expert-parallel layer (csrc/ep_comm.cu): the point-to-point transport
// that moves dispatch rows, pair lists and returned rows between the ranks, and the bounded
// host waits that turn a lost peer into an error status instead of a hang.
#pragma once
#include <cuda_runtime.h>

#include <memory>
#include <string>

namespace strata {

// Groups of sends and receives between the ranks, issued on one stream. Within a group the
// k-th send from rank a to rank b matches the k-th receive of b from a, and both name the
// same byte count (as ncclSend/ncclRecv inside ncclGroupStart/End).
class EpTransport {
  public:
    virtual ~EpTransport() = default;
    virtual const char *kind() const = 0;
    virtual void group_start() = 0;
    virtual void send(const void *p, size_t bytes, int peer) = 0;
    virtual void recv(void *p, size_t bytes, int peer) = 0;
    // Issues the group's transfers on `s`. 0 or nonzero with *msg.
    virtual int group_end(cudaStream_t s, std::string *msg) = 0;
    // Host wait for everything issued on `s`, polled against timeout_ms; a transport error or
    // the deadline returns nonzero with *msg (the caller then aborts the transport).
    virtual int wait(cudaStream_t s, std::string *msg) = 0;
    // Tears down whatever may still wait on a peer (ncclCommAbort for NCCL).
    virtual void abort() {}
    long long timeout_ms = 60000;  // strata_ep_set_timeout: bounds every host wait on the peers
};

struct EpComm {
    std::unique_ptr<EpTransport> t;
    int rank = 0, n = 1;
    bool failed = false;           // a wait ran out or a transfer failed: the communicator is unusable
    std::string failure;
    struct Buf {
        void *p = nullptr;
        size_t cap = 0;
    };
    Buf bufs[25];
    int *h_off = nullptr;  // pinned: [0, n] send offsets, [n + 1, 2n] receive counts
    // Expert placement: d_place = [owner rank of expert e][local blob index of expert e] over
    // placed_experts experts; this rank holds n_local blobs, the experts it owns in ascending id.
    int placed_experts = 0;
    int n_local = 0;
    int *d_place = nullptr;
    size_t place_cap = 0;
    ~EpComm();
    // grow-only device buffer i of at least `bytes`
    void *get(int i, size_t bytes, cudaError_t &e);
    // marks the communicator failed (first reason kept) and aborts the transport
    void fail(const std::string &why);
};

int ep_unique_id(char *out128, std::string *err);
EpComm *ep_create(int rank, int n_ranks, const char *id128, long long timeout_ms, std::string *err);
// Same-device loopback: n virtual ranks, one context (and stream) each, on one GPU. The hub
// is shared by the ranks' communicators; handles count references.
int ep_loopback_hub_create(int n_ranks, unsigned long long *hub, std::string *err);
int ep_loopback_hub_release(unsigned long long hub, std::string *err);
EpComm *ep_create_loopback(unsigned long long hub, int rank, long long timeout_ms, std::string *err);
void ep_destroy(EpComm *c);
int ep_ranks(const EpComm *c);
// Bounded wait for the stream's work (a synchronising call of a context with a communicator).
int ep_wait(EpComm *c, cudaStream_t s, std::string *msg);

}  // namespace strata
