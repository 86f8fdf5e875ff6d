"""Expert-parallel MoE layer (strata_moe_ep_forward): one process per GPU over NCCL, or n
virtual ranks on one GPU over the library's loopback transport (tests).

The layer's routed experts are sharded: by default rank r holds experts [r E/n, (r + 1) E/n);
``ep_set_placement`` gives any other owner per expert, e.g. ``balanced_placement`` of the
experts' routed rows, so that a skewed router does not load one rank with the popular
experts. A rank runs its experts for every rank's tokens that route there; router, shared gate
and shared expert are replicated. Each rank passes its own tokens and gets back their y, ids and weights. The
reference has no multi-GPU path; the layer's arithmetic is the tensor-core path's (routing
bit-exact, y within 2e-3 relative L2).

The NCCL communicator lives in the library (bound at run time to the process's libnccl.so.2);
the ranks share its 128-byte unique id through torch.distributed (any backend).

Failure detection has two layers. In the library, every host wait on the peers is bounded
(strata_ep_set_timeout) and a lost peer aborts the communicator with an error status. On the
host, ``EpHealth`` is a step rendezvous through the process group's store: before each step a
rank announces it and waits, with a deadline, for every peer to announce the same step, so a
rank that crashed or left between steps is reported by name before anyone launches the next
exchange (the reference's analogue is its failed-session state, src/engine.js:147-151).
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from . import synth
from .backend import Buffer, CudaBackend
from .moe import blob_layout


def ep_init(backend: CudaBackend, rank: int, n_ranks: int) -> None:
    """strata_ep_init on every rank; the unique id travels by torch.distributed.broadcast_object_list."""
    import torch.distributed as dist
    ident = [None]
    if rank == 0:
        buf = C.create_string_buffer(128)
        backend._check(backend.lib.strata_ep_unique_id(backend.ctx, buf, 128))
        ident[0] = bytes(buf.raw)
    if n_ranks > 1:
        dist.broadcast_object_list(ident, src=0)
    backend._check(backend.lib.strata_ep_init(backend.ctx, int(rank), int(n_ranks), C.c_char_p(ident[0])))


def ep_init_loopback(backends: list[CudaBackend], timeout_ms: int | None = None) -> None:
    """n virtual ranks on one GPU: backends[r] (one context each, same device) becomes rank r
    of a loopback hub. Drive the ranks' forwards from n host threads (ctypes releases the GIL),
    as separate processes would."""
    b0 = backends[0]
    hub = C.c_uint64()
    b0._check(b0.lib.strata_ep_loopback_create(b0.ctx, len(backends), C.byref(hub)))
    try:
        for r, b in enumerate(backends):
            if timeout_ms is not None:
                b._check(b.lib.strata_ep_set_timeout(b.ctx, int(timeout_ms)))
            b._check(b.lib.strata_ep_init_loopback(b.ctx, r, hub.value))
    finally:
        b0._check(b0.lib.strata_ep_loopback_release(b0.ctx, hub.value))


def ep_set_timeout(backend: CudaBackend, timeout_ms: int) -> None:
    """Bound of every host wait on the peers (default 60 s)."""
    backend._check(backend.lib.strata_ep_set_timeout(backend.ctx, int(timeout_ms)))


def ep_set_placement(backend: CudaBackend, owner) -> None:
    """strata_ep_set_placement: owner[e] = the rank holding expert e (the same on every rank);
    None restores the contiguous placement."""
    if owner is None:
        return
    own = np.ascontiguousarray(owner, dtype=np.int32)
    backend._check(backend.lib.strata_ep_set_placement(backend.ctx, int(own.size), own.ctypes.data_as(C.POINTER(C.c_int32))))


def balanced_placement(rows: np.ndarray, n_ranks: int, expert_cost: float = 64.0) -> np.ndarray:
    """Owner rank per expert from the experts' routed rows (longest processing time first: the
    expert with the most rows goes to the least loaded rank). An expert costs its rows plus
    ``expert_cost`` rows' worth for its weights, which a rank reads once however few rows it has.
    Every rank gets at least one expert."""
    rows = np.asarray(rows, dtype=np.float64)
    E = rows.size
    if E < n_ranks:
        raise ValueError("fewer experts than ranks")
    cost = rows + expert_cost
    owner = np.empty(E, np.int32)
    load = np.zeros(n_ranks)
    count = np.zeros(n_ranks, np.int64)
    for e in np.argsort(-cost, kind="stable"):
        empty = np.flatnonzero(count == 0)
        r = int(empty[0]) if empty.size and (E - count.sum()) <= empty.size else int(np.argmin(load))
        owner[e] = r
        load[r] += cost[e]
        count[r] += 1
    return owner


def owned_experts(owner, rank: int, experts: int, n_ranks: int) -> np.ndarray:
    """The experts rank `rank` holds, in blob order (ascending id)."""
    if owner is None:
        el = experts // n_ranks
        return np.arange(rank * el, (rank + 1) * el)
    return np.flatnonzero(np.asarray(owner) == rank)


class EpPeerFailure(RuntimeError):
    """A peer rank did not reach a step within the deadline, or announced that it left."""

    def __init__(self, missing: list[int], step: int, left: list[int]):
        what = []
        if left:
            what.append(f"rank(s) {left} left")
        if missing:
            what.append(f"rank(s) {missing} did not reach step {step}")
        super().__init__("expert-parallel peers failed: " + "; ".join(what))
        self.missing, self.left, self.step = missing, left, step


class EpHealth:
    """Host-side liveness of the expert-parallel ranks through a torch.distributed store.

    ``arrive(step)`` publishes this rank's step and waits until every peer has published the
    same step; it raises EpPeerFailure naming the ranks that announced ``leave()`` (at once) or
    did not arrive within ``timeout_s``. Call it before each step's exchange: a peer that dies
    between steps is then reported on the host, before any collective with it is launched."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "strata_ep_health"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def leave(self) -> None:
        self.store.set(self._key("left", self.rank), "1")

    def _has(self, key: str) -> bool:
        return bool(self.store.check([key]))

    def arrive(self, step: int, poll_s: float = 0.005) -> None:
        self.store.set(self._key("step", step, self.rank), "1")
        deadline = time.monotonic() + self.timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            pending = [r for r in pending if not self._has(self._key("step", step, r))]
            left = [r for r in range(self.world) if r != self.rank and self._has(self._key("left", r))]
            left_pending = [r for r in left if r in pending]
            if not pending:
                return
            if left_pending or time.monotonic() >= deadline:
                raise EpPeerFailure([r for r in pending if r not in left_pending], step, left_pending)
            time.sleep(poll_s)


@dataclass
class EpMoeLayer:
    backend: CudaBackend
    rank: int
    n_ranks: int
    width: int
    ff: int
    experts: int  # total over the ranks
    top_k: int
    router: Buffer
    experts_blob: Buffer  # this rank's experts / n_ranks blobs
    shared_blob: Buffer
    shared_gate: Buffer
    router_bias: Buffer | None = None
    owner: np.ndarray | None = None  # owner rank per expert (None: contiguous)

    @property
    def local_ids(self) -> np.ndarray:
        return owned_experts(self.owner, self.rank, self.experts, self.n_ranks)

    @property
    def local_experts(self) -> int:
        return int(self.local_ids.size)

    def forward(self, x: Buffer, tokens: int, y: Buffer, ids: Buffer, weights: Buffer) -> None:
        b = self.backend
        st = L.StrataMoeLayer(self.width, self.ff, self.experts, self.top_k, self.router.handle,
                              self.router_bias.handle if self.router_bias is not None else 0, self.experts_blob.handle,
                              self.shared_blob.handle, self.shared_gate.handle)
        b._check(b.lib.strata_moe_ep_forward(b.ctx, C.byref(st), x.handle, int(tokens), y.handle, ids.handle, weights.handle))

    def free(self) -> None:
        for buf in (self.router, self.experts_blob, self.shared_blob, self.shared_gate, self.router_bias):
            if buf is not None:
                self.backend.free(buf)

    @classmethod
    def synthesize(cls, backend: CudaBackend, rank: int, n_ranks: int, seed: int, layer: int, width: int = 2048, ff: int = 512,
                   experts: int = 512, top_k: int = 10, zipf: float | None = None, owner=None) -> "EpMoeLayer":
        """The seeded synthetic layer of stratacuda_b200.moe.MoeLayer.synthesize, this rank's
        experts only (``owner``: the placement set with ep_set_placement; None: contiguous)."""
        if owner is None and experts % n_ranks:
            raise ValueError("experts must be a multiple of the ranks")
        words = blob_layout(width, ff)["blob_bytes"] // 4
        lib, ctx = backend.lib, backend.ctx
        mine = owned_experts(owner, rank, experts, n_ranks)
        el = int(mine.size)
        router = backend.alloc(experts * width, zero=False)
        backend._check(lib.strata_synth_normals(ctx, router.handle, 0, seed, synth.TAG_ROUTER, layer, 0, experts * width, 0.02))
        gate = backend.alloc(width, zero=False)
        backend._check(lib.strata_synth_normals(ctx, gate.handle, 0, seed, synth.TAG_SHARED_GATE, layer, 0, width, 0.02))
        blobs = backend.alloc(el * words, "u32", zero=False)
        i = 0
        while i < el:  # runs of consecutive ids in one call
            j = i + 1
            while j < el and mine[j] == mine[j - 1] + 1:
                j += 1
            backend._check(lib.strata_synth_blobs(ctx, blobs.handle, i * words, seed, layer, int(mine[i]), j - i, width, ff, 0))
            i = j
        shared = backend.alloc(words, "u32", zero=False)
        backend._check(lib.strata_synth_blobs(ctx, shared.handle, 0, seed, layer, 0, 1, width, ff, 1))
        bias = None if zipf is None else backend.alloc(synth.zipf_bias(seed, experts, zipf))
        return cls(backend, rank, n_ranks, width, ff, experts, top_k, router, blobs, shared, gate, bias,
                   None if owner is None else np.asarray(owner, np.int32))


def plan_dispatch(ids: np.ndarray, experts: int, n_ranks: int, placement=None):
    """Host restatement of the dispatch plan the library computes on the device (used by the
    CPU tests). One row per (token, destination rank) that owns at least one of the token's
    experts (placement[e], by default rank r owns [r E/n, (r + 1) E/n)), bucketed by rank,
    token-major inside a bucket. Returns (row of every (token, rank) in the send order or -1
    [T, n], rows per rank [n], pairs: for every send row the token's (k, expert) pairs on that
    rank in k order)."""
    if placement is None:
        placement = np.arange(experts) // (experts // n_ranks)
    placement = np.asarray(placement)
    T, K = ids.shape
    valid = (ids >= 0) & (ids < experts)
    owner = np.where(valid, placement[np.where(valid, ids, 0)], -1)
    has = np.zeros((T, n_ranks), bool)
    for t in range(T):
        for k in range(K):
            if owner[t, k] >= 0:
                has[t, owner[t, k]] = True
    counts = has.sum(axis=0).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    pos = np.full((T, n_ranks), -1, np.int64)
    pairs = [None] * int(counts.sum())
    seen = np.zeros(n_ranks, np.int64)
    for t in range(T):
        for p in range(n_ranks):
            if has[t, p]:
                row = offsets[p] + seen[p]
                seen[p] += 1
                pos[t, p] = row
                pairs[row] = [(k, int(ids[t, k])) for k in range(K) if owner[t, k] == p]
    return pos, counts, pairs
