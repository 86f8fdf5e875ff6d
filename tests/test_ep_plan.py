"""Expert-parallel dispatch/combine protocol on CPU ranks (gloo, world size 2): the host
restatement of the plan the library runs on the device (stratacuda_b200.ep.plan_dispatch:
pairs bucketed by destination rank, token-major inside a bucket), exchanged with variable
all-to-alls, a stand-in expert applied on the owning rank, results returned and combined.
Every pair must reach the rank that owns its expert and every token must get back exactly
its K contributions. No GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, K, H = 512, 10, 8


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def expert_fn(e, row):
    """Stand-in expert: a row-dependent value that identifies the expert."""
    return row * (1.0 + e / 1000.0) + e


def worker(rank, world, port, T, seed, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stratacuda_b200.ep import plan_dispatch
        rng = np.random.default_rng(seed + rank)
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int64)
        if T > 3:
            ids[3, 5] = -1  # a pair without an expert travels nowhere
        x = rng.standard_normal((T, H))
        pos, counts = plan_dispatch(ids, E, world)
        el = E // world
        # send order: rows of x per pair, the pair's expert, the owning rank check
        S = int(counts.sum())
        send_x = np.zeros((S, H))
        send_e = np.zeros(S, np.int64)
        for t in range(T):
            for k in range(K):
                p = pos[t, k]
                if p >= 0:
                    send_x[p] = x[t]
                    send_e[p] = ids[t, k]
        rcounts = torch.empty(world, dtype=torch.int64)
        dist.all_to_all_single(rcounts, torch.tensor(counts))
        rc = rcounts.tolist()
        R = sum(rc)
        recv_x = torch.empty((R, H), dtype=torch.float64)
        recv_e = torch.empty(R, dtype=torch.int64)
        dist.all_to_all_single(recv_x, torch.from_numpy(send_x), rc, counts.tolist())
        dist.all_to_all_single(recv_e, torch.from_numpy(send_e), rc, counts.tolist())
        assert all(rank * el <= int(e) < (rank + 1) * el for e in recv_e.tolist()), "pair on the wrong rank"
        outs = torch.stack([torch.from_numpy(expert_fn(int(e), r.numpy())) for e, r in zip(recv_e, recv_x)]) if R else \
            torch.empty((0, H), dtype=torch.float64)
        back = torch.empty((S, H), dtype=torch.float64)
        dist.all_to_all_single(back, outs, counts.tolist(), rc)
        y = np.zeros((T, H))
        for t in range(T):
            for k in range(K):
                if pos[t, k] >= 0:
                    y[t] += back[pos[t, k]].numpy()
        ref = np.zeros((T, H))
        for t in range(T):
            for k in range(K):
                if ids[t, k] >= 0:
                    ref[t] += expert_fn(int(ids[t, k]), x[t])
        out[rank] = float(np.abs(y - ref).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 37])
def test_ep_plan_two_ranks(T):
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(2, free_port(), T, 5, out), nprocs=2, join=True)
    assert set(out.keys()) == {0, 1}
    assert max(out.values()) < 1e-9


def test_plan_dispatch_is_stable_and_complete():
    from stratacuda_b200.ep import plan_dispatch
    ids = np.array([[5, 300, 1], [300, 2, 511], [-1, 256, 4]])
    pos, counts = plan_dispatch(ids, 512, 2)
    # rank 0 (experts 0..255) in token-major order: (0,0) e5, (0,2) e1, (1,1) e2, (2,2) e4;
    # rank 1 (256..511): (0,1) e300, (1,0) e300, (1,2) e511, (2,1) e256; (2,0) has no expert
    assert counts.tolist() == [4, 4]
    assert pos.tolist() == [[0, 4, 1], [5, 2, 6], [-1, 7, 3]]
