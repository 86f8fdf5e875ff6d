"""Expert-parallel dispatch/combine protocol on CPU ranks (gloo, world size 2): the host
restatement of the plan the library runs on the device (stratacuda_b200.ep.plan_dispatch: one
row per (token, destination rank), bucketed by rank, token-major inside a bucket, with the
token's pairs on that rank), exchanged with variable all-to-alls; the owning rank applies a
stand-in expert to every pair and sums the weighted results per received row (pre-combine);
one row per (token, rank) comes back and the source adds them in rank order. Every token must
get exactly the weighted sum of its K experts. No GPU."""
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
            ids[2] = np.arange(K)  # every expert on rank 0: one row, to rank 0 only
        w = rng.random((T, K))
        x = rng.standard_normal((T, H))
        pos, counts, pairs = plan_dispatch(ids, E, world)
        el = E // world
        S = int(counts.sum())
        # a send row: the token's x, then K (expert, weight) slots (expert -1 unused)
        send_x = np.zeros((S, H))
        send_meta = np.full((S, 2 * K), -1.0)
        for t in range(T):
            for p in range(world):
                row = pos[t, p]
                if row >= 0:
                    send_x[row] = x[t]
                    for j, (k, e) in enumerate(pairs[row]):
                        send_meta[row, 2 * j], send_meta[row, 2 * j + 1] = e, w[t, k]
        rcounts = torch.empty(world, dtype=torch.int64)
        dist.all_to_all_single(rcounts, torch.tensor(counts))
        rc = rcounts.tolist()
        R = sum(rc)
        recv_x = torch.empty((R, H), dtype=torch.float64)
        recv_meta = torch.empty((R, 2 * K), dtype=torch.float64)
        dist.all_to_all_single(recv_x, torch.from_numpy(send_x), rc, counts.tolist())
        dist.all_to_all_single(recv_meta, torch.from_numpy(send_meta), rc, counts.tolist())
        outs = torch.zeros((R, H), dtype=torch.float64)
        for i in range(R):  # pre-combine: the weighted sum of the row's pairs
            for j in range(K):
                e = int(recv_meta[i, 2 * j])
                if e < 0:
                    continue
                assert rank * el <= e < (rank + 1) * el, "pair on the wrong rank"
                outs[i] += float(recv_meta[i, 2 * j + 1]) * torch.from_numpy(expert_fn(e, recv_x[i].numpy()))
        back = torch.empty((S, H), dtype=torch.float64)
        dist.all_to_all_single(back, outs, counts.tolist(), rc)
        y = np.zeros((T, H))
        for t in range(T):
            for p in range(world):
                if pos[t, p] >= 0:
                    y[t] += back[pos[t, p]].numpy()
        ref = np.zeros((T, H))
        for t in range(T):
            for k in range(K):
                if ids[t, k] >= 0:
                    ref[t] += w[t, k] * expert_fn(int(ids[t, k]), x[t])
        out[rank] = (float(np.abs(y - ref).max()), S, T)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 37])
def test_ep_plan_two_ranks(T):
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(2, free_port(), T, 5, out), nprocs=2, join=True)
    assert set(out.keys()) == {0, 1}
    for err, rows, tokens in out.values():
        assert err < 1e-9
        assert rows <= 2 * tokens  # at most one row per (token, rank)


def test_plan_dispatch_is_stable_and_complete():
    from stratacuda_b200.ep import plan_dispatch
    ids = np.array([[5, 300, 1], [300, 2, 511], [-1, 256, 4], [7, 8, 9]])
    pos, counts, pairs = plan_dispatch(ids, 512, 2)
    # rank 0 (experts 0..255), token-major: t0, t1, t2, t3; rank 1 (256..511): t0, t1, t2
    assert counts.tolist() == [4, 3]
    assert pos.tolist() == [[0, 4], [1, 5], [2, 6], [3, -1]]
    assert pairs[0] == [(0, 5), (2, 1)] and pairs[4] == [(1, 300)]
    assert pairs[5] == [(0, 300), (2, 511)] and pairs[6] == [(1, 256)] and pairs[3] == [(0, 7), (1, 8), (2, 9)]


def test_plan_dispatch_with_a_placement():
    """Experts on the ranks of an explicit placement (owner per expert) instead of contiguous
    slices: the rows go where the experts live."""
    from stratacuda_b200.ep import owned_experts, plan_dispatch
    owner = np.zeros(512, np.int64)
    owner[1::2] = 1  # odd experts on rank 1
    ids = np.array([[5, 300, 1], [300, 2, 511], [-1, 256, 4]])
    pos, counts, pairs = plan_dispatch(ids, 512, 2, owner)
    # rank 0 (even): t0 (300), t1 (300, 2), t2 (256, 4); rank 1 (odd): t0 (5, 1), t1 (511)
    assert counts.tolist() == [3, 2]
    assert pos.tolist() == [[0, 3], [1, 4], [2, -1]]
    assert pairs[0] == [(1, 300)] and pairs[3] == [(0, 5), (2, 1)] and pairs[2] == [(1, 256), (2, 4)]
    assert owned_experts(owner, 1, 512, 2).tolist() == list(range(1, 512, 2))


def test_balanced_placement_evens_skewed_rows():
    """Zipf-skewed rows over 512 experts: the placement's heaviest rank is within a few percent
    of the mean (contiguous slices put whole hot runs on one rank), every rank owns an expert,
    and the placement is a function of the rows alone (every rank computes the same)."""
    from stratacuda_b200.ep import balanced_placement
    rng = np.random.default_rng(3)
    bias = np.log(1.0 / np.arange(1, 513) ** 1.1)[rng.permutation(512)]
    # 4096 tokens, top-10 of Gumbel-perturbed biases: an expert takes at most one row per token
    ids = np.argsort(-(bias + rng.gumbel(size=(4096, 512))), axis=1)[:, :10]
    rows = np.bincount(ids.reshape(-1), minlength=512).astype(np.float64)
    for n in (2, 4, 8):
        owner = balanced_placement(rows, n)
        load = np.bincount(owner, weights=rows + 64.0, minlength=n)
        # no better than the heaviest single expert allows, else within 3% of the mean
        assert load.max() <= max(1.03 * load.mean(), (rows + 64.0).max() + 1e-9), (n, load)
        contiguous = np.bincount(np.arange(512) // (512 // n), weights=rows + 64.0, minlength=n)
        assert load.max() <= contiguous.max()
        assert np.bincount(owner, minlength=n).min() >= 1
        assert np.array_equal(owner, balanced_placement(rows.copy(), n))
    tiny = balanced_placement(np.array([100.0, 0, 0, 0]), 4)
    assert sorted(tiny.tolist()) == [0, 1, 2, 3]
