"""Failure detection of the expert-parallel host (stratacuda_b200.ep.EpHealth) with gloo ranks
on the CPU: a rank that leaves or dies between steps is reported by name to the survivors
before their next step, within the deadline; healthy ranks pass every step. No GPU is
involved: the failure is made on the host (a rank that exits), never on a device."""
import multiprocessing as mp
import os
import socket
import time

import pytest

from stratacuda_b200.ep import EpHealth, EpPeerFailure


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, mode, q):
    import datetime

    import torch.distributed as dist
    # the store lives in the test process, so that a rank that dies takes nothing down with it
    store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    health = EpHealth(store, rank, world, timeout_s=3.0)
    result = {"rank": rank, "steps": 0, "error": None, "seconds": None}
    for step in range(4):
        if rank == world - 1 and step == 2 and mode != "healthy":
            if mode == "leave":
                health.leave()
            break  # between steps: nothing of this rank is in flight
        t0 = time.monotonic()
        try:
            health.arrive(step)
        except EpPeerFailure as e:
            result["error"] = (str(e), e.missing, e.left, e.step)
            result["seconds"] = time.monotonic() - t0
            break
        result["steps"] += 1
    q.put(result)
    q.close()
    q.join_thread()
    os._exit(0)  # no collective teardown with a lost peer


def run(world, mode):
    import datetime

    import torch.distributed as dist
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    master = dist.TCPStore("127.0.0.1", port, is_master=True, wait_for_workers=False, timeout=datetime.timedelta(seconds=60))
    procs = [ctx.Process(target=_rank, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + 120
    while len(out) < world and time.monotonic() < deadline:
        try:
            r = q.get(timeout=5)
        except Exception:
            continue
        out[r["rank"]] = r
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    del master
    return out


@pytest.mark.timeout(180)
def test_healthy_ranks_pass_every_step():
    out = run(3, "healthy")
    assert all(out[r]["steps"] == 4 and out[r]["error"] is None for r in range(3)), out


@pytest.mark.timeout(180)
@pytest.mark.parametrize("mode", ["leave", "die"])
def test_survivors_learn_of_a_lost_rank_before_the_next_step(mode):
    world = 3
    out = run(world, mode)
    for r in range(world - 1):
        res = out[r]
        assert res["steps"] == 2, res  # steps 0 and 1 completed with every rank
        msg, missing, left, step = res["error"]
        assert step == 2
        if mode == "leave":
            assert left == [world - 1] and res["seconds"] < 3.0, res  # announced: reported at once
        else:
            assert missing == [world - 1] and 2.5 < res["seconds"] < 10.0, res  # silent: reported at the deadline
        assert str(world - 1) in msg
