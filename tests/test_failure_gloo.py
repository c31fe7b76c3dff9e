"""Failure detection of the multi-rank prefill on CPU ranks (gloo, no GPU).

A rank fails on the host, between steps, in the three ways the runners must
survive: it exits, it stalls past the presence limit, or it raises.  The
surviving ranks must raise ``RankFailure`` naming it before their next step
instead of waiting forever (the reference trainer's per-step presence
all-reduce and error broadcast, train.py:270-275, 140, play the same role).
A collective issued after a peer died must end with an error too, bounded by
the process group's timeout.
"""
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from leanselect_b200.parallel import RankFailure, StepPresence, gather_sequence, local_positions


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exit(queue):
    """Flush what was put on the queue, then leave without any teardown."""
    queue.close()
    queue.join_thread()
    os._exit(0)


def _worker(rank, world, port, mode, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    presence = StepPresence(timeout_s=2.0)
    seq_len = 2 * world * 64
    local = torch.arange(seq_len, dtype=torch.float32)[local_positions(seq_len, world, rank)]
    presence.arrive()                              # step 0: everyone is here
    gather_sequence(local, seq_len)
    failing = rank == world - 1 if mode != "store_host_exits" else rank == 0
    if failing:
        if mode in ("exit", "store_host_exits"):
            queue.put((rank, "left", None, 0.0))
            _exit(queue)                           # leaves between steps, no goodbye
        if mode == "stall":
            queue.put((rank, "stalling", None, 0.0))
            time.sleep(6.0)
            _exit(queue)
        if mode == "raise":
            queue.put((rank, "raised", None, 0.0))
            try:
                raise ValueError("injected failure on the host")
            finally:
                _exit(queue)
    t0 = time.monotonic()
    try:
        presence.arrive()                          # step 1
        queue.put((rank, "no error", None, time.monotonic() - t0))
    except RankFailure as exc:
        queue.put((rank, "RankFailure", exc.missing, time.monotonic() - t0))
    # A collective with the failed peer gone ends with an error, not a hang.
    if mode == "exit":
        t0 = time.monotonic()
        try:
            gather_sequence(local, seq_len)
            queue.put((rank, "collective ok", None, time.monotonic() - t0))
        except Exception as exc:  # gloo raises on a closed peer or at the timeout
            queue.put((rank, "collective error", type(exc).__name__, time.monotonic() - t0))
    _exit(queue)


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.monotonic() + 90
    expected = {"exit": world + world - 1, "stall": world, "raise": world,
                "store_host_exits": world}[mode]
    while len(results) < expected and time.monotonic() < deadline:
        try:
            results.append(queue.get(timeout=5))
        except Exception:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            pytest.fail(f"{mode}: a surviving rank hung")
    return results


@pytest.mark.parametrize("mode", ["exit", "stall", "raise"])
def test_survivor_raises_naming_the_failed_rank(mode):
    results = _run(mode)
    failures = [r for r in results if r[1] == "RankFailure"]
    assert len(failures) == 1, results
    rank, _, missing, waited = failures[0]
    assert rank == 0 and missing == [1]
    assert 1.5 <= waited < 10.0, waited          # the 2 s presence limit, not a hang
    if mode == "exit":
        coll = [r for r in results if r[1].startswith("collective")]
        assert coll and coll[0][1] == "collective error" and coll[0][3] < 30.0, coll


def test_store_host_exit_is_reported_not_waited_on():
    """Rank 0 hosts the key-value store; when it leaves, the other rank's
    presence check fails on the store connection and raises."""
    results = _run("store_host_exits")
    failures = [r for r in results if r[1] == "RankFailure"]
    assert len(failures) == 1 and failures[0][0] == 1, results
    assert failures[0][3] < 10.0


def test_presence_counts_steps_and_accepts_all_ranks():
    """World of one: every step is complete at once."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(free_port()))
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=5))
    try:
        presence = StepPresence(timeout_s=1.0)
        assert [presence.arrive() for _ in range(3)] == [0, 1, 2]
    finally:
        dist.destroy_process_group()
