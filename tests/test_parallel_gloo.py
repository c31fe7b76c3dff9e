"""Sequence-parallel host logic on CPU ranks (gloo, world size 2 and 4).

The partition, the all-gather + zig-zag reorder and the position bookkeeping
of ``leanselect_b200.parallel`` run with the gloo backend on the host; the
CUDA kernels are not involved.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from leanselect_b200.parallel import gather_sequence, local_positions, zigzag_chunks


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, seq_len, result_queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        full = torch.arange(seq_len * 3, dtype=torch.float32).reshape(seq_len, 3)
        pos = local_positions(seq_len, world, rank)
        local = full[pos]
        gathered = gather_sequence(local, seq_len)
        result_queue.put((rank, bool(torch.equal(gathered, full)), pos.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gather_restores_sequence_order(world):
    seq_len = 2 * world * 64 * 3
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq_len, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=60) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results)
    covered = sorted(x for _, _, pos in results for x in pos)
    assert covered == list(range(seq_len))


def test_zigzag_chunks_balance_causal_work():
    n, world = 131072, 8
    loads = []
    for r in range(world):
        chunks = zigzag_chunks(n, world, r)
        assert all(length == n // 16 for _, length in chunks)
        # Causal work of a chunk is proportional to the sum of its positions.
        loads.append(sum(s * length + length * (length - 1) / 2 for s, length in chunks))
    assert max(loads) / min(loads) < 1.0001
    assert zigzag_chunks(n, world, 0)[1][0] + n // 16 == n   # rank 0 holds the last token


def test_zigzag_rejects_unaligned_lengths():
    with pytest.raises(ValueError):
        zigzag_chunks(1000, 2, 0)
    with pytest.raises(ValueError):
        zigzag_chunks(1024, 2, 2)


def test_lpt_shards_cover_every_sequence_once_and_balance():
    from leanselect_b200.parallel import lpt_shards

    import numpy as np
    rng = np.random.default_rng(0)
    lengths = rng.integers(8192, 32769, 64).tolist()   # benchmark config 4
    shards = lpt_shards(lengths, 8)
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(64))
    loads = [sum(lengths[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lengths)
    assert max(loads) / (sum(lengths) / 8) < 1.05


def test_config4_budget_rule():
    from leanselect_b200.attention import config4_budget

    assert config4_budget(8192) == 12 + 3          # 128 pages -> 12
    assert config4_budget(32768) == 51 + 3         # 512 pages -> 51
    assert config4_budget(131072) == 64 + 3        # capped at 64


def test_config4_batch_lengths_are_seeded_and_in_range():
    from measure.batched import batch_lengths
    a, b = batch_lengths(64, 0), batch_lengths(64, 0)
    assert a == b and len(a) == 64
    assert all(8192 <= n <= 32768 for n in a)
    assert batch_lengths(64, 1) != a
