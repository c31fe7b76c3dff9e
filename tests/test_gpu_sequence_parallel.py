"""Sequence-parallel prefill across GPUs vs the single-device prefill (needs >= 2 B200).

Ranks are spawned processes on a NCCL group; rank 0 also runs the whole
prefill on its own GPU.  Token-local GEMMs run with different row counts on
the two paths, so logits are compared with a tolerance, not bit for bit
(the one-rank case is bit-exact, see test_gpu_host_model.py).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:  # pragma: no cover
    pytest.skip("needs at least two CUDA devices", allow_module_level=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shape():
    from leanselect_b200.model import MiniCPMShape

    return MiniCPMShape(vocab_size=1000, hidden_size=2048, intermediate_size=4096, num_layers=2,
                        num_heads=16, num_kv_heads=2, max_position=16384,
                        original_max_position=8192, router_heads=4, router_dim=32)


def _worker(rank, world, port, n, queue):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=120))
    try:
        from leanselect_b200.model import PrefillModel
        from leanselect_b200.parallel import SequenceParallelRunner

        ids = torch.randint(0, 1000, (n,), device=dev,
                            generator=torch.Generator(device=dev).manual_seed(11))
        sp = SequenceParallelRunner(_shape(), dev, seed=7)
        got = sp.prefill_device(ids, [n])
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            ref = PrefillModel(_shape(), dev, seed=7)
            want = ref.prefill(ids, torch.tensor([0, n], dtype=torch.int32, device=dev), [n])
            err = (got - want).abs().max().item() / want.abs().max().item()
            cos = torch.nn.functional.cosine_similarity(got.flatten(), want.flatten(), dim=0)
            queue.put((float(err), float(cos)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 16384), (2, 8192)])
def test_sequence_parallel_matches_single_device(world, n):
    """4096-token chunks overlap the late K/V gather with the early chunk;
    2048-token chunks gather everything first."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, queue)) for r in range(world)]
    for p in procs:
        p.start()
    err, cos = queue.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert cos > 0.999, cos
    assert err < 0.05, err
