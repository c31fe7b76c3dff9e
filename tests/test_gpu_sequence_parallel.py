"""Sequence-parallel prefill across GPUs vs the single device (needs >= 2 B200).

Ranks are spawned processes on a NCCL group (NVLS off).

* The hot path of one layer, bit for bit: every rank builds the same
  full-sequence q/k/v from a seed, runs ``sequence_parallel_layer`` on its
  two zig-zag chunks (K/V all-gathered over NCCL, chunked selection and
  attention) and compares its own rows with ``prefill_layer_attention`` run
  on the whole sequence on its own GPU.  Selection and attention are
  row-independent, so each rank's ``topk_idx`` rows and attention rows must
  be identical.
* The whole model: token-local GEMMs run with different row counts on the
  two paths (cuBLAS may pick other tilings), so logits are compared with a
  tolerance (the one-rank case is bit-exact, test_gpu_host_model.py).
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


def _init(rank, world, port):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=120))
    return dist, dev


def _layer_worker(rank, world, port, n, topk, local, queue):
    dist, dev = _init(rank, world, port)
    try:
        import leanselect_b200 as lsb
        from leanselect_b200.parallel import local_positions, sequence_parallel_layer
        from measure.inputs import config1_layer, make_selector

        q, k, v = config1_layer(n, dev, 3)           # the same tensors on every rank
        sel = make_selector(dev, 3)
        cfg = lsb.LayerConfig(topk=topk, local_blocks=local)
        pos = local_positions(n, world, rank, device=dev)
        cap = {}
        out = sequence_parallel_layer(q[pos].contiguous(), k[pos].contiguous(),
                                      v[pos].contiguous(), n, sel, cfg, capture=cap)
        cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
        want, idx = lsb.prefill_layer_attention(q, k, v, cu, n, sel, cfg, lengths=[n],
                                                return_topk=True)
        torch.cuda.synchronize()
        lsb.ops.check_status(dev)
        same_idx = bool(torch.equal(cap["idx"], idx[:, pos]))
        same_out = bool(torch.equal(out, want[pos]))
        diff = int((cap["idx"] != idx[:, pos]).any(-1).sum().item())
        queue.put((rank, same_idx, same_out, diff))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _model_worker(rank, world, port, n, queue):
    dist, dev = _init(rank, world, port)
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


def _spawn(target, world, *args):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (queue,))
             for r in range(world)]
    for p in procs:
        p.start()
    return procs, queue


@pytest.mark.parametrize("n,topk,local", [(32768, 67, 2), (16384, 96, 32), (8192, 67, 2)])
def test_sequence_parallel_layer_is_bit_exact(n, topk, local):
    """Chunks of 8K and 4K tokens overlap the late K/V gather with the early
    chunk; 2K-token chunks gather everything first.  The stock budget (T=96,
    32 local pages) runs too."""
    world = min(torch.cuda.device_count(), 4)
    procs, queue = _spawn(_layer_worker, world, n, topk, local)
    results = [queue.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same_idx, same_out, diff in results:
        assert same_idx, (rank, diff)
        assert same_out, rank


@pytest.mark.parametrize("world,n", [(2, 16384), (2, 8192)])
def test_sequence_parallel_model_matches_single_device(world, n):
    procs, queue = _spawn(_model_worker, world, n)
    err, cos = queue.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert cos > 0.999, cos
    assert err < 0.05, err
