"""Batched small-model prefill, data-parallel (benchmark config 4).

    python -m measure.batched [--sequences 64] [--steps 2] [--warmup 1]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m measure.batched ...          # data-parallel over N GPUs

Random-init 24-layer model (hidden 2048, 16 query / 2 KV heads, head_dim
128), a batch of ``--sequences`` sequences of uniform-random token ids with
lengths drawn uniformly from [8K, 32K] (seeded), LeanSelect on every layer
with the per-sequence budget min(64, pages // 10) + sink + 2 local pages.
Sequences are sharded over the ranks longest-first (LPT) and every rank
prefills its shard as one packed varlen batch; ranks exchange no data.

Prints one JSON line: aggregate tokens/s of the whole batch over all ranks
(device time per step, max over ranks), per-rank token counts and the
device time of the hot-path stages summed over layers.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from leanselect_b200.attention import LayerConfig, config4_budget
from leanselect_b200.model import MiniCPMShape
from leanselect_b200.parallel import DataParallelRunner, lpt_shards


def batch_lengths(sequences: int, seed: int, lo: int = 8192, hi: int = 32768) -> list[int]:
    gen = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (sequences,), generator=gen)]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--sequences", type=int, default=64)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))
    try:
        cfg = LayerConfig(topk=67, per_sequence_topk=config4_budget)
        shape = MiniCPMShape.small_24l(num_layers=args.layers, sparse=cfg)
        lengths = batch_lengths(args.sequences, args.seed)
        gen = torch.Generator().manual_seed(args.seed + 1)
        ids = torch.randint(0, shape.vocab_size, (sum(lengths),), generator=gen).to(device)
        runner = DataParallelRunner(shape, device, seed=args.seed)
        rank = runner.rank
        mine = lpt_shards(lengths, runner.world)[rank]
        for _ in range(args.warmup):
            runner.prefill_device(ids, lengths)
        torch.cuda.synchronize()
        ms = 0.0
        for _ in range(args.steps):
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            runner.prefill_device(ids, lengths)
            b.record()
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            ms += a.elapsed_time(b)
        tokens_mine = sum(lengths[i] for i in mine)
        counts = [tokens_mine]
        if dist is not None:
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            c = torch.tensor([tokens_mine], device=device, dtype=torch.int64)
            gathered = [torch.zeros_like(c) for _ in range(world)]
            dist.all_gather(gathered, c)
            counts = [int(x.item()) for x in gathered]
        ms_step = ms / args.steps
        if rank == 0:
            total = sum(lengths)
            print(json.dumps({
                "metric": "batched prefill tokens/sec (benchmark config 4)",
                "value": total / (ms_step / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "scaling": "strong", "dtype": "bf16",
                "data": "synthetic (uniform random token ids, random-init weights)",
                "config": {"workload": f"{args.sequences} sequences, lengths U[8K, 32K] "
                                       f"(seed {args.seed}), {args.layers} layers, hidden 2048, "
                                       "16/2 heads, T = min(64, pages // 10) + 3",
                           "tokens": total, "parallelism": f"dp{world}",
                           "tokens_per_rank": counts}}), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
