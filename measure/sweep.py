"""Sequence-length sweep of one hot-path layer (benchmark config 3).

    python -m measure.sweep [--lengths 32768,65536,131072,262144,524288] [--reps 3]
                                    [--method leanselect|uniform] [--topk 67 --local 2]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m measure.sweep ...            # sequence-parallel over N GPUs

One benchmark config-1 layer (bf16, 32 query / 2 KV heads, head_dim 128,
budget 64 pages + sink + 2 local pages of 64 tokens; ``--topk 96 --local
32`` is the reference's stock budget, window 2048) at each length, with
the config-0/1 input distribution: N(0,1) q/k/v, 24 hot pages per KV head
whose keys (and every query) are shifted by 0.5*u, selector head mix
N(0, 1/32) over a 32 x 4 router.  Inputs are generated on the device from
the seed, identically on every rank.  With N ranks the layer runs
sequence-parallel exactly as in the model (zig-zag query chunks, K/V
all-gathered over NCCL, chunked selection and attention).

Prints one JSON line per length: the device time of each stage (CUDA
events, median over ``--reps``, max over ranks) — K/V all-gather,
compression, selection (scoring + top-k), sparse attention — and the
layer's tokens/s.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from leanselect_b200 import ops
from leanselect_b200.attention import LayerConfig, prefill_layer_attention

from .inputs import config1_layer, make_selector

STAGES = ("gather", "compress", "select", "attn")


def run_length(n: int, reps: int, device: torch.device, dist=None, seed: int = 0,
               method: str = "leanselect", topk: int = 67, local: int = 2) -> dict:
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    if method != "leanselect" and world > 1:
        raise ValueError("the sequence-parallel layer serves the LeanSelect method only")
    cfg = LayerConfig(topk=topk, local_blocks=local, selection_method=method)
    q, k, v = config1_layer(n, device, seed)
    sel = make_selector(device, seed)
    if world > 1:
        from leanselect_b200.parallel import sequence_parallel_layer, zigzag_chunks

        chunks = zigzag_chunks(n, world, rank)
        q = torch.cat([q[a:a + c] for a, c in chunks]).contiguous()
        k = torch.cat([k[a:a + c] for a, c in chunks]).contiguous()
        v = torch.cat([v[a:a + c] for a, c in chunks]).contiguous()

        def step(timers):
            return sequence_parallel_layer(q, k, v, n, sel, cfg, None, timers=timers)
    else:
        cu = torch.tensor([0, n], dtype=torch.int32, device=device)

        def step(timers):
            return prefill_layer_attention(q, k, v, cu, n, sel, cfg, lengths=[n], timers=timers)

    step(None)  # warm-up (also builds the selector's folded weights)
    per_stage = {s: [] for s in STAGES}
    totals = []
    for _ in range(reps):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        timers = []
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step(timers)
        b.record()
        torch.cuda.synchronize()
        totals.append(a.elapsed_time(b))
        spans = {s: 0.0 for s in STAGES}
        for name, e0, e1 in timers:
            spans[name] += e0.elapsed_time(e1)  # a stage may run as several spans
        for name, ms in spans.items():
            per_stage[name].append(ms)
    ops.check_status(device)
    ms = {s: (statistics.median(v) if v else 0.0) for s, v in per_stage.items()}
    ms["total"] = statistics.median(totals)
    if dist is not None:
        t = torch.tensor([ms[s] for s in (*STAGES, "total")], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = dict(zip((*STAGES, "total"), t.tolist()))
    return {"workload": f"benchmark config 3: config-1 layer (bf16, 32/2 heads, T={topk}, "
                        f"{local} local pages)",
            "method": method, "seq_len": n, "n_gpus": world, "reps": reps, "ms": ms,
            "tokens_per_s": n / (ms["total"] / 1e3),
            "parallelism": f"sp{world}" if world > 1 else "single"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--lengths", default="32768,65536,131072,262144,524288")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--method", choices=("leanselect", "uniform"), default="leanselect",
                    help="selection method (uniform: the mean-query ablation, one GPU)")
    ap.add_argument("--topk", type=int, default=67, help="pages per (group, token), T")
    ap.add_argument("--local", type=int, default=2, help="local pages before the query's own")
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
        for n in (int(x) for x in args.lengths.split(",")):
            line = run_length(n, args.reps, device, dist, args.seed, args.method, args.topk,
                              args.local)
            if dist is None or dist.get_rank() == 0:
                print(json.dumps(line), flush=True)
            torch.cuda.empty_cache()
    finally:
        if dist is not None:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
