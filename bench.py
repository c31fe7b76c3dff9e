"""Benchmark: 128K-token prefill of a random-init MiniCPM4.1-8B-shaped model.

The metric is prefill tokens/s at 128K for the 8B shape, with
LeanSelect selection and block-sparse attention on every layer; the hot path
(compress -> select -> sparse attention) is also reported as ms per layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--seq-len 131072] [--layers 32]

N=1 runs the whole model on one GPU.  N>1 (launched with torchrun) runs one
sequence-parallel prefill across the ranks (zig-zag token chunks, K/V
all-gathered per layer); ``value`` is then the whole job's tokens/s.
``--impl reference`` times the CPU restatement of the hot path (the oracle;
the reference's stage-2 kernel is CUDA-only and not distributed) on the
host cores and prints its own line.

One JSON line is printed by rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prefill tokens/sec @128K (8B shape); select+attn ms/layer"
# DRAM bytes (read + write) of one sparse-attention launch at 131072 tokens,
# from a committed ncu capture: ncu cannot run inside the timed bench, and a
# multi-pass capture of the 32-layer model would not fit the profiling rules.
ATTN_TRAFFIC_BYTES = 6750.0e6 + 1070.8e6
ATTN_TRAFFIC_SOURCE = (
    "ncu dram__bytes_read.sum + dram__bytes_write.sum of sparse_attn_kernel<16> at 131072 tokens "
    "(python -m measure.profile_case --seq-len 131072, the config-1 layer: same kernel, length "
    "and budget as one bench layer), one-pass capture; summary committed under profiles/")
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seq-len", type=int, default=131072)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-rows", type=int, default=48,
                    help="query rows per layer in the CPU baseline sample")
    return ap.parse_args()


def peaks():
    if PEAKS_FILE.exists():
        data = json.loads(PEAKS_FILE.read_text())
        return data, "measured"
    return FALLBACK_PEAKS, "fallback"


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = [line.split(",") for line in Path(self.file.name).read_text().splitlines()
                if line.strip()]
        os.unlink(self.file.name)
        sm, sm_max, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                sm_max = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": sm_max,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the hot path on the host cores
# ---------------------------------------------------------------------------

class CpuHotPath:
    """The oracle restatement of one layer's hot path on the host cores.

    Per-layer work runs once on the whole layer: compression of all keys,
    the selector's weight folding and the projection of every atom.  Per-row
    work -- the query projection, the row's atom scores, pooling, masking and
    top-k, and the row's sparse attention -- runs for ``rows`` query rows
    drawn from the last quarter of the sequence (where every row has its full
    page budget) and is scaled to all rows.  Input generation happens once,
    outside the timed steps.  Throughput is the hot path's tokens/s for
    ``layers`` layers (the dense backbone GEMMs are not included, which
    favours the CPU).
    """

    def __init__(self, seq_len: int, layers: int, rows: int, seed: int):
        from oracle import leanselect_oracle as ora

        self.ora = ora
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        self.seq_len, self.layers, self.rows = seq_len, layers, rows
        rng = np.random.default_rng(seed)
        self.sample = np.sort(rng.integers(seq_len - seq_len // 4, seq_len, rows))
        self.q, self.k, self.v, self.params = ora.synthetic_keys_and_sample(
            seq_len, self.sample, seed=seed)
        self.cu = np.array([0, seq_len], dtype=np.int32)
        self.last = None

    def step(self) -> float:
        ora, n = self.ora, self.seq_len
        t0 = time.perf_counter()
        kc, _ = ora.compress_keys(self.k, self.cu, policy="bf16")
        q_fused, kv_fused = ora.fold_weights(self.params, "bf16")
        ks = ora.project_atom_keys(kc, kv_fused, "bf16")
        t1 = time.perf_counter()
        qs = ora.project_queries(self.q, q_fused, self.params.num_kv_heads, "bf16")
        pages = ora.pool_atoms_to_pages(ora.atom_scores(qs, ks, "bf16"), n)
        sel = ora.select_from_scores(pages, self.sample, take=67)
        ora.attention_for_queries(self.q, self.sample, self.k, self.v, sel.topk_idx)
        t2 = time.perf_counter()
        per_layer = (t1 - t0) + (t2 - t1) * n / self.rows
        self.last = (t1 - t0, t2 - t1)
        return n / (per_layer * self.layers)

    def describe(self, value: float) -> dict:
        tl, tr = self.last
        return {
            "value": value, "unit": "tokens/s", "cores": self.cores, "kind": "port",
            "sample": (f"one {self.seq_len}-token layer of the oracle hot path: per-layer work "
                       f"(compression, weight folding, atom projection: {tl:.2f} s) once, plus "
                       f"per-row work (query projection, scores, top-k, attention) for "
                       f"{self.rows} query rows ({tr:.2f} s) scaled to {self.seq_len} rows; "
                       f"x {self.layers} layers; dense backbone not included"),
        }


def workload_config(n: int, layers: int, world: int) -> dict:
    """The ``config`` object of both arms' JSON lines (the same workload)."""
    from leanselect_b200.model import MiniCPMShape

    shape = MiniCPMShape.minicpm41_8b(num_layers=layers, max_position=max(n, 65536))
    return {
        "workload": f"random-init MiniCPM4.1-8B-shaped prefill, {n} tokens, batch 1, "
                    f"{layers} layers, LeanSelect T=67 (64 + sink + 2 local) pages of 64",
        "seq_len": n, "layers": layers, "hidden": shape.hidden_size,
        "heads": f"{shape.num_heads}/{shape.num_kv_heads}", "head_dim": shape.head_dim,
        "parallelism": f"sp{world}" if world > 1 else "single",
        "l2": "working set larger than L2 (16 GB of weights, >=1 GB activations per layer)",
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cpu = CpuHotPath(args.seq_len, args.layers, args.cpu_rows, args.seed)
    for _ in range(args.warmup):
        cpu.step()
    steps = [cpu.step() for _ in range(max(1, args.steps))]
    value = statistics.median(steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": len(steps), "warmup": args.warmup,
        "ms_per_step": args.seq_len / value * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args.seq_len, args.layers, args.gpus),
        "cpu_baseline": cpu.describe(value),
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def stage_roofline(shape, n: int, stage_ms: dict, attn_flops: float, pk: dict) -> dict:
    """Algorithmic work of each hot-path stage of one layer against its bound.

    Single sequence of ``n`` tokens; G KV groups, H heads, D = F = 128, page
    64, atoms A = (n - 32) // 16 + 1, pages P.  Compression moves K in and Kc
    out (HBM).  Selection computes the query projection (2 n H D F flops) and
    the causally reachable atom scores (about G F n A flops), and moves Q in,
    the pooled-score rows out and back (about G n P / 2 floats each way) and
    the page lists out (HBM).  Attention is the kernel of ``roofline``.  The
    stage times are the bench's own per-layer CUDA-event spans.
    """
    g, h, d = shape.num_kv_heads, shape.num_heads, shape.head_dim
    f = shape.router_heads * shape.router_dim
    atoms = (n - 32) // 16 + 1 if n >= 32 else 0
    pages = (n + 63) // 64
    take = min(shape.sparse.topk, pages)
    hbm = pk["hbm_gbs"] * 1e9
    tensor = pk["bf16_tflops_sustained"] * 1e12
    comp_bytes = (n + atoms) * g * d * 2
    sel_flops = 2.0 * n * h * d * f + g * f * n * atoms
    sel_bytes = n * h * d * 2 + 2 * (g * n * pages / 2) * 4 + g * n * take * 4
    t_c, t_s, t_a = (stage_ms[k] / 1e3 for k in ("compress", "select", "attn"))
    return {
        "compress": {"bound": "hbm", "bytes": comp_bytes, "achieved_gbs": comp_bytes / t_c / 1e9,
                     "frac": comp_bytes / t_c / hbm},
        "select": {"flops": sel_flops, "bytes": sel_bytes,
                   "achieved_tflops": sel_flops / t_s / 1e12, "tensor_frac": sel_flops / t_s / tensor,
                   "achieved_gbs": sel_bytes / t_s / 1e9, "hbm_frac": sel_bytes / t_s / hbm},
        "select_attn": {"flops": sel_flops + attn_flops,
                        "achieved_tflops": (sel_flops + attn_flops) / (t_s + t_a) / 1e12,
                        "tensor_frac": (sel_flops + attn_flops) / (t_s + t_a) / tensor},
        "peaks": "MEASURED_PEAKS.json hbm_gbs and bf16_tflops_sustained",
    }


def gather_roofline(runner, ids_dev, lengths, keys_last_layer: int, reps: int = 3,
                    warmup_pairs: int = 3) -> dict:
    """The attention kernel against its own data movement (measured roofline).

    Re-runs the last layer's attention call on the bench's own inputs next to
    ``ls_sparse_attn_gather_only``, which moves the same K/V pages from L2
    into shared memory with the same grid and TMA ring but does no math: the
    ratio is how close the kernel runs to the gather bound it cannot beat.
    Untimed by the bench's step clock (after the timed region).
    """
    from leanselect_b200 import ops

    cap = {}
    runner.prefill_device(ids_dev, lengths, capture=cap)
    q, k, v, idx, cu, max_len = (cap[x] for x in ("q", "k", "v", "idx", "cu", "max_len"))

    def attn():
        ops.sparse_attn(q, k, v, cu, cu, max_len, max_len, idx)

    def gather():
        ops.sparse_attn_gather_only(q, k, v, cu, cu, max_len, max_len, idx)

    # The two launches alternate so that both run at the same SM clock: right
    # after the model the power controller still holds the clock down, and it
    # takes ~100 ms to recover; the warm-up pairs cover that.
    for _ in range(warmup_pairs):
        attn()
        gather()
    times = {attn: [], gather: []}
    events = []
    for _ in range(reps):
        for fn in (attn, gather):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            events.append((fn, a, b))
    torch.cuda.synchronize()
    for fn, a, b in events:
        times[fn].append(a.elapsed_time(b))
    attn_ms = statistics.median(times[attn])
    gather_ms = statistics.median(times[gather])
    ops.check_status(q.device)
    gathered = keys_last_layer * 2 * q.shape[-1] * q.element_size()  # K and V rows
    return {"gathered_bytes": gathered, "attn_ms": attn_ms, "gather_only_ms": gather_ms,
            "achieved_tbs": gathered / (attn_ms / 1e3) / 1e12,
            "ceiling_tbs": gathered / (gather_ms / 1e3) / 1e12,
            "frac": gather_ms / attn_ms,
            "note": "L2 -> shared-memory page gather; ceiling = same launch with the math "
                    "removed; the two launches alternate (median of 3 each) at one clock"}


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    import leanselect_b200 as lsb
    from leanselect_b200.model import MiniCPMShape

    shape = MiniCPMShape.minicpm41_8b(num_layers=args.layers, max_position=max(args.seq_len, 65536))
    n = args.seq_len
    gen = torch.Generator().manual_seed(args.seed)
    ids_host = torch.randint(0, shape.vocab_size, (n,), generator=gen).pin_memory()

    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        from leanselect_b200.parallel import SequenceParallelRunner

        # NCCL's initialisation log (one line set per rank and channel) shows
        # how many ranks joined and over which transport.
        # A level below INFO (some machines preset VERSION or WARN) is raised
        # to INFO; an explicit INFO or TRACE is kept.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        runner = SequenceParallelRunner(shape, dev, seed=args.seed)
    else:
        dist = None
        from leanselect_b200.runner import PrefillRunner

        runner = PrefillRunner(shape, dev, seed=args.seed)

    def barrier():
        if dist is not None:
            dist.barrier()

    ids_dev = ids_host.to(dev)
    lengths = [n]
    # Instrumentation pass (untimed): attended keys per layer for the FLOP count.
    key_counts = []
    runner.prefill_device(ids_dev, lengths, key_counts=key_counts)
    for _ in range(args.warmup):
        runner.prefill_device(ids_dev, lengths)
    torch.cuda.synchronize()

    # K device-timed steps (inputs resident in HBM, CUDA events on the launching
    # stream) interleaved with K end-to-end steps through the public call
    # (pinned host ids -> host logits, wall clock), so that both see the same
    # clocks; every step is bracketed by a barrier and a synchronize.
    timers = []
    stream = torch.cuda.current_stream(dev)
    dev_ms, e2e_wall = 0.0, 0.0
    with ClockSampler(local_rank) as clocks:
        for _ in range(args.steps):
            barrier()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            runner.prefill_device(ids_dev, lengths, timers=timers)
            end.record(stream)
            torch.cuda.synchronize()
            barrier()
            dev_ms += start.elapsed_time(end)
            barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            logits = runner(ids_host, lengths)
            torch.cuda.synchronize()
            barrier()
            e2e_wall += time.perf_counter() - t0
    ms_total, e2e_total = dev_ms, e2e_wall
    if dist is not None:
        t = torch.tensor([ms_total, e2e_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total, e2e_total = float(t[0].item()), float(t[1].item())
    ms_step = ms_total / args.steps
    value = n / (ms_step / 1e3)
    e2e_s = e2e_total / args.steps

    # "gather": the visible part of the K/V all-gather (sequence-parallel only).
    stage = {"compress": [], "select": [], "attn": [], "gather": []}
    for name, a, b in timers:
        stage[name].append(a.elapsed_time(b))

    d2h = logits.numel() * logits.element_size() if rank == 0 else 0

    pk, pk_kind = peaks()
    layers = len(key_counts)
    hg = shape.num_heads // shape.num_kv_heads
    # Per layer of this rank: one attention launch on a single GPU, two (the
    # early and the late zig-zag chunk) when sequence-parallel; stage spans
    # are summed per layer.
    layer_steps = max(1, args.steps * layers)
    stage_ms = {k: sum(v) / layer_steps for k, v in stage.items() if v}
    flops_per_layer = 4 * shape.head_dim * hg * (sum(key_counts) / max(layers, 1))
    attn_ms = stage_ms.get("attn", float("nan"))
    achieved = flops_per_layer / (attn_ms / 1e3) / 1e12
    peak = pk["bf16_tflops_sustained"]
    # Our kernels per layer: per query chunk (one on a single GPU, two zig-zag
    # chunks per rank when sequence-parallel) compressed seqlens, compression,
    # key projection, scoring, top-k and sparse attention; plus the host
    # model's fused RMSNorm (2 + MLP chunks), RoPE and SiLU kernels.
    chunks = 1 if world == 1 else 2
    mlp_chunks = -(-(n // world) // 16384)
    launches_per_layer = 6 * chunks + (1 + 2 * mlp_chunks + 1)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform random token ids, random-init weights)",
        "config": workload_config(n, args.layers, world),
        "select_attn_ms_per_layer": stage_ms["select"] + attn_ms + stage_ms["compress"],
        "stage_ms_per_layer": stage_ms,
        "kv_gather_ms_per_layer": stage_ms.get("gather"),
        "e2e": {"value": n / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": n * 8,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_layer * layers * args.steps,
        "roofline": {
            "kernel": "sparse_attn_kernel",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "peak_kind": f"{pk_kind} (bf16 dense, sustained)",
            "flops_per_layer": flops_per_layer,
            "attn_launches_per_layer": chunks,
            # The capture is of one single-GPU 128K launch; a rank's chunk
            # launches are smaller, so no per-launch figure is claimed there.
            "traffic": ATTN_TRAFFIC_BYTES if world == 1 else None,
            "traffic_source": ATTN_TRAFFIC_SOURCE if world == 1 else None,
        },
        "clocks": clocks.summary(),
    }
    if world == 1:
        line["roofline"]["l2_gather"] = gather_roofline(runner, ids_dev, lengths, key_counts[-1])
        line["stage_roofline"] = stage_roofline(shape, n, stage_ms, flops_per_layer, pk)
    if rank == 0 and world == 1:
        cpu = CpuHotPath(n, args.layers, args.cpu_rows, args.seed)
        line["cpu_baseline"] = cpu.describe(cpu.step())
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
