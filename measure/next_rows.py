"""Timings of the rows next to the prefill path on one GPU, one JSON line each.

* f1 ``compress_dual``: both compressions a prefill leaves in the decode
  cache (32/16 and 128/64, minicpm.py:2785-2792) from one pass over K,
  against the two separate compression launches.
* f2 ``atom_scores``: NOSA's raw LeanSelect atom scores (nosa.py:1822-1853).
* f4 ``decode_attention``: one decode step of sparse attention (one query
  per sequence against a 128K-token cache, T = 67 random pages per row),
  one CTA per (token, group) against page lists cut into slices; also
  device time per step from CUDA-graph replays of 16 steps (no host gaps).

Seeded synthetic inputs (the benchmark layer's distribution); CUDA events on
the launching stream, median of ``--reps``; the L2 is flushed (a 256 MB
write) before every timed call, so each call reads its inputs from HBM.

Usage: ``python -m measure.next_rows [--reps 10] [--small]``

``--small`` runs each call once on reduced sizes (f1 at 32K keys, f2 at 8K
tokens, f4 at batch 1 on 32K caches): the workload for profiler captures.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from leanselect_b200 import ops
from measure.inputs import config1_layer, make_selector

DEV = torch.device("cuda", 0)


def timed(fn, reps: int, flush: torch.Tensor) -> float:
    fn()
    times = []
    for _ in range(reps):
        flush.fill_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def peaks():
    import pathlib
    p = pathlib.Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--small", action="store_true", help="one call each, reduced sizes")
    args = ap.parse_args(argv)
    if args.small:
        return small()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=DEV)
    hbm, hbm_kind = peaks()

    # f1: 128K keys, both compressions.
    n = 131072
    q, k, v = config1_layer(n, DEV, 0)
    cu = torch.tensor([0, n], dtype=torch.int32, device=DEV)
    sep = timed(lambda: (ops.compress_keys(k, cu, lengths=[n]),
                         ops.compress_keys(k, cu, kernel_size=128, kernel_stride=64, lengths=[n])),
                args.reps, flush)
    dual = timed(lambda: ops.compress_keys_dual(k, cu, lengths=[n]), args.reps, flush)
    a1, a2 = ops.atom_count(n), ops.atom_count(n, 128, 64)
    nbytes = 2 * 2 * 128 * (n + a1 + a2)
    print(json.dumps({"row": "f1", "what": "compress_dual", "tokens": n, "separate_ms": sep,
                      "dual_ms": dual, "algorithmic_bytes": nbytes,
                      "dual_gbs": nbytes / dual / 1e6, "hbm_frac": nbytes / dual / 1e6 / hbm,
                      "peak": f"{hbm_kind} hbm_gbs {hbm}"}), flush=True)

    # f2: atom scores of a 32K-token sequence.
    n2 = 32768
    q2, k2, _ = config1_layer(n2, DEV, 1)
    cu2 = torch.tensor([0, n2], dtype=torch.int32, device=DEV)
    w = make_selector(DEV, 1).kernel_weights()
    kc2, cu_c2 = ops.compress_keys(k2, cu2, lengths=[n2])
    ks2 = ops.project_atom_keys(kc2, w.wk_t)
    atoms = kc2.shape[0]
    t2 = timed(lambda: ops.atom_scores(q2, w, ks2, cu2, cu_c2, n2, atoms), args.reps, flush)
    out_bytes = 2 * n2 * atoms * 2
    flops = 2 * n2 * 32 * 128 * 128 + 2 * 2 * n2 * atoms * 128
    print(json.dumps({"row": "f2", "what": "atom_scores", "tokens": n2, "atoms": atoms,
                      "ms": t2, "out_bytes": out_bytes, "out_gbs": out_bytes / t2 / 1e6,
                      "hbm_frac": (out_bytes + q2.numel() * 2) / t2 / 1e6 / hbm,
                      "tflops": flops / t2 / 1e9}), flush=True)
    del q, k, v, q2, k2

    # f4: decode steps against 128K-token caches.
    cache = 131072
    pages = cache // 64
    gen = torch.Generator(device="cpu").manual_seed(7)
    for batch in (1, 8, 64):
        kk = torch.randn(batch * cache, 2, 128, device=DEV, dtype=torch.bfloat16)
        vv = torch.randn_like(kk)
        qq = torch.randn(batch, 32, 128, device=DEV, dtype=torch.bfloat16)
        idx = torch.stack([torch.randperm(pages, generator=gen)[:67]
                           for _ in range(2 * batch)]).view(2, batch, 67)
        idx = idx.to(torch.int32).to(DEV)
        cu_q = torch.arange(batch + 1, dtype=torch.int32, device=DEV)
        cu_k = torch.arange(batch + 1, dtype=torch.int32, device=DEV) * cache

        def step(splits):
            return ops.sparse_attn(qq, kk, vv, cu_q, cu_k, 1, cache, idx, causal=False,
                                   splits=splits)

        auto = ops.attn_splits(2 * batch, 1, cache, 67, DEV)
        t_one = timed(lambda: step(1), args.reps, flush)
        t_split = timed(lambda: step(None), args.reps, flush)
        # Device time without host launch gaps: 16 steps captured in a CUDA
        # graph and replayed (caches stay in L2 between the steps here).
        graph_us = {}
        for name, sp in (("one_cta_per_row", 1), ("split", auto)):
            step(sp)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(16):
                    step(sp)
            graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(4):
                graph.replay()
            b.record()
            torch.cuda.synchronize()
            graph_us[name] = a.elapsed_time(b) * 1e3 / 64
            del graph
        gathered = 2 * batch * 67 * 64 * 512
        print(json.dumps({"row": "f4", "what": "decode_attention", "batch": batch,
                          "cache_tokens": cache, "topk": 67, "one_cta_per_row_ms": t_one,
                          "split_ms": t_split, "splits": auto,
                          "graph_us_per_step": graph_us, "gathered_bytes": gathered,
                          "split_gbs": gathered / t_split / 1e6,
                          "hbm_frac": gathered / t_split / 1e6 / hbm}), flush=True)
        del kk, vv
    assert ops.check_status(DEV) == 0
    return 0


def small() -> int:
    """One call of each kernel on reduced inputs (for profiler captures)."""
    n = 32768
    _, k, _ = config1_layer(n, DEV, 0)
    cu = torch.tensor([0, n], dtype=torch.int32, device=DEV)
    ops.compress_keys_dual(k, cu, lengths=[n])
    n2 = 8192
    q2, k2, _ = config1_layer(n2, DEV, 1)
    cu2 = torch.tensor([0, n2], dtype=torch.int32, device=DEV)
    w = make_selector(DEV, 1).kernel_weights()
    kc2, cu_c2 = ops.compress_keys(k2, cu2, lengths=[n2])
    ks2 = ops.project_atom_keys(kc2, w.wk_t)
    ops.atom_scores(q2, w, ks2, cu2, cu_c2, n2, kc2.shape[0])
    cache = 32768
    gen = torch.Generator(device="cpu").manual_seed(7)
    kk = torch.randn(cache, 2, 128, device=DEV, dtype=torch.bfloat16)
    vv = torch.randn_like(kk)
    qq = torch.randn(1, 32, 128, device=DEV, dtype=torch.bfloat16)
    idx = torch.stack([torch.randperm(cache // 64, generator=gen)[:67] for _ in range(2)])
    idx = idx.view(2, 1, 67).to(torch.int32).to(DEV)
    cu_q = torch.tensor([0, 1], dtype=torch.int32, device=DEV)
    cu_k = torch.tensor([0, cache], dtype=torch.int32, device=DEV)
    ops.sparse_attn(qq, kk, vv, cu_q, cu_k, 1, cache, idx, causal=False)
    torch.cuda.synchronize()
    assert ops.check_status(DEV) == 0
    print("next_rows small ok", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
