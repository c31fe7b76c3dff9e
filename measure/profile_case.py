"""One layer of the hot path on synthetic inputs, for profilers.

    python -m measure.profile_case [--seq-len 32768] [--topk 67] [--repeat 1]

Builds benchmark config-1-shaped inputs (32 query / 2 KV heads, head_dim 128,
N(0,1) q/k/v, selector with a 32x4 router) on ``cuda:0`` and runs
compression -> key projection -> fused scoring + top-k -> sparse attention
``--repeat`` times, then checks the device status word.  Meant to be run
under ``ncu`` with a kernel filter; it prints one line and exits 0.
"""
from __future__ import annotations

import argparse

import torch

from leanselect_b200 import LeanSelectSelector, ops


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--topk", type=int, default=67)
    ap.add_argument("--repeat", type=int, default=1)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    n = args.seq_len
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(n, 32, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(n, 2, 128, device=dev, generator=g).bfloat16()
    v = torch.randn(n, 2, 128, device=dev, generator=g).bfloat16()
    sel = LeanSelectSelector(num_heads=32, num_kv_heads=2, head_dim=128, router_heads=32,
                             router_dim=4).to(dev)
    cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
    w = sel.kernel_weights()
    take = min(args.topk, (n + 63) // 64)
    for _ in range(args.repeat):
        kc, cu_c = ops.compress_keys(k, cu, lengths=[n])
        ks = ops.project_atom_keys(kc, w.wk_t)
        idx = ops.select_pages(q, w, ks, cu, cu_c, n, take=take)
        ops.sparse_attn(q, k, v, cu, cu, n, n, idx)
    torch.cuda.synchronize()
    ops.check_status(dev)
    print(f"profile_case ok: seq_len={n} take={take} repeat={args.repeat}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
