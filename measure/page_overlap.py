"""How much neighbouring tokens' page lists overlap (the benchmark layer).

    python -m measure.page_overlap [--seq-len 131072]

Runs the LeanSelect selection of one config-1 layer (T = 67) on the GPU and
prints, for groups of 1, 2, 4, ... 64 consecutive query tokens (past the
first 8192), the size of the union of their page lists as a fraction of the
lists' total, and the mean union size: how many distinct pages a CTA serving
that many tokens would gather.
"""
from __future__ import annotations

import argparse
import json

import torch

from leanselect_b200 import ops
from measure.inputs import config1_layer, make_selector


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--seq-len", type=int, default=131072)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    n = args.seq_len
    q, k, _ = config1_layer(n, dev, 0)
    w = make_selector(dev, 0).kernel_weights()
    cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
    kc, cu_c = ops.compress_keys(k, cu, lengths=[n])
    ks = ops.project_atom_keys(kc, w.wk_t)
    idx = ops.select_pages(q, w, ks, cu, cu_c, n, take=67)   # [2, n, 67]
    pages = (n + 63) // 64
    start = min(8192, n // 2)
    for tt in (1, 2, 4, 8, 16, 32, 64):
        total, union, groups = 0, 0, 0
        for g in range(idx.shape[0]):
            usable = (n - start) // tt * tt
            rows = idx[g, start:start + usable].reshape(-1, tt * idx.shape[2]).long()
            seen = torch.zeros(rows.shape[0], pages + 1, dtype=torch.bool, device=dev)
            seen.scatter_(1, torch.where(rows < 0, pages, rows), True)
            union += int(seen[:, :pages].sum().item())
            total += int((rows >= 0).sum().item())
            groups += rows.shape[0]
        print(json.dumps({"tokens_per_group": tt, "union_over_total": union / total,
                          "mean_union_pages": union / groups, "seq_len": n}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
