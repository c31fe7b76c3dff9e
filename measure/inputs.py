"""Seeded synthetic inputs of the benchmark configurations, generated on the device.

``config1_layer`` draws BASELINE config 0/1's distribution for one sequence:
N(0,1) q/k/v, 24 hot pages per KV head whose keys (and every query) are
shifted by 0.5*u; ``make_selector`` builds the selector of those configs
(a 32 x 4 router with an N(0, 1/32) head mix).  The same seed gives the same
tensors on every rank.  Used by the measurement drivers of this folder and
by the GPU tests.
"""
from __future__ import annotations

import math

import torch

from leanselect_b200 import LeanSelectSelector


def config1_layer(n: int, device: torch.device, seed: int = 0, num_heads: int = 32,
                  num_kv_heads: int = 2, head_dim: int = 128, hot_pages: int = 24,
                  hot_shift: float = 0.5):
    """benchmark config-0/1 distribution for one sequence of ``n`` tokens, on ``device``."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(n, num_heads, head_dim, device=device, generator=g)
    k = torch.randn(n, num_kv_heads, head_dim, device=device, generator=g)
    v = torch.randn(n, num_kv_heads, head_dim, device=device, generator=g)
    u = torch.randn(head_dim, device=device, generator=g)
    u /= u.norm()
    pages = (n + 63) // 64
    for kv in range(num_kv_heads):
        hot = torch.randperm(pages, device=device, generator=g)[:hot_pages]
        rows = (hot[:, None] * 64 + torch.arange(64, device=device)[None, :]).reshape(-1)
        rows = rows[rows < n]
        k[rows, kv] += hot_shift * u
    q += hot_shift * u
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def make_selector(device: torch.device, seed: int = 0, num_heads: int = 32,
                  num_kv_heads: int = 2) -> LeanSelectSelector:
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)  # the projections' own initialisation, identical on every rank
        sel = LeanSelectSelector(num_heads=num_heads, num_kv_heads=num_kv_heads, head_dim=128,
                                 router_heads=32, router_dim=4)
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        sel.head_mix.copy_(torch.randn(sel.head_mix.shape, generator=gen) / math.sqrt(32))
    return sel.to(device)
