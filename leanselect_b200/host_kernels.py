"""Torch wrappers of the benchmark host model's fused kernels (``ls_bb_*``).

See ``include/leanselect_b200_backbone.h``.  Like :mod:`leanselect_b200.ops`
these run on CUDA tensors only, on the current stream.
"""
from __future__ import annotations

import torch

from .ops import _call, _require_cuda, _stream


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dev = _require_cuda(x, weight)
    x = x.contiguous()
    out = torch.empty_like(x)
    _call(dev, "ls_bb_rms_norm", x.data_ptr(), weight.data_ptr(), x.numel() // x.shape[-1],
               x.shape[-1], float(eps), out.data_ptr(), _stream(dev))
    return out


def rope_split(qkv: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
               scaling: float, num_heads: int, num_kv_heads: int, head_dim: int = 128):
    """``qkv [N, (H+2G)*D]`` -> rotated ``q [N,H,D]``, ``k [N,G,D]`` and ``v [N,G,D]``."""
    dev = _require_cuda(qkv, positions, inv_freq)
    n = qkv.shape[0]
    qkv = qkv.contiguous()
    pos = positions.to(torch.int64).contiguous()
    inv = inv_freq.to(torch.float32).contiguous()
    q = torch.empty(n, num_heads, head_dim, dtype=qkv.dtype, device=dev)
    k = torch.empty(n, num_kv_heads, head_dim, dtype=qkv.dtype, device=dev)
    v = torch.empty(n, num_kv_heads, head_dim, dtype=qkv.dtype, device=dev)
    _call(dev, "ls_bb_rope_split", qkv.data_ptr(), pos.data_ptr(), inv.data_ptr(),
               float(scaling), n, num_heads, num_kv_heads, head_dim, q.data_ptr(), k.data_ptr(),
               v.data_ptr(), _stream(dev))
    return q, k, v


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(gate_up)
    gate_up = gate_up.contiguous()
    n, two_i = gate_up.shape
    out = torch.empty(n, two_i // 2, dtype=gate_up.dtype, device=dev)
    _call(dev, "ls_bb_silu_mul", gate_up.data_ptr(), n, two_i // 2, out.data_ptr(), _stream(dev))
    return out
