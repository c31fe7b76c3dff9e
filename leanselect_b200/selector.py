"""``LeanSelectSelector`` with the reference's API, computed by the B200 kernels.

Mirrors ``leanselect/selector.py:69-214``: same constructor arguments, the
same four canonical parameters (``head_mix [H, R]``, ``kv_head_mix [G, R]``,
``q_proj [R, D, r]``, ``k_proj [R, D, r]``), the same initialisation, the
same ``ValueError`` on bad shapes, and the methods ``fused_weights``,
``project_queries``, ``project_atom_keys`` and ``score_pages``.  The
methods run the CUDA library on CUDA tensors and raise on CPU tensors.

Numerics: the kernels compute in bf16 with fp32 accumulation.  For bf16
inputs this is the reference's own rounding (its ``fused_weights`` casts to
the query dtype and its bf16 ``einsum`` calls return bf16: projections and
atom scores alike).  fp32 inputs are rounded to bf16 at the boundary and
the results are returned in the input dtype.
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops

LEANSELECT_CANONICAL_TENSORS = ("head_mix", "kv_head_mix", "q_proj", "k_proj")


class LeanSelectSelector(nn.Module):
    """Low-rank router that emits one page plan per GQA group (selector.py:69)."""

    def __init__(self, *, num_heads: int, num_kv_heads: int, head_dim: int,
                 router_heads: int = 4, router_dim: int = 32) -> None:
        super().__init__()
        values = {
            "num_heads": int(num_heads),
            "num_kv_heads": int(num_kv_heads),
            "head_dim": int(head_dim),
            "router_heads": int(router_heads),
            "router_dim": int(router_dim),
        }
        if any(value <= 0 for value in values.values()):
            raise ValueError("all LeanSelect dimensions must be positive")
        if values["router_heads"] > values["num_heads"]:
            raise ValueError("router_heads cannot exceed num_heads")
        if values["num_heads"] % values["num_kv_heads"]:
            raise ValueError("num_heads must be divisible by num_kv_heads")
        for name, value in values.items():
            setattr(self, name, value)
        self.head_mix = nn.Parameter(torch.empty(self.num_heads, self.router_heads))
        self.kv_head_mix = nn.Parameter(torch.empty(self.num_kv_heads, self.router_heads))
        self.q_proj = nn.Parameter(torch.empty(self.router_heads, self.head_dim, self.router_dim))
        self.k_proj = nn.Parameter(torch.empty(self.router_heads, self.head_dim, self.router_dim))
        for parameter in self.parameters():
            parameter._is_indexer = True
        self._kernel_weights = None
        self._kernel_key = None
        self.reset_parameters()

    @classmethod
    def from_reference(cls, module: nn.Module) -> "LeanSelectSelector":
        """Wrap a reference ``LeanSelectSelector``, sharing its parameter tensors."""
        new = cls.__new__(cls)
        nn.Module.__init__(new)
        for name in ("num_heads", "num_kv_heads", "head_dim", "router_heads", "router_dim"):
            setattr(new, name, int(getattr(module, name)))
        for name in LEANSELECT_CANONICAL_TENSORS:
            setattr(new, name, getattr(module, name))
        new._kernel_weights = None
        new._kernel_key = None
        return new

    def reset_parameters(self) -> None:
        """Group-mean head mix and a scaled orthonormal frame (selector.py:112-137)."""
        with torch.no_grad():
            heads_per_group = self.num_heads // self.num_kv_heads
            self.head_mix.fill_(1.0 / heads_per_group)
            self.kv_head_mix.fill_(1.0)
            width = self.router_heads * self.router_dim
            if width <= self.head_dim:
                frame = torch.linalg.qr(torch.randn(self.head_dim, width, dtype=torch.float32),
                                        mode="reduced").Q
            else:
                frame = torch.linalg.qr(torch.randn(width, self.head_dim, dtype=torch.float32),
                                        mode="reduced").Q.T
            frame.mul_(self.head_dim ** -0.25)
            projection = frame.reshape(self.head_dim, self.router_heads,
                                       self.router_dim).permute(1, 0, 2)
            self.q_proj.copy_(projection)
            self.k_proj.copy_(projection)
        self._kernel_weights = None

    def canonical_state(self) -> dict[str, torch.Tensor]:
        return {name: getattr(self, name) for name in LEANSELECT_CANONICAL_TENSORS}

    # -- folded weights ---------------------------------------------------------------

    def fused_weights(self, *, dtype: torch.dtype | None = None):
        """``(q_fused [H, D, F], kv_fused [G, D, F])`` (selector.py:144-158)."""
        return ops.fold_weights(self.head_mix, self.kv_head_mix, self.q_proj, self.k_proj,
                                reference_layout=True, dtype=dtype)

    def kernel_weights(self) -> ops.FoldedWeights:
        """Folded bf16 weights in kernel layout, cached until a parameter changes."""
        params = [getattr(self, n) for n in LEANSELECT_CANONICAL_TENSORS]
        key = tuple((p.data_ptr(), p._version, p.device) for p in params)
        if self._kernel_weights is None or self._kernel_key != key:
            self._kernel_weights = ops.fold_weights(*params)
            self._kernel_key = key
        return self._kernel_weights

    # -- projections and scores ----------------------------------------------------

    def project_queries(self, query: torch.Tensor) -> torch.Tensor:
        if query.ndim != 3 or tuple(query.shape[1:]) != (self.num_heads, self.head_dim):
            raise ValueError("query must have shape [N, num_heads, head_dim]")
        out = ops.project_queries(query.detach(), self.kernel_weights().wq_t, self.num_kv_heads)
        return out if query.dtype == torch.bfloat16 else out.to(query.dtype)

    def project_atom_keys(self, compressed_keys: torch.Tensor) -> torch.Tensor:
        if compressed_keys.ndim != 3 or tuple(compressed_keys.shape[1:]) != (
                self.num_kv_heads, self.head_dim):
            raise ValueError("compressed_keys must have shape [A, num_kv_heads, head_dim]")
        out = ops.project_atom_keys(compressed_keys.detach(), self.kernel_weights().wk_t)
        return out if compressed_keys.dtype == torch.bfloat16 else out.to(compressed_keys.dtype)

    def score_pages(self, query: torch.Tensor, compressed_keys: torch.Tensor, *, seq_len: int,
                    block_size: int, kernel_stride: int) -> torch.Tensor:
        """Pooled page scores ``[G, N, ceil(seq_len/block_size)]`` (selector.py:192-214).

        As the reference: the page count follows ``seq_len`` (any number of
        query rows), page ``p`` pools the atoms of its window that exist,
        and pages without an atom are ``-inf``.
        """
        if query.ndim != 3 or tuple(query.shape[1:]) != (self.num_heads, self.head_dim):
            raise ValueError("query must have shape [N, num_heads, head_dim]")
        if compressed_keys.ndim != 3 or tuple(compressed_keys.shape[1:]) != (
                self.num_kv_heads, self.head_dim):
            raise ValueError("compressed_keys must have shape [A, num_kv_heads, head_dim]")
        if min(int(seq_len), int(block_size), int(kernel_stride)) <= 0:
            raise ValueError("page geometry must be positive")   # pages.py:163-164
        weights = self.kernel_weights()
        ks = ops.project_atom_keys(compressed_keys.detach(), weights.wk_t)
        pages = ops.score_pages_single(query.detach(), weights, ks, int(seq_len),
                                       block_size=int(block_size),
                                       kernel_stride=int(kernel_stride))
        return pages if query.dtype == torch.float32 else pages.to(query.dtype)
