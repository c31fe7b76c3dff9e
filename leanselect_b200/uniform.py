"""The uniform selection method (the matched ablation of LeanSelect) on B200.

Mirrors ``leanselect.ops.uniform`` (ops/uniform.py): ``uniform_prefill_topk_idx``
scores compressed keys with the mean query of each GQA group
(``uniform_group_queries``, pages.py:62-71; ``uniform_varlen_stage1``,
head_mix.py:80-170), pools atoms into pages, forces sink and local pages and
takes the top pages.  On B200 this is the LeanSelect scoring kernel with a
special folded weight (1/Hg on each head block's diagonal) and the
compressed keys as the atom keys, plus the uniform rules in its epilogue and
in the top-k kernel (``ls_uniform_select_pages``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from . import ops

DEFAULT_BLOCK_SIZE = 64
DEFAULT_KERNEL_STRIDE = 16
DEFAULT_INIT_BLOCKS = 1
DEFAULT_LOCAL_BLOCKS = 32


@dataclass
class SelectionDiagnostics:
    """Profiling metadata (uniform.py:61-65)."""

    extra: dict[str, Any] = field(default_factory=dict)


def uniform_prefill_topk_idx(q_unpad: torch.Tensor, k_compressed: torch.Tensor, *,
                             cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                             max_seqlen_q: int, topk: int, block_size: int = DEFAULT_BLOCK_SIZE,
                             kernel_stride: int = DEFAULT_KERNEL_STRIDE,
                             init_blocks: int = DEFAULT_INIT_BLOCKS,
                             local_blocks: int = DEFAULT_LOCAL_BLOCKS,
                             q_lengths=None):
    """``uniform_prefill_topk_idx`` (uniform.py:185-320): ``(topk_idx, diagnostics)``.

    ``topk_idx`` is ``[G, total_q, min(topk, max_pages)]`` int32.  Each row
    lists sink pages, selected pages and local pages in ascending order, then
    ``-1`` (the reference lists them by score; the sets are the same).
    Raises ``ValueError`` like the reference for non-3D inputs and for query
    lengths <= 1.  ``q_lengths`` (host list) avoids reading ``cu_seqlens_q``
    back to the host.
    """
    if q_unpad.ndim != 3 or k_compressed.ndim != 3:
        raise ValueError("q_unpad and k_compressed must be 3D")
    lengths = list(q_lengths) if q_lengths is not None else ops.host_lengths(cu_seqlens_q)
    if not lengths or min(lengths) <= 1:
        raise ValueError("Uniform is prefill-only; decode must use vanilla Sparse")
    block = int(block_size)
    max_pages = max((n + block - 1) // block for n in lengths)
    take = min(int(topk), max_pages)
    idx = ops.uniform_select_pages(q_unpad, k_compressed, cu_seqlens_q, cu_seqlens_k,
                                   int(max(lengths)), take=take, init_blocks=int(init_blocks),
                                   local_blocks=int(local_blocks), block_size=block,
                                   kernel_stride=int(kernel_stride))
    return idx, SelectionDiagnostics(extra={
        "selector_phase": "prefill",
        "prefill_impl": "b200_mean_mix_score_pool_topk",
        "uniform_prefill_head_mix": "uniform",
    })
