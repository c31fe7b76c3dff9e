"""PyTorch custom operators over the C ABI (``torch.ops.leanselect_b200.*``).

The hot-path entry points registered with ``torch.library.custom_op``, each
with a fake (meta) implementation that gives the output shapes from the
inputs and integer arguments alone, so the ops can sit inside graphs that
``torch.compile`` / FakeTensor tracing walks (the reference wraps its CUDA
extension the same way, with fake-op shape functions for
``infllmv2_attn_varlen_func``).  The real implementations are the functions
of :mod:`leanselect_b200.ops`; on CPU tensors they raise (no fallback).

    out, lse = torch.ops.leanselect_b200.sparse_attn(q, k, v, cu_q, cu_k, max_q, max_k,
                                                     topk_idx, 0.0, True)
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import ops


@torch.library.custom_op("leanselect_b200::compress_keys", mutates_args=())
def compress_keys(k: Tensor, cu_seqlens_k: Tensor, total_c: int, kernel_size: int,
                  kernel_stride: int) -> tuple[Tensor, Tensor]:
    """``CompressK.forward`` (minicpm.py:1169-1185); ``total_c`` = number of atoms."""
    return ops.compress_keys(k, cu_seqlens_k, kernel_size=kernel_size, kernel_stride=kernel_stride,
                             total_c=total_c)


@compress_keys.register_fake
def _(k, cu_seqlens_k, total_c, kernel_size, kernel_stride):
    return (k.new_empty((total_c, k.shape[1], k.shape[2]), dtype=torch.bfloat16),
            cu_seqlens_k.new_empty(cu_seqlens_k.shape, dtype=torch.int32))


@torch.library.custom_op("leanselect_b200::project_atom_keys", mutates_args=())
def project_atom_keys(kc: Tensor, wk_t: Tensor) -> Tensor:
    """``project_atom_keys`` (selector.py:179-190): ``[A, G, D] -> [G, A, F]`` bf16."""
    return ops.project_atom_keys(kc, wk_t)


@project_atom_keys.register_fake
def _(kc, wk_t):
    return kc.new_empty((kc.shape[1], kc.shape[0], wk_t.shape[1]), dtype=torch.bfloat16)


def _weights(q: Tensor, wq_t: Tensor) -> ops.FoldedWeights:
    return ops.FoldedWeights(wq_t=wq_t, wk_t=None, num_heads=q.shape[1],
                             num_kv_heads=wq_t.shape[0], head_dim=q.shape[2],
                             width=wq_t.shape[1])


@torch.library.custom_op("leanselect_b200::select_pages", mutates_args=())
def select_pages(q: Tensor, wq_t: Tensor, ks: Tensor, cu_seqlens_q: Tensor, cu_seqlens_c: Tensor,
                 max_seqlen_q: int, take: int, init_blocks: int, local_blocks: int) -> Tensor:
    """Scoring + pooling + forced pages + top-T (minicpm.py:3093-3141): ``[G, total_q, take]``."""
    return ops.select_pages(q, _weights(q, wq_t), ks, cu_seqlens_q, cu_seqlens_c, max_seqlen_q,
                            take=take, init_blocks=init_blocks, local_blocks=local_blocks)


@select_pages.register_fake
def _(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, max_seqlen_q, take, init_blocks, local_blocks):
    return q.new_empty((wq_t.shape[0], q.shape[0], take), dtype=torch.int32)


@torch.library.custom_op("leanselect_b200::score_pages", mutates_args=())
def score_pages(q: Tensor, wq_t: Tensor, ks: Tensor, cu_seqlens_q: Tensor, cu_seqlens_c: Tensor,
                max_seqlen_q: int) -> Tensor:
    """``score_pages`` + max pooling (selector.py:192-214): ``[G, total_q, P]`` fp32."""
    return ops.score_pages(q, _weights(q, wq_t), ks, cu_seqlens_q, cu_seqlens_c, max_seqlen_q)


@score_pages.register_fake
def _(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, max_seqlen_q):
    pages = (max_seqlen_q + 63) // 64
    return q.new_empty((wq_t.shape[0], q.shape[0], pages), dtype=torch.float32)


@torch.library.custom_op("leanselect_b200::sparse_attn", mutates_args=())
def sparse_attn(q: Tensor, k: Tensor, v: Tensor, cu_seqlens_q: Tensor, cu_seqlens_k: Tensor,
                max_seqlen_q: int, max_seqlen_k: int, topk_idx: Tensor, softmax_scale: float,
                causal: bool) -> tuple[Tensor, Tensor]:
    """``infllmv2_attn_varlen_func(..., topk_idx=)`` (minicpm.py:3229-3243): ``(out, lse)``.

    ``softmax_scale`` 0 means ``head_dim**-0.5``.
    """
    return ops.sparse_attn(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           topk_idx, softmax_scale=softmax_scale or None, causal=causal,
                           return_lse=True)


@sparse_attn.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, topk_idx, softmax_scale,
      causal):
    return (torch.empty_like(q), q.new_empty((q.shape[1], q.shape[0]), dtype=torch.float32))


OPS = ("compress_keys", "project_atom_keys", "select_pages", "score_pages", "sparse_attn")

__all__ = list(OPS)
