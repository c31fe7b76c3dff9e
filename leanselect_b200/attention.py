"""Drop-in replacements for the MiniCPM InfLLM-v2 hot-path call sites.

* :class:`CompressK` -- ``CompressK`` (minicpm.py:1158-1185).
* :func:`lightweight_compressed_attention` -- the LeanSelect branch of
  ``MiniCPMInfLLMv2Attention._lightweight_compressed_attention``
  (minicpm.py:3061-3142), same arguments, result and errors.
* :func:`infllmv2_attn_varlen_func` -- the stage-2 call
  ``infllm_v2.infllmv2_attn_varlen_func(..., topk_idx=)`` (minicpm.py:3229-3243).
* :func:`prefill_layer_attention` -- the whole prefill hot path of one layer
  (compress -> select -> sparse attention) for callers that hold the
  post-RoPE q/k/v directly.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
from torch import nn

from . import ops
from .selector import LeanSelectSelector


class CompressK(nn.Module):
    """Mean-pool compression of keys (minicpm.py:1158-1185) on the GPU."""

    def __init__(self, head_num_k: int, head_dim: int, kernel_size: int, kernel_stride: int = 16):
        super().__init__()
        self.kernel_size = kernel_size
        self.head_num_k = head_num_k
        self.head_dim = head_dim
        self.kernel_stride = kernel_stride

    def forward(self, k: torch.Tensor, cu_seqlens: torch.Tensor, lengths=None):
        """bf16 keys compress in bf16, fp32 keys in fp32; other dtypes go through bf16."""
        kc, cu_c = ops.compress_keys(k, cu_seqlens, kernel_size=self.kernel_size,
                                     kernel_stride=self.kernel_stride, lengths=lengths)
        if kc.dtype != k.dtype:
            kc = kc.to(k.dtype)
        return kc, cu_c


def _as_selector(module) -> LeanSelectSelector:
    sel = getattr(module, "leanselect", None)
    if sel is None:
        raise RuntimeError("LeanSelect selector was not initialized")
    if not isinstance(sel, LeanSelectSelector):
        sel = LeanSelectSelector.from_reference(sel)
        module.leanselect = sel
    return sel


def lightweight_compressed_attention(module, q_unpad: torch.Tensor, k_compressed: torch.Tensor,
                                     cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                                     max_seqlen_q: int, cache_lens: torch.Tensor | None = None,
                                     q_pred_for_topk: torch.Tensor | None = None,
                                     q_lengths=None) -> torch.Tensor:
    """``topk_idx [G, total_q, take]`` int32 for a packed prefill batch.

    ``module`` supplies ``leanselect``, ``topk``, ``block_size``,
    ``init_blocks``, ``local_blocks``, ``kernel_stride`` and
    ``num_key_value_heads`` like the reference attention module; the reference
    method can be replaced by ``functools.partial(lightweight_compressed_attention, module)``.
    ``cu_seqlens_k`` are the *compressed* offsets (as in the reference).
    ``q_lengths`` (host list) avoids reading ``cu_seqlens_q`` back.
    """
    del q_pred_for_topk
    if cache_lens is not None:
        raise ValueError("Lightweight selection is prefill only")
    method = getattr(module, "selection_method", "leanselect")
    lengths = list(q_lengths) if q_lengths is not None else ops.host_lengths(cu_seqlens_q)
    if method == "uniform":
        # minicpm.py:3073-3087
        from .uniform import uniform_prefill_topk_idx
        return uniform_prefill_topk_idx(
            q_unpad, k_compressed, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
            max_seqlen_q=max_seqlen_q, topk=int(module.topk), block_size=int(module.block_size),
            kernel_stride=int(module.kernel_stride), init_blocks=int(module.init_blocks),
            local_blocks=int(module.local_blocks), q_lengths=lengths)[0]
    if method != "leanselect":
        raise NotImplementedError(f"selection_method={method!r} is not served by leanselect_b200")
    selector = _as_selector(module)
    block = int(module.block_size)
    max_pages = max(((n + block - 1) // block for n in lengths), default=0)
    take = min(int(module.topk), max_pages)
    if q_unpad.dtype == torch.float32:
        # fp32 inputs are selected in fp32, as the reference's fp32 einsums do.
        q_fused, kv_fused = selector.fused_weights()
        return ops.select_pages_f32(q_unpad, q_fused, k_compressed, kv_fused, cu_seqlens_q,
                                    cu_seqlens_k, int(max(lengths, default=0)), take=take,
                                    init_blocks=int(module.init_blocks),
                                    local_blocks=int(module.local_blocks), block_size=block,
                                    kernel_stride=int(module.kernel_stride))
    weights = selector.kernel_weights()
    ks = ops.project_atom_keys(k_compressed, weights.wk_t)
    return ops.select_pages(q_unpad, weights, ks, cu_seqlens_q, cu_seqlens_k,
                            int(max(lengths, default=0)), take=take,
                            init_blocks=int(module.init_blocks),
                            local_blocks=int(module.local_blocks), block_size=block,
                            kernel_stride=int(module.kernel_stride))


def nosa_atom_scores(module, query_layer: torch.Tensor, compressed_k: torch.Tensor,
                     cu_seqlens_q: torch.Tensor, compressed_cu_seqlens: torch.Tensor,
                     q_lengths=None, c_lengths=None) -> torch.Tensor:
    """NOSA's ``LlamaSdpaAttention._leanselect_atom_scores`` (nosa.py:1822-1853).

    ``[G, total_q, max_atoms]`` raw LeanSelect atom scores in the query dtype,
    ``-inf`` past each sequence's atoms, for NOSA's ``compressed_attention``
    (``precomputed_qk_score``).  Computed by the same tcgen05 scoring kernel
    as the MiniCPM path.
    """
    selector = _as_selector(module)
    if selector is None:
        raise RuntimeError("NOSA LeanSelect selector was not initialized")
    lens_c = list(c_lengths) if c_lengths is not None else ops.host_lengths(compressed_cu_seqlens)
    lens_q = list(q_lengths) if q_lengths is not None else ops.host_lengths(cu_seqlens_q)
    weights = selector.kernel_weights()
    ks = ops.project_atom_keys(compressed_k, weights.wk_t)
    out = ops.atom_scores(query_layer, weights, ks, cu_seqlens_q, compressed_cu_seqlens,
                          int(max(lens_q, default=0)), int(max(lens_c, default=0)))
    return out if query_layer.dtype == torch.bfloat16 else out.to(query_layer.dtype)


def infllmv2_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                              dropout_p: float = 0.0, softmax_scale=None, causal: bool = False,
                              window_size=(-1, -1), softcap: float = 0.0, alibi_slopes=None,
                              deterministic: bool = False, return_attn_probs: bool = False,
                              block_table=None, topk_idx=None):
    """Stage-2 block-sparse attention with the InfLLM-v2 varlen signature.

    Only the sparse prefill form used by LeanSelect is served: ``topk_idx``
    must be given, without dropout, softcap, ALiBi, sliding windows or a
    paged block table.  Returns ``out`` or, with ``return_attn_probs``,
    ``(out, softmax_lse, None)``.
    """
    del deterministic
    if topk_idx is None:
        raise NotImplementedError("dense attention is not part of the LeanSelect hot path")
    if dropout_p or softcap or alibi_slopes is not None or block_table is not None:
        raise NotImplementedError("dropout, softcap, alibi and block tables are not supported")
    if tuple(window_size) != (-1, -1):
        raise NotImplementedError("sliding-window attention is not supported")
    result = ops.sparse_attn(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                             topk_idx, softmax_scale=softmax_scale, causal=causal,
                             return_lse=return_attn_probs)
    if return_attn_probs:
        out, lse = result
        return out, lse, None
    return result


def _not_served(name):
    def fn(*args, **kwargs):
        raise NotImplementedError(f"{name} belongs to the native InfLLM-v2 selection method, "
                                  "which leanselect_b200 does not serve")
    fn.__name__ = name
    return fn


# Symbols the reference's load_model presence check looks up
# (models/__init__.py:69-85); only the LeanSelect method is served.
infllmv2_attn_stage1 = _not_served("infllmv2_attn_stage1")
max_pooling_1d_varlen = _not_served("max_pooling_1d_varlen")


@dataclass
class LayerConfig:
    """Sparse geometry of one layer (sparse_config, minicpm.py:1957-1966)."""

    topk: int = 67            # total pages per (group, token), the reference's self.topk
    block_size: int = 64
    kernel_size: int = 32
    kernel_stride: int = 16
    init_blocks: int = 1
    local_blocks: int = 2
    selection_method: str = "leanselect"
    # Optional per-sequence budget: maps a sequence length to its total page
    # count T (e.g. benchmark config 4: min(64, pages // 10) + sink + local).
    # The reference takes one T per packed call (minicpm.py:3104), so such a
    # batch is selected sequence by sequence and padded to the largest T.
    per_sequence_topk: Callable[[int], int] | None = None


def config4_budget(seq_len: int, block_size: int = 64, init_blocks: int = 1,
                   local_blocks: int = 2) -> int:
    """benchmark config 4 budget: min(64, floor(0.1 * pages)) + sink + local pages."""
    pages = (int(seq_len) + block_size - 1) // block_size
    return min(64, pages // 10) + init_blocks + local_blocks


class _LayerView:
    """Namespace with the attributes ``lightweight_compressed_attention`` reads."""

    def __init__(self, cfg: LayerConfig, selector: LeanSelectSelector):
        self.leanselect = selector
        self.topk = cfg.topk
        self.block_size = cfg.block_size
        self.init_blocks = cfg.init_blocks
        self.local_blocks = cfg.local_blocks
        self.kernel_stride = cfg.kernel_stride
        self.selection_method = cfg.selection_method
        self.num_key_value_heads = selector.num_kv_heads


def count_attended_keys(topk_idx: torch.Tensor, lengths, block_size: int = 64,
                        positions: torch.Tensor | None = None) -> int:
    """Number of (group, token, key) triples the sparse attention computes.

    Counts, for each token, the keys of its selected pages that are causally
    visible (each page at most once; the selection never repeats a page).
    Used to state the attention's algorithmic FLOPs (4 * D * Hg per triple).
    ``positions`` (token positions inside their sequences) replaces
    ``lengths`` for query chunks of a longer sequence.
    """
    dev = topk_idx.device
    if positions is None:
        pos = torch.cat([torch.arange(int(n), device=dev) for n in lengths])
    else:
        pos = positions.to(dev)
    start = topk_idx.long() * block_size
    visible = torch.clamp(torch.minimum(start + block_size, pos[None, :, None] + 1) - start, min=0)
    return int((visible * (topk_idx >= 0)).sum().item())


def _select_per_sequence(q: torch.Tensor, kc: torch.Tensor, lens, selector: LeanSelectSelector,
                         cfg: LayerConfig) -> torch.Tensor:
    """Selection with a per-sequence budget: one call per sequence, padded with -1."""
    budgets = [int(cfg.per_sequence_topk(n)) for n in lens]
    takes = [min(t, (n + cfg.block_size - 1) // cfg.block_size) for t, n in zip(budgets, lens)]
    idx = torch.full((selector.num_kv_heads, q.shape[0], max(takes, default=0)), -1,
                     dtype=torch.int32, device=q.device)
    q0 = c0 = 0
    for n, t in zip(lens, budgets):
        a = ops.atom_count(n, cfg.kernel_size, cfg.kernel_stride)
        if n > 0:
            view = _LayerView(cfg, selector)
            view.topk = t
            cu_q = torch.tensor([0, n], dtype=torch.int32, device=q.device)
            cu_c = torch.tensor([0, a], dtype=torch.int32, device=q.device)
            part = lightweight_compressed_attention(view, q[q0:q0 + n], kc[c0:c0 + a], cu_q,
                                                    cu_c, n, q_lengths=[n])
            idx[:, q0:q0 + n, :part.shape[2]] = part
        q0 += n
        c0 += a
    return idx


def prefill_layer_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            cu_seqlens: torch.Tensor, max_seqlen: int,
                            selector: LeanSelectSelector, cfg: LayerConfig, *, lengths=None,
                            return_topk: bool = False, timers: list | None = None):
    """Compress -> select -> sparse attention for one layer's packed prefill.

    ``q [total, H, D]``, ``k``/``v [total, G, D]`` are post-RoPE; queries and
    keys share ``cu_seqlens`` (prefill).  Returns ``out [total, H, D]`` (and
    ``topk_idx`` with ``return_topk``).  ``timers`` (optional list) receives
    ``(stage, start_event, end_event)`` for the stages ``compress``,
    ``select`` and ``attn`` on the current stream.
    """
    def mark():
        if timers is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    lens = list(lengths) if lengths is not None else ops.host_lengths(cu_seqlens)
    e0 = mark()
    kc, cu_c = ops.compress_keys(k, cu_seqlens, kernel_size=cfg.kernel_size,
                                 kernel_stride=cfg.kernel_stride, lengths=lens)
    e1 = mark()
    if cfg.per_sequence_topk is None or len(lens) == 1:
        view = _LayerView(cfg, selector)
        if cfg.per_sequence_topk is not None:
            view.topk = int(cfg.per_sequence_topk(lens[0]))
        idx = lightweight_compressed_attention(view, q, kc, cu_seqlens, cu_c, max_seqlen,
                                               q_lengths=lens)
    else:
        idx = _select_per_sequence(q, kc, lens, selector, cfg)
    e2 = mark()
    out = ops.sparse_attn(q, k, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen, idx,
                          causal=True)
    e3 = mark()
    if timers is not None:
        timers.extend([("compress", e0, e1), ("select", e1, e2), ("attn", e2, e3)])
    return (out, idx) if return_topk else out
