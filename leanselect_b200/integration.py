"""Route a reference LeanSelect model's prefill hot path through leanselect_b200.

For a model loaded with the reference's ``load_model(..., method="leanselect")``:

    import leanselect.models.minicpm as minicpm
    from leanselect_b200.integration import install, install_module_symbols
    install_module_symbols(minicpm)          # before load_model: satisfies its presence check
    model, tokenizer = load_model("minicpm", path, method="leanselect", ...)
    install(model)

``install`` patches every ``MiniCPMInfLLMv2Attention`` (minicpm.py:1948) and
every module that owns a ``leanselect`` selector (NOSA's ``LlamaSdpaAttention``,
nosa.py:1822-1853):

* ``compress_k`` / ``compress_k2`` -> :class:`leanselect_b200.CompressK`
  (minicpm.py:2035-2046 instantiates them, 2476-2481 calls them);
* ``leanselect`` -> :class:`leanselect_b200.LeanSelectSelector` sharing the
  reference selector's parameter tensors;
* ``_lightweight_compressed_attention`` -> the fused selection
  (minicpm.py:3061-3142);
* ``sparse_forward`` -> the block-sparse attention kernel (minicpm.py:3216-3244).

The reference tree is not imported here; objects are matched by attribute.
"""
from __future__ import annotations

import functools
import types

from .attention import (CompressK, infllmv2_attn_stage1, infllmv2_attn_varlen_func,
                        lightweight_compressed_attention, max_pooling_1d_varlen,
                        nosa_atom_scores)
from .selector import LeanSelectSelector

ATTENTION_CLASS_NAMES = ("MiniCPMInfLLMv2Attention",)


def install_module_symbols(module) -> None:
    """Bind the stage-2 symbols the reference module looks up.

    ``load_model`` requires ``infllmv2_attn_stage1``, ``infllmv2_attn_varlen_func``
    and ``max_pooling_1d_varlen`` to be callable (models/__init__.py:69-85) and
    ``sparse_forward`` calls the module-level ``infllmv2_attn_varlen_func`` for
    prefill and decode alike.  The attention is always the B200 kernel.  The
    native InfLLM-v2 stage-1 selection (used by the reference for decode and
    for the native method) is not part of this library: the module's own
    functions are kept when the extension provided them, and stubs that raise
    are bound only where they are missing.
    """
    module.infllmv2_attn_varlen_func = infllmv2_attn_varlen_func
    if getattr(module, "infllmv2_attn_stage1", None) is None:
        module.infllmv2_attn_stage1 = infllmv2_attn_stage1
    if getattr(module, "max_pooling_1d_varlen", None) is None:
        module.max_pooling_1d_varlen = max_pooling_1d_varlen


def _sparse_forward(self, query_layer, key_layer, value_layer, cu_seqlens_q, cu_seqlens_k,
                    max_seqlen_in_batch_q, max_seqlen_in_batch_k, topk_idx, no_rope_param=None):
    """``MiniCPMInfLLMv2Attention.sparse_forward`` (minicpm.py:3216-3244)."""
    del no_rope_param
    return infllmv2_attn_varlen_func(
        query_layer, key_layer, value_layer, cu_seqlens_q, cu_seqlens_k, max_seqlen_in_batch_q,
        max_seqlen_in_batch_k, dropout_p=0.0, softmax_scale=None,
        causal=max_seqlen_in_batch_q != 1, topk_idx=topk_idx)


def patch_attention(attn) -> None:
    """Patch one reference attention module in place."""
    heads_k = int(attn.num_key_value_heads)
    head_dim = int(attn.head_dim)
    ks, st = int(attn.kernel_size), int(attn.kernel_stride)
    attn.compress_k = CompressK(heads_k, head_dim, kernel_size=ks, kernel_stride=st)
    if getattr(attn, "compress_k2", None) is not None:
        attn.compress_k2 = CompressK(heads_k, head_dim, kernel_size=ks * 4, kernel_stride=st * 4)
    patch_selector_owner(attn)
    attn._lightweight_compressed_attention = functools.partial(
        lightweight_compressed_attention, attn)
    attn.sparse_forward = types.MethodType(_sparse_forward, attn)


def patch_selector_owner(owner) -> None:
    """Swap ``owner.leanselect`` for the B200 selector (shared parameters); on
    NOSA layers also route ``_leanselect_atom_scores`` to the atom-score kernel."""
    sel = getattr(owner, "leanselect", None)
    if sel is not None and not isinstance(sel, LeanSelectSelector):
        owner.leanselect = LeanSelectSelector.from_reference(sel)
    if hasattr(owner, "_leanselect_atom_scores"):
        owner._leanselect_atom_scores = functools.partial(nosa_atom_scores, owner)


def install(model) -> int:
    """Patch every LeanSelect attention module of ``model``; returns how many."""
    count = 0
    for module in list(model.modules()):
        name = type(module).__name__
        if name in ATTENTION_CLASS_NAMES:
            patch_attention(module)
            count += 1
        elif getattr(module, "leanselect", None) is not None:
            patch_selector_owner(module)
            count += 1
    return count
