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
* ``get_compress_k`` -> the prefill branch computes both compressions in one
  pass over the keys and fills the ``InfLLMv2Cache`` through its own
  ``update_*`` methods, as minicpm.py:2782-2866 does; decode steps and the
  KL-target caches keep the reference's method;
* ``leanselect`` -> :class:`leanselect_b200.LeanSelectSelector` sharing the
  reference selector's parameter tensors;
* ``_lightweight_compressed_attention`` -> the fused selection
  (minicpm.py:3061-3142);
* ``sparse_forward`` -> the block-sparse attention kernel (minicpm.py:3216-3244).

The reference tree is not imported here; objects are matched by attribute.
"""
from __future__ import annotations

import functools
import sys
import types

import torch

from . import ops
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


def _get_compress_k(self, key_states, attention_mask, past_key_value,
                    enable_kl_target_cache: bool = False):
    """``MiniCPMInfLLMv2Attention.get_compress_k`` (minicpm.py:2774-2964).

    Prefill: unpad the keys with the reference module's own
    ``_unpad_one_tensor``, compute ``compress_k`` (32/16) and ``compress_k2``
    (128/64) in one pass over K (``ops.compress_keys_dual``, bit for bit
    what the two compressor modules give), and hand the cache the same
    updates as minicpm.py:2794-2866: both compressions with their
    cu_seqlens, and per sequence the keys after the last atom's start
    (``A * kernel_stride`` on, resp. ``A2 * 4 * kernel_stride``) as the
    uncompressed tails a decode step extends.  Decode steps, KL-target
    caches and other geometries or dtypes call the reference method.
    """
    layer = past_key_value.layers[self.layer_idx]
    prefilling = not layer.compress_k_cache
    kl_target = enable_kl_target_cache and getattr(self, "_kl_target_compress_differs", False)
    geometry = (int(self.kernel_size), int(self.kernel_stride)) == (32, 16)
    if not prefilling or kl_target or not geometry or key_states.dtype != torch.bfloat16:
        return self._reference_get_compress_k(key_states, attention_mask, past_key_value,
                                              enable_kl_target_cache)
    unpad = sys.modules[type(self).__module__]._unpad_one_tensor
    unpadded, _, cu_seqlens, _ = unpad(key_states, attention_mask=attention_mask)
    lengths = ops.host_lengths(cu_seqlens)
    kc, cu_c, kc2, cu_c2 = ops.compress_keys_dual(unpadded, cu_seqlens, lengths=lengths)
    past_key_value.update_compress_k(kc, self.layer_idx, cu_c)
    past_key_value.update_compress_k2(kc2, self.layer_idx, cu_c2)
    stride = int(self.kernel_stride)
    starts = [0]
    for n in lengths:
        starts.append(starts[-1] + n)
    tails = [unpadded[s0 + ops.atom_count(n, 32, 16) * stride:s0 + n].clone()
             for s0, n in zip(starts, lengths)]
    past_key_value.update_no_compress_k(tails, self.layer_idx, kernel_stride=stride,
                                        kernel_size=int(self.kernel_size))
    tails2 = [unpadded[s0 + ops.atom_count(n, 128, 64) * stride * 4:s0 + n].clone()
              for s0, n in zip(starts, lengths)]
    past_key_value.update_no_compress_k2(tails2, self.layer_idx, kernel_stride=stride * 4,
                                         kernel_size=int(self.kernel_size) * 4)
    return kc, cu_c, kc2, cu_c2


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
    reference = getattr(attn, "get_compress_k", None)
    if reference is not None and getattr(reference, "__func__", None) is not _get_compress_k:
        attn._reference_get_compress_k = reference
        attn.get_compress_k = types.MethodType(_get_compress_k, attn)


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
