"""B200-native (sm_100a) LeanSelect prefill hot path.

Stages: key compression -> selector scoring with the folded head mix ->
per-group top-T page selection (forced sink/local pages) -> block-sparse
causal attention over the selected pages.  Hand-written CUDA behind a C ABI
(``include/leanselect_b200.h``); PyTorch supplies device memory and streams.
"""
from . import ops
from ._native import LeanSelectError, LS_MAX_TOPK, version
from .attention import (CompressK, LayerConfig, infllmv2_attn_varlen_func,
                        lightweight_compressed_attention, nosa_atom_scores,
                        prefill_layer_attention)
from .selector import LeanSelectSelector
from .uniform import uniform_prefill_topk_idx

__all__ = [
    "ops", "LeanSelectError", "LS_MAX_TOPK", "version", "CompressK", "LayerConfig",
    "infllmv2_attn_varlen_func", "lightweight_compressed_attention", "nosa_atom_scores",
    "prefill_layer_attention",
    "LeanSelectSelector", "uniform_prefill_topk_idx",
]
