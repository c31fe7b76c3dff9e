"""Wiring of the reference-model integration shim (CPU, no kernel launches)."""
import types

import pytest

import torch
from torch import nn

import leanselect_b200 as lsb
from leanselect_b200 import integration


class RefSelector(nn.Module):
    """Stand-in with the reference LeanSelectSelector's attributes (selector.py:69-108)."""

    def __init__(self):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = 32, 2, 128
        self.router_heads, self.router_dim = 4, 32
        self.head_mix = nn.Parameter(torch.randn(32, 4))
        self.kv_head_mix = nn.Parameter(torch.ones(2, 4))
        self.q_proj = nn.Parameter(torch.randn(4, 128, 32))
        self.k_proj = nn.Parameter(torch.randn(4, 128, 32))


class MiniCPMInfLLMv2Attention(nn.Module):
    """Stand-in carrying the attributes the shim reads (minicpm.py:1951-2046)."""

    def __init__(self):
        super().__init__()
        self.num_key_value_heads, self.head_dim = 2, 128
        self.kernel_size, self.kernel_stride = 32, 16
        self.compress_k = nn.Identity()
        self.compress_k2 = nn.Identity()
        self.leanselect = RefSelector()
        self.topk, self.block_size, self.init_blocks, self.local_blocks = 67, 64, 1, 2
        self.selection_method = "leanselect"
        self.layer_idx = 0

    def get_compress_k(self, key_states, attention_mask, past_key_value,
                       enable_kl_target_cache=False):
        return "reference"


class NosaAttention(nn.Module):
    def __init__(self):
        super().__init__()
        self.leanselect = RefSelector()

    def _leanselect_atom_scores(self, *args):  # replaced by install()
        raise AssertionError("reference path should have been patched")


def test_install_patches_every_attention_module():
    model = nn.ModuleList([MiniCPMInfLLMv2Attention(), MiniCPMInfLLMv2Attention(), NosaAttention()])
    ref_params = [m.leanselect.head_mix for m in model]
    assert integration.install(model) == 3
    for attn in model[:2]:
        assert isinstance(attn.compress_k, lsb.CompressK)
        assert attn.compress_k2.kernel_size == 128 and attn.compress_k2.kernel_stride == 64
        assert isinstance(attn.leanselect, lsb.LeanSelectSelector)
        assert attn._lightweight_compressed_attention.func is lsb.lightweight_compressed_attention
        assert isinstance(attn.sparse_forward, types.MethodType)
        assert attn.get_compress_k.__func__ is integration._get_compress_k
        assert attn._reference_get_compress_k(None, None, None) == "reference"
    # Installing twice keeps the reference method, not the patched one.
    integration.install(model)
    assert model[0]._reference_get_compress_k(None, None, None) == "reference"
    assert isinstance(model[2].leanselect, lsb.LeanSelectSelector)
    assert model[2]._leanselect_atom_scores.func is lsb.nosa_atom_scores
    # The selectors share the reference parameter tensors (checkpoints keep working).
    for m, p in zip(model, ref_params):
        assert m.leanselect.head_mix is p


def test_module_symbols_satisfy_the_presence_check():
    mod = types.ModuleType("fake_minicpm")
    integration.install_module_symbols(mod)
    for name in ("infllmv2_attn_stage1", "infllmv2_attn_varlen_func", "max_pooling_1d_varlen"):
        assert callable(getattr(mod, name))


def test_module_symbols_keep_the_native_stage1_when_present():
    """The reference's own stage-1 (native decode selection) survives install."""
    def stage1(*args, **kwargs):
        return "native"

    mod = types.ModuleType("fake_minicpm")
    mod.infllmv2_attn_stage1 = stage1
    mod.max_pooling_1d_varlen = None
    mod.infllmv2_attn_varlen_func = None
    integration.install_module_symbols(mod)
    assert mod.infllmv2_attn_stage1 is stage1
    assert mod.infllmv2_attn_varlen_func is lsb.infllmv2_attn_varlen_func
    with pytest.raises(NotImplementedError):
        mod.max_pooling_1d_varlen()
