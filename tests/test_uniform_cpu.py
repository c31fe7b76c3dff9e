"""Host-side behaviour of the uniform-method mirror (no GPU needed)."""
import pytest
import torch

from leanselect_b200.uniform import uniform_prefill_topk_idx


def test_rejects_decode_lengths():
    q = torch.zeros(3, 32, 128)
    kc = torch.zeros(1, 2, 128)
    with pytest.raises(ValueError, match="prefill-only"):
        uniform_prefill_topk_idx(q, kc, cu_seqlens_q=torch.tensor([0, 1, 3]),
                                 cu_seqlens_k=torch.tensor([0, 0, 1]), max_seqlen_q=2, topk=4)


def test_rejects_non_3d_inputs():
    with pytest.raises(ValueError, match="3D"):
        uniform_prefill_topk_idx(torch.zeros(3, 128), torch.zeros(1, 2, 128),
                                 cu_seqlens_q=torch.tensor([0, 3]),
                                 cu_seqlens_k=torch.tensor([0, 1]), max_seqlen_q=3, topk=4)


def test_cpu_tensors_have_no_fallback():
    q = torch.zeros(64, 32, 128, dtype=torch.bfloat16)
    kc = torch.zeros(3, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        uniform_prefill_topk_idx(q, kc, cu_seqlens_q=torch.tensor([0, 64]),
                                 cu_seqlens_k=torch.tensor([0, 3]), max_seqlen_q=64, topk=4)
