"""The torch.library custom ops: registration and fake (meta) shapes, no GPU needed."""
import pytest
import torch

import leanselect_b200.torch_ops  # noqa: F401  (registers torch.ops.leanselect_b200.*)

OPS = torch.ops.leanselect_b200
META = torch.device("meta")


def t(*shape, dtype=torch.bfloat16):
    return torch.empty(shape, dtype=dtype, device=META)


def test_all_ops_are_registered():
    for name in ("compress_keys", "project_atom_keys", "select_pages", "score_pages",
                 "sparse_attn"):
        assert hasattr(OPS, name)


def test_fake_shapes():
    N, H, G, D, F = 4096, 32, 2, 128, 128
    cu = t(3, dtype=torch.int32)
    kc, cu_c = OPS.compress_keys(t(N, G, D), cu, 250, 32, 16)
    assert kc.shape == (250, G, D) and kc.dtype == torch.bfloat16
    assert cu_c.shape == (3,) and cu_c.dtype == torch.int32
    ks = OPS.project_atom_keys(kc, t(G, F, D))
    assert ks.shape == (G, 250, F)
    idx = OPS.select_pages(t(N, H, D), t(G, F, (H // G) * D), ks, cu, cu_c, 3000, 67, 1, 2)
    assert idx.shape == (G, N, 67) and idx.dtype == torch.int32
    scores = OPS.score_pages(t(N, H, D), t(G, F, (H // G) * D), ks, cu, cu_c, 3000)
    assert scores.shape == (G, N, 47) and scores.dtype == torch.float32
    out, lse = OPS.sparse_attn(t(N, H, D), t(N, G, D), t(N, G, D), cu, cu, 3000, 3000, idx, 0.0,
                               True)
    assert out.shape == (N, H, D) and lse.shape == (H, N) and lse.dtype == torch.float32


def test_cpu_tensors_raise():
    with pytest.raises(RuntimeError, match="CUDA"):
        OPS.project_atom_keys(torch.zeros(8, 2, 128, dtype=torch.bfloat16),
                              torch.zeros(2, 128, 128, dtype=torch.bfloat16))
