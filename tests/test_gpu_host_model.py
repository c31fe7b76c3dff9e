"""The benchmark host model on a B200: fused host kernels and prefill paths.

* ``ls_bb_*`` kernels vs their PyTorch references (one bf16 ulp);
* the sequence-parallel runner on a one-rank process group reproduces the
  single-device prefill bit for bit (same per-row math, chunked launches).
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs CUDA", allow_module_level=True)

from leanselect_b200 import host_kernels as hk  # noqa: E402
from leanselect_b200.model import (MiniCPMShape, PrefillModel, apply_rope,  # noqa: E402
                                   rms_norm)

DEV = torch.device("cuda", 0)


def close_bf16(a, b, ulps=2):
    a, b = a.float(), b.float()
    tol = ulps * 2 ** -8 * b.abs() + 1e-6
    assert torch.all((a - b).abs() <= tol), (a - b).abs().max()


def test_rms_norm_kernel():
    g = torch.Generator(device=DEV).manual_seed(0)
    x = (torch.randn(300, 4096, device=DEV, generator=g) * 3).bfloat16()
    w = (1 + 0.1 * torch.randn(4096, device=DEV, generator=g)).bfloat16()
    close_bf16(hk.rms_norm(x, w, 1e-6), rms_norm(x, w, 1e-6))


def test_rope_split_kernel():
    shape = MiniCPMShape(num_heads=32, num_kv_heads=2, max_position=131072)
    from leanselect_b200.model import LongRoPE

    rope = LongRoPE(shape, DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    n = 777
    qkv = torch.randn(n, 36 * 128, device=DEV, generator=g).bfloat16()
    pos = torch.arange(70000, 70000 + n, device=DEV)
    q, k, v = hk.rope_split(qkv, pos, rope.frequencies(131072), rope.scaling, 32, 2)
    cos, sin = rope.tables(pos, 131072)
    q_ref = apply_rope(qkv[:, :4096].view(n, 32, 128), cos, sin)
    k_ref = apply_rope(qkv[:, 4096:4352].view(n, 2, 128), cos, sin)
    close_bf16(q, q_ref, ulps=4)
    close_bf16(k, k_ref, ulps=4)
    assert torch.equal(v, qkv[:, 4352:].view(n, 2, 128))


def test_silu_mul_kernel():
    g = torch.Generator(device=DEV).manual_seed(2)
    gu = torch.randn(100, 2 * 1024, device=DEV, generator=g).bfloat16()
    ref = (torch.nn.functional.silu(gu[:, :1024].float()) * gu[:, 1024:].float()).bfloat16()
    close_bf16(hk.silu_mul(gu), ref)


def small_shape():
    return MiniCPMShape(vocab_size=1000, hidden_size=2048, intermediate_size=4096, num_layers=2,
                        num_heads=16, num_kv_heads=2, max_position=8192,
                        original_max_position=4096, router_heads=4, router_dim=32)


def test_prefill_is_finite_and_deterministic():
    model = PrefillModel(small_shape(), DEV, seed=3)
    ids = torch.randint(0, 1000, (2 * 4096,), device=DEV)
    cu = torch.tensor([0, 4096, 8192], dtype=torch.int32, device=DEV)
    a = model.prefill(ids, cu, [4096, 4096])
    b = model.prefill(ids, cu, [4096, 4096])
    assert a.shape == (2, 1000) and torch.isfinite(a).all()
    assert torch.equal(a, b)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [8192, 4096])
def test_sequence_parallel_single_rank_matches_single_device(n):
    """Bit-equal with and without the overlapped late gather (4096- and 2048-token chunks)."""
    import torch.distributed as dist
    from leanselect_b200.parallel import SequenceParallelRunner

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=DEV)
    try:
        shape = small_shape()
        ids = torch.randint(0, 1000, (n,), device=DEV, generator=torch.Generator(device=DEV).manual_seed(4))
        sp = SequenceParallelRunner(shape, DEV, seed=5)
        ref = PrefillModel(shape, DEV, seed=5)
        got = sp.prefill_device(ids, [n])
        want = ref.prefill(ids, torch.tensor([0, n], dtype=torch.int32, device=DEV), [n])
        assert torch.equal(got, want)
    finally:
        dist.destroy_process_group()
