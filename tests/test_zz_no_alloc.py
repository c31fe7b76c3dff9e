"""ls_select_pages_noalloc: selection without any device allocation (needs a B200).

The entry point serves callers that cannot allocate device memory (for
instance a C host whose device-memory budget is owned by another runtime, or
a caller that must not pay for cudaMalloc's device-wide synchronisation).  It
runs the same kernels as ls_select_pages on a scratch buffer compiled into
the library, so its output must equal ls_select_pages' output exactly.  The
test calls it twice in a row through the C ABI, the second time on a smaller
batch, so scratch contents left by the first call would show up as a
mismatch.  It lives in its own file, collected last.
"""
import ctypes

import pytest
import torch

from oracle import leanselect_oracle as ora

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs CUDA", allow_module_level=True)

import leanselect_b200 as lsb  # noqa: E402
from leanselect_b200 import _native, ops  # noqa: E402

DEV = torch.device("cuda", 0)


def _inputs(lens, seed):
    inp = ora.synthetic_layer(lens, num_heads=32, num_kv_heads=2, head_dim=128, router_heads=4,
                              router_dim=32, hot_pages=3, seed=seed, bf16=True)
    sel = lsb.LeanSelectSelector(num_heads=32, num_kv_heads=2, head_dim=128, router_heads=4,
                                 router_dim=32)
    with torch.no_grad():
        for name in ("head_mix", "kv_head_mix", "q_proj", "k_proj"):
            getattr(sel, name).copy_(torch.from_numpy(getattr(inp.params, name)))
    sel = sel.to(DEV)
    w = sel.kernel_weights()
    q = torch.from_numpy(inp.q).to(DEV, torch.bfloat16)
    cu = torch.from_numpy(inp.cu_seqlens).to(DEV)
    kc, cu_c = ops.compress_keys(torch.from_numpy(inp.k).to(DEV, torch.bfloat16), cu)
    ks = ops.project_atom_keys(kc, w.wk_t)
    return q, w, ks, cu, cu_c


def _noalloc(q, w, ks, cu, cu_c, max_len, take):
    lib = _native.load()
    out = torch.full((2, q.shape[0], take), -7, dtype=torch.int32, device=DEV)
    rc = lib.ls_select_pages_noalloc(
        q.data_ptr(), w.wq_t.data_ptr(), ks.data_ptr(), cu.data_ptr(), cu_c.data_ptr(),
        cu.numel() - 1, max_len, q.shape[0], ks.shape[1], 32, 2, 128, 128, take, 1, 2, 64, 16,
        out.data_ptr(), ops.status_word(DEV).data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _native.LS_OK, lib.ls_last_error().decode()
    return out


@pytest.mark.parametrize("first,second", [(([3000, 700, 20, 1500], 35), ([900, 65], 12))])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(first, second):
    ops.status_word(DEV).zero_()
    for (lens, topk), seed in ((first, 1), (second, 2)):
        q, w, ks, cu, cu_c = _inputs(lens, seed)
        take = min(topk, max((n + 63) // 64 for n in lens))
        got = _noalloc(q, w, ks, cu, cu_c, max(lens), take)
        want = ops.select_pages(q, w, ks, cu, cu_c, max(lens), take=take)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert ops.check_status(DEV) == 0


def test_noalloc_accepts_a_request_of_exactly_its_scratch():
    """One 16384-token sequence with 2 KV groups needs exactly the 16 MiB built
    into the library: accepted, and equal to the workspace entry point."""
    from measure.inputs import config1_layer, make_selector

    n = 16384
    lib = _native.load()
    assert lib.ls_select_pages_workspace_bytes(n, 2, n) == 16 << 20
    ops.status_word(DEV).zero_()
    q, k, _ = config1_layer(n, DEV, 4)
    w = make_selector(DEV, 4).kernel_weights()
    cu = torch.tensor([0, n], dtype=torch.int32, device=DEV)
    kc, cu_c = ops.compress_keys(k, cu, lengths=[n])
    ks = ops.project_atom_keys(kc, w.wk_t)
    for take in (67, 96):
        out = torch.full((2, n, take), -7, dtype=torch.int32, device=DEV)
        rc = lib.ls_select_pages_noalloc(
            q.data_ptr(), w.wq_t.data_ptr(), ks.data_ptr(), cu.data_ptr(), cu_c.data_ptr(), 1, n,
            n, ks.shape[1], 32, 2, 128, 128, take, 1, 2, 64, 16, out.data_ptr(),
            ops.status_word(DEV).data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == _native.LS_OK, lib.ls_last_error().decode()
        want = ops.select_pages(q, w, ks, cu, cu_c, n, take=take)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert ops.check_status(DEV) == 0


def test_noalloc_rejects_requests_beyond_its_scratch():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    # One 32K-token sequence needs 2 * 32768 * 512 * 2 bytes = 64 MiB of scratch.
    rc = lib.ls_select_pages_noalloc(fake, fake, fake, fake, fake, 1, 32768, 32768, 2047, 32, 2,
                                     128, 128, 67, 1, 2, 64, 16, fake, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED
    assert b"scratch" in lib.ls_last_error()
