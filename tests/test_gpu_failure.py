"""A bounded device wait that expires, on purpose and without a fault (needs a B200).

``ls_wait_timeout_probe`` launches one CTA shaped like the scoring kernel:
it allocates tensor memory and waits on an mbarrier that nothing completes.
After the limit the kernel must record LS_DEVERR_TIMEOUT, unwind through the
CTA's abort flag, release its tensor memory and return.  The test then runs
the tcgen05 selection kernels on every SM of the same context: they allocate
tensor memory themselves, so they would not complete if the probe had kept
any.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs CUDA", allow_module_level=True)

from leanselect_b200 import _native, ops  # noqa: E402
from oracle import leanselect_oracle as ora  # noqa: E402

DEV = torch.device("cuda", 0)


def test_expired_wait_reports_timeout_and_releases_tensor_memory():
    lib = _native.load()
    stream = torch.cuda.current_stream(DEV)
    for timeout_ms in (2, 5):
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        done = torch.zeros(1, dtype=torch.int32, device=DEV)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rc = lib.ls_wait_timeout_probe(status.data_ptr(), done.data_ptr(), timeout_ms * 1000000,
                                       stream.cuda_stream)
        b.record(stream)
        assert rc == _native.LS_OK, lib.ls_last_error().decode()
        torch.cuda.synchronize()
        assert int(status.item()) == _native.LS_DEVERR_TIMEOUT
        assert int(done.item()) == 1
        assert a.elapsed_time(b) >= timeout_ms * 0.9

    # The context is healthy and every SM's tensor memory is free again.
    lens = [20000, 12000]
    inp = ora.synthetic_layer(lens, num_heads=32, num_kv_heads=2, head_dim=128, router_heads=4,
                              router_dim=32, hot_pages=3, seed=5, bf16=True)
    import leanselect_b200 as lsb
    sel = lsb.LeanSelectSelector(num_heads=32, num_kv_heads=2, head_dim=128, router_heads=4,
                                 router_dim=32)
    with torch.no_grad():
        for name in ("head_mix", "kv_head_mix", "q_proj", "k_proj"):
            getattr(sel, name).copy_(torch.from_numpy(getattr(inp.params, name)))
    w = sel.to(DEV).kernel_weights()
    q = torch.from_numpy(inp.q).to(DEV, torch.bfloat16)
    cu = torch.from_numpy(inp.cu_seqlens).to(DEV)
    kc, cu_c = ops.compress_keys(torch.from_numpy(inp.k).to(DEV, torch.bfloat16), cu)
    ks = ops.project_atom_keys(kc, w.wk_t)
    ops.status_word(DEV).zero_()
    idx = ops.select_pages(q, w, ks, cu, cu_c, max(lens), take=67).cpu().numpy()
    assert ops.check_status(DEV) == 0
    rows = np.array([0, 100, 5000, 19999, 20000 + 11999])
    ekc, ecu = ora.compress_keys(inp.k, inp.cu_seqlens, policy="bf16")
    for row in rows:
        b = int(np.searchsorted(inp.cu_seqlens, row, side="right") - 1)
        q0, c0, c1 = int(inp.cu_seqlens[b]), int(ecu[b]), int(ecu[b + 1])
        want = ora.select_for_queries(inp.q[row:row + 1], [row - q0], lens[b], ekc[c0:c1],
                                      inp.params, take=67)
        bad = ora.selection_mismatches(idx[:, row:row + 1], want, rel_tol=1e-3, ulps=1)
        assert not bad, (row, bad)
