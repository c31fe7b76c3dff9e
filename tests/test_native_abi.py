"""The C ABI library and the host-side API, without a GPU.

Only calls that fail argument validation are made here: validation happens
on the host before any CUDA call, so these run on a machine without a GPU.
"""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import leanselect_b200 as lsb
from leanselect_b200 import _native

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    text = "\n".join(h.read_text() for h in HEADERS)
    return sorted(set(re.findall(r"^(?:const char\*|int|size_t)\s+(ls_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    names = declared_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(_native.SIGNATURES) | set(_native.STRING_FUNCS) | set(_native.SIZE_FUNCS) == set(names)


def test_version_and_status_strings():
    assert "sm_100a" in lsb.version()
    lib = _native.load()
    assert lib.ls_status_string(0) == b"LS_OK"
    assert lib.ls_status_string(2) == b"LS_ERR_UNSUPPORTED"
    assert lib.ls_status_string(99) == b"LS_ERR_UNKNOWN"


def test_null_pointers_are_rejected():
    lib = _native.load()
    rc = lib.ls_sparse_attn(None, None, None, None, None, 1, 1, 1, 1, 1, 32, 2, 128, None, 1, 64,
                            0.0, 1, None, None, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    assert b"null" in lib.ls_last_error()


def test_unsupported_geometry_is_reported():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    rc = lib.ls_select_pages(fake, fake, fake, fake, fake, 1, 64, 64, 3, 32, 2, 64, 128, 5, 1, 2,
                             64, 16, fake, fake, 1 << 20, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED
    rc = lib.ls_select_pages(fake, fake, fake, fake, fake, 1, 64, 64, 3, 32, 2, 128, 128, 129, 1,
                             2, 64, 16, fake, fake, 1 << 20, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # take > LS_MAX_TOPK
    rc = lib.ls_sparse_attn(fake, fake, fake, fake, fake, 1, 64, 64, 64, 64, 24, 2, 128, fake, 4,
                            64, 0.0, 1, fake, None, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # 12 heads per group
    rc = lib.ls_compress_keys(fake, fake, 1, 64, 2, 128, 48, 16, fake, fake, 3, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # kernel_size/stride = 3


def test_workspace_size_and_check():
    lib = _native.load()
    # 2 groups x 1000 rows x round8(ceil(1000/64) = 16) pages x 2 bytes (bf16 scores)
    assert lib.ls_select_pages_workspace_bytes(1000, 2, 1000) == 2 * 1000 * 16 * 2
    assert lib.ls_select_pages_workspace_bytes(1000, 2, 1100) == 2 * 1000 * 24 * 2
    fake = ctypes.c_void_p(1 << 20)
    rc = lib.ls_select_pages(fake, fake, fake, fake, fake, 1, 1000, 1000, 61, 32, 2, 128, 128, 35,
                             1, 2, 64, 16, fake, fake, 100, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.ls_last_error()


def test_split_attention_workspace_and_argument_checks():
    lib = _native.load()
    # splits x rows x (128 output floats + max + sum) x 4 bytes; nothing for one slice
    assert lib.ls_sparse_attn_split_workspace_bytes(3, 32, 8) == 8 * 3 * 32 * 130 * 4
    assert lib.ls_sparse_attn_split_workspace_bytes(3, 32, 1) == 0
    fake = ctypes.c_void_p(1 << 20)
    args = (fake, fake, fake, fake, fake, 3, 1, 4096, 3, 3 * 4096, 32, 2, 128, fake, 67, 64, 0.0,
            0)
    for splits in (0, _native.LS_MAX_ATTN_SPLITS + 1):
        rc = lib.ls_sparse_attn_split(*args, splits, fake, 1 << 20, fake, None, None, None)
        assert rc == _native.LS_ERR_INVALID_ARGUMENT
        assert b"splits" in lib.ls_last_error()
    rc = lib.ls_sparse_attn_split(*args, 8, None, 0, fake, None, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    rc = lib.ls_sparse_attn_split(*args, 8, fake, 8 * 3 * 32 * 130 * 4 - 1, fake, None, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.ls_last_error()


def test_split_count_choice():
    from leanselect_b200 import ops

    class Props:
        multi_processor_count = 148

    orig = torch.cuda.get_device_properties
    torch.cuda.get_device_properties = lambda dev: Props()
    try:
        dev = torch.device("cpu")
        assert ops.attn_splits(2, 1, 131072, 67, dev) == 16        # batch 1: pages // 4 caps it
        assert ops.attn_splits(16, 1, 131072, 67, dev) == 9        # batch 8
        assert ops.attn_splits(128, 1, 131072, 67, dev) == 1       # batch 64
        assert ops.attn_splits(1024, 1, 131072, 67, dev) == 1      # enough rows
        assert ops.attn_splits(2, 1, 200, 67, dev) == 1            # 4 pages: nothing to cut
        assert ops.attn_splits(2, 4096, 131072, 67, dev) == 1      # prefill is never split
    finally:
        torch.cuda.get_device_properties = orig


def test_noalloc_checks_arguments_before_its_scratch_limit():
    """A malformed call gets ls_select_pages' own error, not the scratch-size one;
    a well-formed call one token past the 16 MiB limit gets LS_ERR_UNSUPPORTED."""
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    # head_dim 64 on a request far beyond the scratch: the geometry error wins.
    rc = lib.ls_select_pages_noalloc(fake, fake, fake, fake, fake, 1, 65536, 65536, 4095, 32, 2,
                                     64, 128, 67, 1, 2, 64, 16, fake, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED
    assert b"head_dim" in lib.ls_last_error()
    rc = lib.ls_select_pages_noalloc(fake, fake, fake, fake, fake, 1, 65536, 65536, 4095, 32, 2,
                                     128, 128, 67, 1, 2, 64, 16, None, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    assert b"topk_idx" in lib.ls_last_error()
    # 16384 tokens x 2 groups x 256 pages x 2 bytes is exactly 16 MiB; one more token is not.
    assert lib.ls_select_pages_workspace_bytes(16384, 2, 16384) == 16 << 20
    assert lib.ls_select_pages_workspace_bytes(16385, 2, 16385) > 16 << 20
    rc = lib.ls_select_pages_noalloc(fake, fake, fake, fake, fake, 1, 16385, 16385, 1023, 32, 2,
                                     128, 128, 67, 1, 2, 64, 16, fake, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED
    assert b"scratch" in lib.ls_last_error()


def test_wait_probe_validates_on_host():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    assert lib.ls_wait_timeout_probe(None, fake, 1000000, None) == _native.LS_ERR_INVALID_ARGUMENT
    assert lib.ls_wait_timeout_probe(fake, fake, 10, None) == _native.LS_ERR_INVALID_ARGUMENT
    assert lib.ls_wait_timeout_probe(fake, fake, 3 * 10 ** 9, None) == _native.LS_ERR_INVALID_ARGUMENT
    assert b"timeout_ns" in lib.ls_last_error()


def test_misaligned_pointer_is_reported():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    odd = ctypes.c_void_p((1 << 20) + 2)
    rc = lib.ls_sparse_attn(odd, fake, fake, fake, fake, 1, 64, 64, 64, 64, 32, 2, 128, fake, 4,
                            64, 0.0, 1, fake, None, None, None)
    assert rc == _native.LS_ERR_ALIGNMENT


def test_selector_geometry_errors_match_reference():
    """Constructor checks of selector.py:81-94."""
    for kwargs in ({"num_heads": 7}, {"router_heads": 9}, {"head_dim": 0}):
        config = dict(num_heads=8, num_kv_heads=2, head_dim=8)
        config.update(kwargs)
        with pytest.raises(ValueError):
            lsb.LeanSelectSelector(**config)


def test_selector_shape_errors_match_reference():
    """project_* reject bad shapes with ValueError (selector.py:161-166, 180-186)."""
    sel = lsb.LeanSelectSelector(num_heads=8, num_kv_heads=2, head_dim=8, router_heads=2,
                                 router_dim=4)
    with pytest.raises(ValueError):
        sel.project_queries(torch.randn(2, 3, 8))
    with pytest.raises(ValueError):
        sel.project_atom_keys(torch.randn(2, 3, 8))


def test_product_path_has_no_cpu_fallback():
    sel = lsb.LeanSelectSelector(num_heads=32, num_kv_heads=2, head_dim=128)
    with pytest.raises(RuntimeError, match="CUDA"):
        sel.project_queries(torch.zeros(4, 32, 128))
    with pytest.raises(RuntimeError, match="CUDA"):
        lsb.ops.sparse_attn(torch.zeros(4, 32, 128), torch.zeros(4, 2, 128),
                            torch.zeros(4, 2, 128), torch.tensor([0, 4]), torch.tensor([0, 4]),
                            4, 4, torch.zeros(2, 4, 1, dtype=torch.int32))


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="not found"):
        _native.load(tmp_path / "missing.so")


def test_selector_initialisation_matches_reference_rule():
    """reset_parameters (selector.py:112-137): group mean mix, scaled orthonormal frame."""
    torch.manual_seed(7)
    sel = lsb.LeanSelectSelector(num_heads=8, num_kv_heads=2, head_dim=8, router_heads=2,
                                 router_dim=4)
    assert torch.allclose(sel.head_mix, torch.full((8, 2), 0.25))
    assert torch.all(sel.kv_head_mix == 1)
    frame = sel.q_proj.permute(1, 0, 2).reshape(8, 8) * 8 ** 0.25
    assert torch.allclose(frame.T @ frame, torch.eye(8), atol=1e-5)
    assert torch.equal(sel.q_proj, sel.k_proj)


def test_selector_initialisation_is_bit_identical_to_reference():
    """``tests/golden/selector_init.npz`` holds the reference selector's own
    initial parameters under fixed seeds (narrow, benchmark and wide router)."""
    import numpy as np

    fixture = np.load(ROOT / "tests" / "golden" / "selector_init.npz")
    for i in range(3):
        h, g, d, rh, rd = (int(x) for x in fixture[f"{i}_shape"])
        torch.manual_seed(int(fixture[f"{i}_seed"]))
        sel = lsb.LeanSelectSelector(num_heads=h, num_kv_heads=g, head_dim=d, router_heads=rh,
                                     router_dim=rd)
        for name in ("head_mix", "kv_head_mix", "q_proj", "k_proj"):
            assert np.array_equal(getattr(sel, name).detach().numpy(), fixture[f"{i}_{name}"]), \
                (i, name)


@pytest.mark.parametrize("shape", [(8, 2, 8, 2, 4), (32, 2, 128, 4, 32)])
def test_full_width_initialisation_is_scaled_head_mean_dot(shape):
    """The reference's known answer (test_core.py:59-65): at router width
    R*r = head_dim the initial selector scores query n against atom a as the
    group-mean query dotted with the key, over sqrt(head_dim).  Checked for
    the reference test's shape and for the benchmark's (32/2 heads, D 128,
    4 x 32 router), through the folded weights the kernels consume."""
    import numpy as np

    from oracle import leanselect_oracle as ora

    h, g, d, rh, rd = shape
    torch.manual_seed(11)
    sel = lsb.LeanSelectSelector(num_heads=h, num_kv_heads=g, head_dim=d, router_heads=rh,
                                 router_dim=rd)
    params = ora.SelectorParams(*(getattr(sel, name).detach().numpy()
                                  for name in ("head_mix", "kv_head_mix", "q_proj", "k_proj")))
    rng = np.random.default_rng(4)
    q = rng.standard_normal((3, h, d)).astype(np.float32)
    k = rng.standard_normal((7, g, d)).astype(np.float32)
    q_fused, kv_fused = ora.fold_weights(params)
    actual = ora.atom_scores(ora.project_queries(q, q_fused, g), ora.project_atom_keys(k, kv_fused))
    expected = np.einsum("ngd,agd->gna", q.reshape(3, g, h // g, d).mean(2), k) / np.sqrt(d)
    np.testing.assert_allclose(actual, expected, atol=1e-5, rtol=1e-4)


def test_reference_budget_mapping():
    """Budget arithmetic of load_model / the attention module (minicpm.py:1965-1966)."""
    cfg = lsb.LayerConfig()
    assert (cfg.topk, cfg.local_blocks, cfg.init_blocks) == (67, 2, 1)
    assert lsb.ops.atom_count(31) == 0 and lsb.ops.atom_count(32768) == 2047


def test_uniform_and_atom_score_entry_points_validate_on_host():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    # 2 groups x (16 heads x 128 x 128 bf16 weights, padded) + Ks + selection workspace
    need = lib.ls_uniform_select_workspace_bytes(1000, 61, 32, 2, 1000)
    assert need == 32 * 128 * 128 * 2 + (2 * 61 * 128 * 2 + 255) // 256 * 256 + 2 * 1000 * 16 * 2
    rc = lib.ls_uniform_select_pages(fake, fake, fake, fake, 1, 1000, 1000, 61, 32, 2, 128, 35, 1,
                                     2, 64, 16, 0.0, fake, fake, need - 1, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT and b"workspace" in lib.ls_last_error()
    rc = lib.ls_uniform_select_pages(fake, fake, fake, fake, 1, 1000, 1000, 61, 32, 2, 64, 35, 1,
                                     2, 64, 16, 0.0, fake, fake, need, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # head_dim 64
    rc = lib.ls_uniform_select_pages(None, fake, fake, fake, 1, 1000, 1000, 61, 32, 2, 128, 35, 1,
                                     2, 64, 16, 0.0, fake, fake, need, None, None)
    assert rc == _native.LS_ERR_INVALID_ARGUMENT
    rc = lib.ls_atom_scores(fake, fake, fake, fake, fake, 1, 1000, 1000, 61, 32, 2, 128, 64, 61,
                            fake, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # selector width 64
    rc = lib.ls_sparse_attn_gather_only(fake, fake, fake, fake, fake, 1, 64, 64, 64, 64, 24, 2, 128,
                                        fake, 4, 64, 1, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED  # 12 heads per group


def test_noalloc_rejects_oversize_requests_on_host():
    lib = _native.load()
    fake = ctypes.c_void_p(1 << 20)
    # one 2-group sequence of 64K tokens needs 2 x 65536 x 1024 x 4 bytes = 512 MiB > 16 MiB
    rc = lib.ls_select_pages_noalloc(fake, fake, fake, fake, fake, 1, 65536, 65536, 4095, 32, 2,
                                     128, 128, 67, 1, 2, 64, 16, fake, None, None)
    assert rc == _native.LS_ERR_UNSUPPORTED
    assert b"scratch" in lib.ls_last_error()
