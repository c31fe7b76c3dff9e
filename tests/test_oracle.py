"""The CPU oracle against the reference's golden fixtures (no GPU needed).

Fixtures come from ``tests/golden/make_golden.py``, which ran the reference's
own code.  Stage-2 attention has no runnable reference, so its restatement is
checked against ``torch.nn.functional.scaled_dot_product_attention`` with an
explicit mask built from the page lists.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import leanselect_oracle as ora

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_pool_known_answers():
    """tests/test_core.py:68-76 of the reference, plus a random case."""
    g = load("pool_known.npz")
    np.testing.assert_array_equal(
        ora.pool_atoms_to_pages(np.arange(15, dtype=np.float32), 256), g["arange15_seq256"])
    assert g["arange15_seq256"].tolist() == [3.0, 7.0, 11.0, 14.0]
    atom = np.zeros(31, dtype=np.float32)
    atom[19] = 1
    pages = ora.pool_atoms_to_pages(atom, 512)
    np.testing.assert_array_equal(pages, g["hot19_seq512"])
    assert np.nonzero(pages)[0].tolist() == [4, 5]
    np.testing.assert_array_equal(
        ora.pool_atoms_to_pages(g["rand_atoms"], int(g["rand_seq_len"])), g["rand_pages"])


def test_compression_matches_compressk():
    g = load("compress.npz")
    kc, cu_c = ora.compress_keys(g["k"], g["cu_seqlens"])
    np.testing.assert_array_equal(cu_c, g["cu_c"])
    np.testing.assert_allclose(kc, g["kc"], rtol=1e-6, atol=1e-6)
    # bf16 policy: CompressK on bf16 keys returns bf16; allow one bf16 ulp
    # (torch's and the oracle's fp32 summation orders differ).
    kb, _ = ora.compress_keys(ora.bf16_round(g["k"]), g["cu_seqlens"], policy="bf16")
    np.testing.assert_allclose(kb, g["kc_bf16"], rtol=2 ** -7, atol=1e-6)
    assert np.mean(kb == g["kc_bf16"]) > 0.95
    # compress_keys_mean over one long sequence is the same math.
    kc300, _ = ora.compress_keys(g["k"][:300], np.array([0, 300]))
    np.testing.assert_allclose(kc300, g["mean_kc_300"], rtol=1e-6, atol=1e-6)
    # The 128/64 compressor instantiated by the backbone.
    kc2, cu2 = ora.compress_keys(g["k"], g["cu_seqlens"], kernel_size=128, kernel_stride=64)
    np.testing.assert_array_equal(cu2, g["cu_c_128_64"])
    np.testing.assert_allclose(kc2, g["kc_128_64"], rtol=1e-6, atol=1e-6)


def test_short_sequences_have_no_atoms():
    """CompressK keeps no window for sequences shorter than kernel_size."""
    assert ora.atom_count(31) == 0
    assert ora.atom_count(32) == 1
    assert ora.atom_count(47) == 1
    assert ora.atom_count(48) == 2
    cu = ora.compressed_cu_seqlens(np.array([0, 20, 52, 52, 152]))
    assert cu.tolist() == [0, 0, 1, 1, 6]


def test_folding_and_projections():
    g = load("selector.npz")
    params = ora.SelectorParams(g["head_mix"], g["kv_head_mix"], g["q_proj"], g["k_proj"])
    qf, kf = ora.fold_weights(params)
    np.testing.assert_array_equal(qf, g["q_fused"])
    np.testing.assert_array_equal(kf, g["kv_fused"])
    qf16, kf16 = ora.fold_weights(params, "bf16")
    np.testing.assert_array_equal(qf16, g["q_fused_bf16"])
    np.testing.assert_array_equal(kf16, g["kv_fused_bf16"])
    qs = ora.project_queries(g["q"], qf, 2)
    ks = ora.project_atom_keys(g["kc"], kf)
    np.testing.assert_allclose(qs, g["qs"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(ks, g["ks"], rtol=1e-5, atol=1e-5)
    pages = ora.score_pages(g["q"], g["kc"], params, seq_len=200)
    np.testing.assert_allclose(pages, g["pages"], rtol=1e-5, atol=1e-5)
    # bf16 rounding points (project_* return bf16 in the model dtype).
    qs16 = ora.project_queries(ora.bf16_round(g["q"]), qf16, 2, "bf16")
    ks16 = ora.project_atom_keys(ora.bf16_round(g["kc"]), kf16, "bf16")
    np.testing.assert_allclose(qs16, g["qs_bf16"], rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(ks16, g["ks_bf16"], rtol=2 ** -7, atol=1e-6)
    assert np.mean(qs16 == g["qs_bf16"]) > 0.97


def _params_from(case, name):
    h, gq, d, rh, rd = (int(x) for x in case[f"{name}__dims"])
    return h, gq, d, rh, rd


SELECTION_CASES = ["tiny_single", "ragged_pack", "wide_budget", "no_local", "two_sinks",
                   "gqa8_d128"]


@pytest.mark.parametrize("name", SELECTION_CASES)
def test_selection_matches_reference(name):
    g = load("selection_small.npz")
    h, gq, d, rh, rd = _params_from(g, name)
    lens = g[f"{name}__lens"].tolist()
    inputs = ora.synthetic_layer(lens, num_heads=h, num_kv_heads=gq, head_dim=d,
                                 router_heads=rh, router_dim=rd, hot_pages=3,
                                 seed=int(g[f"{name}__seed"]))
    assert digest(inputs.q, inputs.k, inputs.v) == str(g[f"{name}__input_digest"])
    kc, cu_c = ora.compress_keys(inputs.k, inputs.cu_seqlens)
    np.testing.assert_array_equal(cu_c, g[f"{name}__cu_c"])
    sel = ora.lightweight_compressed_attention(
        inputs.q, kc, inputs.cu_seqlens, cu_c, inputs.params, topk=int(g[f"{name}__topk"]),
        init_blocks=int(g[f"{name}__init"]), local_blocks=int(g[f"{name}__local"]))
    expected = g[f"{name}__idx"].astype(np.int32)
    assert sel.topk_idx.shape == expected.shape
    bad = ora.selection_mismatches(expected, sel)
    assert not bad, bad[:5]
    # Adjacent pages share one atom of their 5-atom windows, so exact score
    # ties are common; torch breaks them differently from the oracle's
    # lowest-page-wins rule.  Most rows still agree exactly.
    exact = np.mean(np.all(np.sort(sel.topk_idx, -1) == np.sort(expected, -1), -1))
    assert exact > 0.9


def test_config0_selection_matches_reference():
    """benchmark config 0 (fp32, N=8192, T=35) against the reference's topk_idx."""
    g = load("config0.npz")
    inputs = ora.synthetic_layer([8192], seed=int(g["seed"]))
    assert digest(inputs.q, inputs.k, inputs.v) == str(g["input_digest"])
    kc, cu_c = ora.compress_keys(inputs.k, inputs.cu_seqlens)
    np.testing.assert_allclose(kc[::50], g["kc_rows"], rtol=1e-5, atol=1e-6)
    rows = g["rows"]
    sel = ora.lightweight_compressed_attention(inputs.q, kc, inputs.cu_seqlens, cu_c,
                                               inputs.params, topk=35)
    expected = np.full_like(sel.topk_idx, -1)
    expected[:, rows] = g["idx_rows"].astype(np.int32)
    sub = ora.Selection(sel.topk_idx[:, rows], sel.boundary[:, rows],
                        [(0, sel.page_scores[0][1][:, rows])])
    bad = ora.selection_mismatches(expected[:, rows], sub)
    assert not bad, bad[:5]


def test_bf16_selection_matches_reference():
    """Reference run on bf16 tensors: rounding points and the selected sets."""
    g = load("bf16_selection.npz")
    inputs = ora.synthetic_layer([1024], seed=int(g["seed"]), bf16=True)
    assert digest(inputs.q, inputs.k, inputs.v) == str(g["input_digest"])
    kc, cu_c = ora.compress_keys(inputs.k, inputs.cu_seqlens, policy="bf16")
    np.testing.assert_allclose(kc, g["kc"], rtol=2 ** -7, atol=1e-6)
    qf, kf = ora.fold_weights(inputs.params, "bf16")
    qs = ora.project_queries(inputs.q, qf, 2, "bf16")
    ks = ora.project_atom_keys(g["kc"], kf, "bf16")
    np.testing.assert_allclose(qs, g["qs"], rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(ks, g["ks"], rtol=2 ** -7, atol=1e-6)
    sel = ora.lightweight_compressed_attention(inputs.q, g["kc"], inputs.cu_seqlens, cu_c,
                                               inputs.params, topk=19, policy="bf16")
    # Atom scores are rounded to bf16 as the reference rounds them, so the
    # sets differ only by exact ties at the budget boundary (torch.topk
    # breaks them its own way), inside north_star's 1e-3 band.
    bad = ora.selection_mismatches(g["idx"], sel, rel_tol=1e-3)
    assert not bad, bad[:5]
    # The reference's own page scores (bf16) against the oracle's.
    ref_pages = ora.from_bf16_bits(g["page_bits"].view(np.uint16))
    mine = ora.score_pages(inputs.q, g["kc"], inputs.params, seq_len=1024, policy="bf16")
    err = np.abs(mine - ref_pages)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
    assert np.mean(err == 0) > 0.98


def _sdpa_reference(q, k, v, cu, idx, causal=True):
    """Independent check: torch SDPA with an explicit token x key mask."""
    total, h, d = q.shape
    g = k.shape[1]
    hg = h // g
    out = np.zeros_like(q)
    for b in range(len(cu) - 1):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        n = s1 - s0
        if n == 0:
            continue
        mask = np.zeros((g, n, n), dtype=bool)
        for gi in range(g):
            for t in range(n):
                for p in idx[gi, s0 + t]:
                    if p >= 0:
                        mask[gi, t, p * 64:min(p * 64 + 64, n)] = True
        if causal:
            mask &= np.tril(np.ones((n, n), dtype=bool))[None]
        qt = torch.from_numpy(q[s0:s1]).double().permute(1, 0, 2)
        kt = torch.from_numpy(k[s0:s1]).double().permute(1, 0, 2).repeat_interleave(hg, 0)
        vt = torch.from_numpy(v[s0:s1]).double().permute(1, 0, 2).repeat_interleave(hg, 0)
        m = torch.from_numpy(mask).repeat_interleave(hg, 0)
        o = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=m)
        o = torch.where(m.any(-1, keepdim=True), o, torch.zeros_like(o))
        out[s0:s1] = o.permute(1, 0, 2).float().numpy()
    return out


def test_sparse_attention_matches_sdpa_with_page_mask():
    inputs = ora.synthetic_layer([200, 77, 130], num_heads=8, num_kv_heads=2, head_dim=32,
                                 router_heads=4, router_dim=8, hot_pages=1, seed=4)
    rng = np.random.default_rng(1)
    total = inputs.q.shape[0]
    idx = rng.integers(-1, 4, size=(2, total, 3)).astype(np.int32)
    idx[:, :, 0] = 0
    out, lse = ora.sparse_attention(inputs.q, inputs.k, inputs.v, inputs.cu_seqlens,
                                    inputs.cu_seqlens, idx)
    ref = _sdpa_reference(inputs.q, inputs.k, inputs.v, inputs.cu_seqlens, idx)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)
    assert np.isfinite(lse).all()


def test_sparse_attention_all_pages_is_dense_causal():
    inputs = ora.synthetic_layer([300], num_heads=4, num_kv_heads=2, head_dim=16,
                                 router_heads=2, router_dim=8, hot_pages=1, seed=8)
    idx = np.broadcast_to(np.arange(5, dtype=np.int32), (2, 300, 5)).copy()
    out, _ = ora.sparse_attention(inputs.q, inputs.k, inputs.v, inputs.cu_seqlens,
                                  inputs.cu_seqlens, idx)
    qt = torch.from_numpy(inputs.q).double().permute(1, 0, 2)
    kt = torch.from_numpy(inputs.k).double().permute(1, 0, 2).repeat_interleave(2, 0)
    vt = torch.from_numpy(inputs.v).double().permute(1, 0, 2).repeat_interleave(2, 0)
    ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True)
    np.testing.assert_allclose(out, ref.permute(1, 0, 2).numpy(), rtol=1e-5, atol=1e-5)


def test_sparse_attention_edge_rows():
    """Empty selections give zeros and lse=+inf; duplicates count once."""
    inputs = ora.synthetic_layer([130], num_heads=4, num_kv_heads=2, head_dim=16,
                                 router_heads=2, router_dim=8, hot_pages=1, seed=2)
    idx = np.full((2, 130, 3), -1, dtype=np.int32)
    idx[:, 70, :] = [1, 1, 0]
    idx[:, 71, :] = [2, 9, -1]   # page 2 is the last page; 9 is out of range
    out, lse = ora.sparse_attention(inputs.q, inputs.k, inputs.v, inputs.cu_seqlens,
                                    inputs.cu_seqlens, idx)
    assert np.all(out[0] == 0) and np.all(np.isposinf(lse[:, 0]))
    # Page 2 starts at key 128 > 71: no visible key.
    assert np.all(out[71] == 0) and np.all(np.isposinf(lse[:, 71]))
    single = idx.copy()
    single[:, 70, :] = [1, 0, -1]
    out2, _ = ora.sparse_attention(inputs.q, inputs.k, inputs.v, inputs.cu_seqlens,
                                   inputs.cu_seqlens, single)
    np.testing.assert_array_equal(out[70], out2[70])


def test_bf16_round_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 37
    x[:4] = [np.inf, -np.inf, 0.0, -0.0]
    expect = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(ora.bf16_round(x), expect)
    bits = ora.to_bf16_bits(x)
    np.testing.assert_array_equal(ora.from_bf16_bits(bits), expect)


def test_row_level_helpers_agree_with_full_oracle():
    """select_for_queries / attention_for_queries restate the packed functions on rows."""
    inp = ora.synthetic_layer([900], num_heads=8, num_kv_heads=2, head_dim=32, router_heads=4,
                              router_dim=8, hot_pages=3, seed=17, bf16=True)
    kc, cu_c = ora.compress_keys(inp.k, inp.cu_seqlens, policy="bf16")
    full = ora.lightweight_compressed_attention(inp.q, kc, inp.cu_seqlens, cu_c, inp.params,
                                                topk=9, policy="bf16")
    rows = np.array([0, 5, 64, 300, 777, 899])
    sub = ora.select_for_queries(inp.q[rows], rows, 900, kc, inp.params, take=9)
    np.testing.assert_array_equal(sub.topk_idx, full.topk_idx[:, rows])
    out, _ = ora.sparse_attention(inp.q, inp.k, inp.v, inp.cu_seqlens, inp.cu_seqlens,
                                  full.topk_idx, rows=rows)
    got = ora.attention_for_queries(inp.q[rows], rows, inp.k, inp.v, full.topk_idx[:, rows])
    np.testing.assert_allclose(got, out[rows], rtol=1e-6, atol=1e-6)


UNIFORM_CASES = ["ragged_fp32", "ragged_bf16", "equal_bf16_d128", "two_sinks", "no_local"]


@pytest.mark.parametrize("name", UNIFORM_CASES)
def test_uniform_selection_matches_reference(name):
    """The uniform method (ops/uniform.py:185-320) against the reference's own output.

    Exact score ties (adjacent pages sharing a window atom) are the only
    differences allowed: tolerance 0 beyond ``abs_floor``.
    """
    g = load("uniform_selection.npz")
    h, gq, d = (int(x) for x in g[f"{name}__dims"])
    bf16 = bool(g[f"{name}__bf16"])
    lens = g[f"{name}__lens"].tolist()
    inputs = ora.synthetic_layer(lens, num_heads=h, num_kv_heads=gq, head_dim=d, router_heads=4,
                                 router_dim=d // 4, hot_pages=3, seed=int(g[f"{name}__seed"]),
                                 bf16=bf16)
    assert digest(inputs.q, inputs.k, inputs.v) == str(g[f"{name}__input_digest"])
    policy = "bf16" if bf16 else "fp32"
    kc, cu_c = ora.compress_keys(inputs.k, inputs.cu_seqlens, policy=policy)
    np.testing.assert_array_equal(cu_c, g[f"{name}__cu_c"])
    sel = ora.uniform_prefill_topk_idx(inputs.q, kc, inputs.cu_seqlens, cu_c,
                                       topk=int(g[f"{name}__topk"]),
                                       init_blocks=int(g[f"{name}__init"]),
                                       local_blocks=int(g[f"{name}__local"]), policy=policy)
    expected = g[f"{name}__idx"].astype(np.int32)
    assert sel.topk_idx.shape == expected.shape
    bad = ora.uniform_selection_mismatches(expected, sel, rel_tol=0.0)
    assert not bad, bad[:5]
    # bf16 page scores tie often; the rows that differ differ only by ties.
    exact = np.mean(np.all(np.sort(sel.topk_idx, -1) == np.sort(expected, -1), -1))
    assert exact > 0.9


def test_uniform_future_page_takes_a_slot():
    """A query in the last stride of its page sees page q_page+1's first
    window atom; when that page makes the cut its slot stays -1."""
    n, g = 512, 1
    atoms = np.full((g, 1, ora.atom_count(n)), -5.0, dtype=np.float32)
    atoms[0, 0, 23] = 10.0   # starts at token 368; window atom of pages 5 (19..23) and 6 (23..27)
    sel, _, masked = ora.uniform_select_rows(atoms, [376], seq_len=n, take=3, topk=3,
                                             init_blocks=1, local_blocks=0)
    assert masked[0, 0, 6] == np.float32(10.0)
    assert sorted(sel[0, 0].tolist()) == [-1, 0, 5]   # sink, local page 5; page 6 dropped
    sel, _, _ = ora.uniform_select_rows(atoms, [360], seq_len=n, take=3, topk=3,
                                        init_blocks=1, local_blocks=0)
    assert sorted(sel[0, 0].tolist()) == [0, 1, 5]    # atom 23 not visible yet at token 360


def test_nosa_atom_scores_match_reference():
    """Raw atom scores of NOSA's precomputed-score path (nosa.py:1822-1853), bf16."""
    g = load("nosa_atom_scores.npz")
    lens = g["lens"].tolist()
    inputs = ora.synthetic_layer(lens, num_heads=32, num_kv_heads=2, head_dim=128, router_heads=4,
                                 router_dim=32, hot_pages=3, seed=int(g["seed"]), bf16=True)
    assert digest(inputs.q, inputs.k, inputs.v) == str(g["input_digest"])
    kc, cu_c = ora.compress_keys(inputs.k, inputs.cu_seqlens, policy="bf16")
    np.testing.assert_array_equal(cu_c, g["cu_c"])
    ref = ora.from_bf16_bits(g["scores_bits"].view(np.uint16))
    qf, kf = ora.fold_weights(inputs.params, "bf16")
    for b, n in enumerate(lens):
        q0, c0, c1 = inputs.cu_seqlens[b], cu_c[b], cu_c[b + 1]
        rows = ref[:, q0:q0 + n]
        if c1 > c0:
            want = ora.bf16_round(ora.atom_scores(
                ora.project_queries(inputs.q[q0:q0 + n], qf, 2, "bf16"),
                ora.project_atom_keys(kc[c0:c1], kf, "bf16")))
            got = rows[..., :c1 - c0]
            # Same bf16 inputs; only the fp32 accumulation order differs.
            np.testing.assert_allclose(got, want, rtol=2 ** -7, atol=2e-3)
            assert np.mean(got == want) > 0.95
        assert np.all(np.isneginf(rows[..., c1 - c0:]))


STOCK_CASES = ["stock_8k", "stock_ragged", "bench_16k"]


def _stock_case(name):
    g = load("stock_budget.npz")
    lens = g[f"{name}__lens"].tolist()
    inputs = ora.synthetic_layer(lens, seed=int(g[f"{name}__seed"]), bf16=True)
    assert digest(inputs.q, inputs.k, inputs.v) == str(g[f"{name}__input_digest"])
    kc = ora.from_bf16_bits(g[f"{name}__kc"].view(np.uint16))
    return g, lens, inputs, kc


@pytest.mark.parametrize("name", STOCK_CASES)
def test_stock_budget_selection_matches_reference(name):
    """bf16 selection at the reference's stock budget (T=96, 32 local pages,
    models/__init__.py:119-127) and at the benchmark's (T=67, local 2).

    Three pins: (1) given the reference's own bf16 page scores, the oracle's
    masking and top-k pick the reference's sets exactly (exact score ties
    aside); (2) the oracle's page scores equal the reference's except for
    rare one-ulp differences of fp32 accumulation order; (3) end to end, the
    oracle's selection differs from the reference's only by exact ties at the
    budget boundary (north_star's 1e-3 band).
    """
    g, lens, inputs, kc = _stock_case(name)
    topk, init, local = (int(g[f"{name}__{k}"]) for k in ("topk", "init", "local"))
    cu, cu_c = inputs.cu_seqlens, g[f"{name}__cu_c"]
    ekc, ecu = ora.compress_keys(inputs.k, cu, policy="bf16")
    np.testing.assert_array_equal(ecu, cu_c)
    np.testing.assert_allclose(ekc, kc, rtol=2 ** -7, atol=1e-6)
    rows = g[f"{name}__rows"]
    want = g[f"{name}__idx_rows"].astype(np.int32)
    page_bits = g[f"{name}__page_bits"].view(np.uint16)
    take = want.shape[-1]
    page_at, ulp_flips, scored = 0, 0, 0
    for b, n in enumerate(lens):
        sel_rows = rows[(rows >= cu[b]) & (rows < cu[b + 1])]
        c0, c1 = int(cu_c[b]), int(cu_c[b + 1])
        pos = sel_rows - cu[b]
        got = ora.select_for_queries(inputs.q[sel_rows], pos, n, kc[c0:c1], inputs.params,
                                     take=take, init_blocks=init, local_blocks=local)
        mine = np.isin(rows, sel_rows)
        if c1 == c0:
            assert np.all(want[:, mine] == -1)   # no atoms: the reference leaves -1
            continue
        # (3) end to end
        bad = ora.selection_mismatches(want[:, mine], got, rel_tol=1e-3)
        assert not bad, bad[:5]
        # (1) the reference's page scores through the oracle's masking + top-k
        prow = np.arange(0, len(sel_rows), 4)
        p_count = (n + 63) // 64
        ref_pages = ora.from_bf16_bits(page_bits[:, page_at:page_at + len(prow), :p_count])
        page_at += len(prow)
        from_ref = ora.select_from_scores(ref_pages, pos[prow], take=take, init_blocks=init,
                                          local_blocks=local)
        bad = ora.selection_mismatches(want[:, mine][:, prow], from_ref, rel_tol=1e-3)
        assert not bad, bad[:5]
        # (2) page scores, oracle vs reference: north_star's score tolerance,
        # and almost all of them bit-identical
        mine_pages = ora.score_pages(inputs.q[sel_rows[prow]], kc[c0:c1], inputs.params, seq_len=n,
                                     policy="bf16")
        vis = np.isfinite(ref_pages)
        assert np.array_equal(np.isfinite(mine_pages), vis)
        err = np.abs(mine_pages[vis] - ref_pages[vis])
        assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
        ulp_flips += int(np.count_nonzero(err))
        scored += int(vis.sum())
    assert ulp_flips <= 0.02 * max(scored, 1), (ulp_flips, scored)
