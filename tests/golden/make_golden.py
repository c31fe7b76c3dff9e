"""Write the golden fixtures that pin the oracle to the LeanSelect reference.

Run in a container where the reference source tree is available::

    LEANSELECT_REFERENCE=/path/to/LeanSelect python tests/golden/make_golden.py

It imports the reference's own hot-path code (``leanselect.pages``,
``leanselect.selector`` and ``MiniCPMInfLLMv2Attention._lightweight_compressed_attention``
called unbound on a namespace, the same trick the reference tests rely on),
runs it on seeded inputs and stores inputs (or their seeds and checksums) and
outputs as compressed ``.npz`` files next to this script.  The tests only read
the fixtures; nothing at test or bench time touches the reference tree.
"""
from __future__ import annotations

import hashlib
import math
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
REFERENCE = os.environ.get("LEANSELECT_REFERENCE")
if not REFERENCE:
    raise SystemExit("set LEANSELECT_REFERENCE to the LeanSelect source tree")
sys.path.insert(0, REFERENCE)

from oracle import leanselect_oracle as ora  # noqa: E402

from leanselect.pages import compress_keys_mean, pool_atoms_to_pages  # noqa: E402
from leanselect.selector import LeanSelectSelector  # noqa: E402
from leanselect.models.minicpm import CompressK, MiniCPMInfLLMv2Attention  # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def make_selector(params: ora.SelectorParams) -> LeanSelectSelector:
    sel = LeanSelectSelector(num_heads=params.num_heads, num_kv_heads=params.num_kv_heads,
                             head_dim=params.head_dim, router_heads=params.q_proj.shape[0],
                             router_dim=params.q_proj.shape[2])
    with torch.no_grad():
        sel.head_mix.copy_(torch.from_numpy(params.head_mix))
        sel.kv_head_mix.copy_(torch.from_numpy(params.kv_head_mix))
        sel.q_proj.copy_(torch.from_numpy(params.q_proj))
        sel.k_proj.copy_(torch.from_numpy(params.k_proj))
    return sel.float()


def reference_select(sel, q, kc, cu_q, cu_c, *, topk, init_blocks, local_blocks,
                     block_size=64, kernel_stride=16):
    ns = SimpleNamespace(selection_method="leanselect", leanselect=sel, block_size=block_size,
                         topk=topk, local_blocks=local_blocks, init_blocks=init_blocks,
                         num_key_value_heads=sel.num_kv_heads, kernel_stride=kernel_stride)
    with torch.no_grad():
        out = MiniCPMInfLLMv2Attention._lightweight_compressed_attention(
            ns, q, kc, torch.as_tensor(cu_q, dtype=torch.int32),
            torch.as_tensor(cu_c, dtype=torch.int32), int(np.diff(cu_q).max()))
    return np.sort(np.where(out.numpy() < 0, np.iinfo(np.int32).max, out.numpy()), axis=-1)


def canon(idx):
    idx = np.sort(np.where(idx < 0, np.iinfo(np.int32).max, idx), axis=-1)
    return np.where(idx == np.iinfo(np.int32).max, -1, idx).astype(np.int32)


def known_answers():
    """The reference's known answers for page pooling (tests/test_core.py:68-76)."""
    a = pool_atoms_to_pages(torch.arange(15).float(), seq_len=256).numpy()
    atom = torch.zeros(31)
    atom[19] = 1
    b = pool_atoms_to_pages(atom, seq_len=512).numpy()
    rng = np.random.default_rng(11)
    rand_atoms = rng.standard_normal((3, 5, 37)).astype(np.float32)
    c = pool_atoms_to_pages(torch.from_numpy(rand_atoms), seq_len=37 * 16 + 16 + 5).numpy()
    np.savez_compressed(HERE / "pool_known.npz", arange15_seq256=a, hot19_seq512=b,
                        rand_atoms=rand_atoms, rand_seq_len=np.int64(37 * 16 + 16 + 5),
                        rand_pages=c)


def compression_cases():
    """``CompressK`` and ``compress_keys_mean`` on packed ragged sequences."""
    rng = np.random.default_rng(5)
    lens = [100, 31, 64, 300, 32, 47, 1]
    total = sum(lens)
    k = rng.standard_normal((total, 2, 16)).astype(np.float32)
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    module = CompressK(2, 16, kernel_size=32, kernel_stride=16)
    kc, cu_c = module(torch.from_numpy(k), torch.from_numpy(cu))
    kc_bf16, _ = module(torch.from_numpy(k).bfloat16(), torch.from_numpy(cu))
    mean_kc = compress_keys_mean(torch.from_numpy(k[:300])[None]).numpy()[0]
    mean_short = compress_keys_mean(torch.from_numpy(k[:20])[None]).numpy()[0]
    # Also the 128/64 compressor the backbone instantiates (minicpm.py:2790).
    kc2, cu_c2 = CompressK(2, 16, kernel_size=128, kernel_stride=64)(
        torch.from_numpy(k), torch.from_numpy(cu))
    np.savez_compressed(
        HERE / "compress.npz", k=k, cu_seqlens=cu, kc=kc.numpy(), cu_c=cu_c.numpy(),
        kc_bf16=kc_bf16.float().numpy(), mean_kc_300=mean_kc, mean_short_20=mean_short,
        kc_128_64=kc2.numpy(), cu_c_128_64=cu_c2.numpy())


def selector_cases():
    """Folding and projections, fp32 and bf16, on a small selector."""
    rng = np.random.default_rng(9)
    params = ora.selector_params(8, 2, 16, 2, 4, rng)
    params.head_mix = rng.standard_normal((8, 2)).astype(np.float32) / math.sqrt(2)
    params.kv_head_mix = (1.0 + 0.1 * rng.standard_normal((2, 2))).astype(np.float32)
    sel = make_selector(params)
    q = rng.standard_normal((200, 8, 16)).astype(np.float32)
    kc = rng.standard_normal((11, 2, 16)).astype(np.float32)
    with torch.no_grad():
        qf, kf = sel.fused_weights()
        qf16, kf16 = sel.fused_weights(dtype=torch.bfloat16)
        qs = sel.project_queries(torch.from_numpy(q)).numpy()
        ks = sel.project_atom_keys(torch.from_numpy(kc)).numpy()
        pages = sel.score_pages(torch.from_numpy(q), torch.from_numpy(kc), seq_len=200,
                                block_size=64, kernel_stride=16).numpy()
        qb = torch.from_numpy(q).bfloat16()
        kb = torch.from_numpy(kc).bfloat16()
        qs16 = sel.project_queries(qb).float().numpy()
        ks16 = sel.project_atom_keys(kb).float().numpy()
    np.savez_compressed(
        HERE / "selector.npz", head_mix=params.head_mix, kv_head_mix=params.kv_head_mix,
        q_proj=params.q_proj, k_proj=params.k_proj, q=q, kc=kc, q_fused=qf.numpy(),
        kv_fused=kf.numpy(), q_fused_bf16=qf16.float().numpy(),
        kv_fused_bf16=kf16.float().numpy(), qs=qs, ks=ks, pages=pages, qs_bf16=qs16,
        ks_bf16=ks16)


def selection_cases():
    """``_lightweight_compressed_attention`` outputs on small packed batches."""
    cases = {}
    specs = [
        # name, lens, H, G, D, R, r, topk(total), init, local
        ("tiny_single", [256], 4, 2, 16, 2, 8, 3, 1, 1),
        ("ragged_pack", [300, 130, 20, 700, 64, 65], 8, 2, 32, 4, 8, 6, 1, 2),
        ("wide_budget", [500], 8, 2, 32, 4, 8, 40, 1, 2),
        ("no_local", [640, 257], 8, 2, 32, 4, 8, 5, 1, 0),
        ("two_sinks", [900], 8, 2, 32, 4, 8, 7, 2, 3),
        ("gqa8_d128", [1000, 1500], 16, 2, 128, 4, 32, 12, 1, 2),
    ]
    for name, lens, h, g, d, rh, rd, topk, init, local in specs:
        seed = sum(ord(c) for c in name)
        inputs = ora.synthetic_layer(lens, num_heads=h, num_kv_heads=g, head_dim=d,
                                     router_heads=rh, router_dim=rd, hot_pages=3, seed=seed)
        kc_t, cu_c_t = CompressK(g, d, kernel_size=32, kernel_stride=16)(
            torch.from_numpy(inputs.k), torch.from_numpy(inputs.cu_seqlens))
        kc, cu_c = kc_t.numpy(), cu_c_t.numpy()
        sel = make_selector(inputs.params)
        idx = reference_select(sel, torch.from_numpy(inputs.q), torch.from_numpy(kc),
                               inputs.cu_seqlens, cu_c, topk=topk, init_blocks=init,
                               local_blocks=local)
        # Inputs are regenerated from (lens, heads, seed) by the oracle generator;
        # their digest guards against a changed random stream.
        cases[name] = dict(lens=np.array(lens, dtype=np.int64),
                           dims=np.array([h, g, d, rh, rd], dtype=np.int64),
                           seed=np.int64(seed),
                           input_digest=np.array(digest(inputs.q, inputs.k, inputs.v)),
                           kc_digest=np.array(digest(kc)), cu_c=cu_c,
                           topk=np.int64(topk), init=np.int64(init), local=np.int64(local),
                           idx=canon(idx).astype(np.int16))
    flat = {f"{name}__{key}": value for name, case in cases.items() for key, value in case.items()}
    flat["names"] = np.array(list(cases))
    np.savez_compressed(HERE / "selection_small.npz", **flat)


def config0_case():
    """benchmark config 0 (N=8192, 32/2 heads, D=128, T=35, fp32) via the reference.

    The inputs are regenerated from the seed by the oracle generator; the
    fixture keeps their SHA-256 so a changed random stream fails loudly.
    A row subset of the reference's ``topk_idx`` is stored.
    """
    inputs = ora.synthetic_layer([8192], seed=0)
    kc_ref, cu_c = CompressK(2, 128, kernel_size=32, kernel_stride=16)(
        torch.from_numpy(inputs.k), torch.from_numpy(inputs.cu_seqlens))
    sel = make_selector(inputs.params)
    idx = reference_select(sel, torch.from_numpy(inputs.q), kc_ref, inputs.cu_seqlens,
                           cu_c.numpy(), topk=35, init_blocks=1, local_blocks=2)
    rows = np.unique(np.concatenate([np.arange(0, 8192, 7), np.arange(8192 - 256, 8192)]))
    np.savez_compressed(
        HERE / "config0.npz", seed=np.int64(0), rows=rows.astype(np.int32),
        idx_rows=canon(idx)[:, rows].astype(np.int16),
        input_digest=np.array(digest(inputs.q, inputs.k, inputs.v)),
        kc_digest=np.array(digest(kc_ref.numpy())), kc_rows=kc_ref.numpy()[::50])


def bf16_selection_case():
    """A bf16 run of the reference selection, to pin the bf16 rounding points."""
    inputs = ora.synthetic_layer([1024], seed=3, bf16=True)
    kc_ref, cu_c = CompressK(2, 128, kernel_size=32, kernel_stride=16)(
        torch.from_numpy(inputs.k).bfloat16(), torch.from_numpy(inputs.cu_seqlens))
    sel = make_selector(inputs.params)
    q16 = torch.from_numpy(inputs.q).bfloat16()
    with torch.no_grad():
        qs = sel.project_queries(q16).float().numpy()
        ks = sel.project_atom_keys(kc_ref).float().numpy()
    idx = reference_select(sel, q16, kc_ref, inputs.cu_seqlens, cu_c.numpy(), topk=19,
                           init_blocks=1, local_blocks=2)
    np.savez_compressed(
        HERE / "bf16_selection.npz", seed=np.int64(3),
        input_digest=np.array(digest(inputs.q, inputs.k, inputs.v)),
        kc=kc_ref.float().numpy(), qs=qs, ks=ks, idx=canon(idx),
        page_bits=reference_page_scores(sel, q16, kc_ref, 1024))


def reference_page_scores(sel, q, kc, seq_len):
    """The reference's pooled page scores (``score_pages``, selector.py:192-214), bf16 bits."""
    with torch.no_grad():
        pages = sel.score_pages(q, kc, seq_len=seq_len, block_size=64, kernel_stride=16)
    return pages.contiguous().view(torch.int16).numpy()


def stock_budget_cases():
    """bf16 selection at the reference's stock budget and at the benchmark's.

    The reference's defaults are ``window_size=2048`` -> ``local_blocks=32``
    and ``topk = 64 + 32 = 96`` (models/__init__.py:119-127,
    minicpm.py:1957-1966).  Cases: one 8192-token sequence and a ragged pack
    with sequences shorter than the 33 forced pages, at T=96 / local 32; and
    one 16384-token sequence at the benchmark budget T=67 / local 2.  A row
    sample of each ``topk_idx`` is stored, with the reference's own bf16
    page scores of those rows (to pin scoring and selection separately).
    """
    out = {}
    specs = [
        # name, lens, topk, init, local, seed
        ("stock_8k", [8192], 96, 1, 32, 31),
        ("stock_ragged", [3000, 1500, 64, 20, 2100, 900], 96, 1, 32, 32),
        ("bench_16k", [16384], 67, 1, 2, 33),
    ]
    for name, lens, topk, init, local, seed in specs:
        inputs = ora.synthetic_layer(lens, seed=seed, bf16=True)
        q16 = torch.from_numpy(inputs.q).bfloat16()
        kc_ref, cu_c = CompressK(2, 128, kernel_size=32, kernel_stride=16)(
            torch.from_numpy(inputs.k).bfloat16(), torch.from_numpy(inputs.cu_seqlens))
        sel = make_selector(inputs.params)
        idx = canon(reference_select(sel, q16, kc_ref, inputs.cu_seqlens, cu_c.numpy(), topk=topk,
                                     init_blocks=init, local_blocks=local))
        rows, scores = [], []
        cu, cc = inputs.cu_seqlens, cu_c.numpy()
        for b, n in enumerate(lens):
            r = np.unique(np.concatenate([np.arange(0, n, 7), np.arange(max(0, n - 32), n)]))
            rows.append(r + cu[b])
            if cc[b + 1] > cc[b]:
                bits = reference_page_scores(sel, q16[cu[b]:cu[b] + n], kc_ref[cc[b]:cc[b + 1]], n)
                scores.append(bits[:, r[::4]])
        rows = np.concatenate(rows).astype(np.int32)
        out[f"{name}__lens"] = np.array(lens, dtype=np.int64)
        out[f"{name}__seed"] = np.int64(seed)
        out[f"{name}__topk"] = np.int64(topk)
        out[f"{name}__init"] = np.int64(init)
        out[f"{name}__local"] = np.int64(local)
        out[f"{name}__input_digest"] = np.array(digest(inputs.q, inputs.k, inputs.v))
        out[f"{name}__kc"] = kc_ref.view(torch.int16).numpy()
        out[f"{name}__cu_c"] = cc
        out[f"{name}__rows"] = rows
        out[f"{name}__idx_rows"] = idx[:, rows].astype(np.int16)
        # Page scores of every 4th sampled row of each sequence with atoms,
        # concatenated along the row axis and padded to the widest row.
        width = max(s.shape[-1] for s in scores)
        padded = [np.pad(s, ((0, 0), (0, 0), (0, width - s.shape[-1])), constant_values=-128)
                  for s in scores]   # -128 = 0xFF80, bf16 -inf
        out[f"{name}__page_bits"] = np.concatenate(padded, axis=1)
    out["names"] = np.array([s[0] for s in specs])
    np.savez_compressed(HERE / "stock_budget.npz", **out)


def uniform_cases():
    """``uniform_prefill_topk_idx`` (ops/uniform.py:185-320) on small packed batches.

    fp32 and bf16 inputs; equal-packed and ragged batches; a sequence too
    short for any atom; two sinks; no local pages.
    """
    from leanselect.ops.uniform import uniform_prefill_topk_idx

    cases = {}
    specs = [
        # name, lens, H, G, D, topk, init, local, bf16
        ("ragged_fp32", [700, 1500, 20, 64], 8, 2, 32, 12, 1, 2, False),
        ("ragged_bf16", [700, 1500, 20, 64], 8, 2, 32, 12, 1, 2, True),
        ("equal_bf16_d128", [1024, 1024], 16, 2, 128, 20, 1, 2, True),
        ("two_sinks", [900], 8, 2, 32, 7, 2, 3, True),
        ("no_local", [640, 257], 8, 2, 32, 5, 1, 0, True),
    ]
    for name, lens, h, g, d, topk, init, local, bf16 in specs:
        seed = sum(ord(c) for c in name)
        inputs = ora.synthetic_layer(lens, num_heads=h, num_kv_heads=g, head_dim=d,
                                     router_heads=4, router_dim=d // 4, hot_pages=3, seed=seed,
                                     bf16=bf16)
        dtype = torch.bfloat16 if bf16 else torch.float32
        kc_t, cu_c_t = CompressK(g, d, kernel_size=32, kernel_stride=16)(
            torch.from_numpy(inputs.k).to(dtype), torch.from_numpy(inputs.cu_seqlens))
        with torch.no_grad():
            idx, _ = uniform_prefill_topk_idx(
                torch.from_numpy(inputs.q).to(dtype), kc_t,
                cu_seqlens_q=torch.from_numpy(inputs.cu_seqlens), cu_seqlens_k=cu_c_t,
                max_seqlen_q=max(lens), topk=topk, block_size=64, kernel_stride=16,
                init_blocks=init, local_blocks=local)
        cases[name] = dict(lens=np.array(lens, dtype=np.int64),
                           dims=np.array([h, g, d], dtype=np.int64), seed=np.int64(seed),
                           bf16=np.bool_(bf16),
                           input_digest=np.array(digest(inputs.q, inputs.k, inputs.v)),
                           kc_digest=np.array(digest(kc_t.float().numpy())),
                           cu_c=cu_c_t.numpy(), topk=np.int64(topk), init=np.int64(init),
                           local=np.int64(local), idx=canon(idx.numpy()).astype(np.int16))
    flat = {f"{name}__{key}": value for name, case in cases.items() for key, value in case.items()}
    flat["names"] = np.array(list(cases))
    np.savez_compressed(HERE / "uniform_selection.npz", **flat)


def nosa_atom_score_cases():
    """NOSA's ``LlamaSdpaAttention._leanselect_atom_scores`` (nosa.py:1822-1853), bf16.

    Called unbound on a namespace carrying the selector and the KV-head count,
    on a ragged pack that includes a sequence too short for any atom.
    """
    from leanselect.models.nosa import LlamaSdpaAttention

    lens = [700, 20, 1333]
    inputs = ora.synthetic_layer(lens, num_heads=32, num_kv_heads=2, head_dim=128,
                                 router_heads=4, router_dim=32, hot_pages=3, seed=97, bf16=True)
    kc, cu_c = CompressK(2, 128, kernel_size=32, kernel_stride=16)(
        torch.from_numpy(inputs.k).bfloat16(), torch.from_numpy(inputs.cu_seqlens))
    sel = make_selector(inputs.params)  # fp32 parameters, bf16 activations (fused_weights casts)
    ns = SimpleNamespace(leanselect=sel, num_key_value_heads=2)
    with torch.no_grad():
        scores = LlamaSdpaAttention._leanselect_atom_scores(
            ns, torch.from_numpy(inputs.q).bfloat16(), kc, torch.from_numpy(inputs.cu_seqlens),
            cu_c)
    np.savez_compressed(
        HERE / "nosa_atom_scores.npz", seed=np.int64(97), lens=np.array(lens, dtype=np.int64),
        input_digest=np.array(digest(inputs.q, inputs.k, inputs.v)), cu_c=cu_c.numpy(),
        scores_bits=scores.view(torch.int16).numpy())


def selector_init_cases():
    """Default initialisation (``reset_parameters``, selector.py:112-137) under fixed seeds:
    the reference test's shape, the benchmark's, and a router wider than head_dim."""
    out = {}
    shapes = [(8, 2, 8, 2, 4), (32, 2, 128, 4, 32), (8, 2, 16, 8, 4)]
    for i, (h, g, d, rh, rd) in enumerate(shapes):
        torch.manual_seed(100 + i)
        sel = LeanSelectSelector(num_heads=h, num_kv_heads=g, head_dim=d, router_heads=rh,
                                 router_dim=rd)
        for name in ("head_mix", "kv_head_mix", "q_proj", "k_proj"):
            out[f"{i}_{name}"] = getattr(sel, name).detach().numpy()
        out[f"{i}_shape"] = np.array([h, g, d, rh, rd], dtype=np.int64)
        out[f"{i}_seed"] = np.int64(100 + i)
    np.savez_compressed(HERE / "selector_init.npz", **out)

CASES = {
    "known_answers": known_answers,
    "compression": compression_cases,
    "selector": selector_cases,
    "selection": selection_cases,
    "config0": config0_case,
    "bf16_selection": bf16_selection_case,
    "stock_budget": stock_budget_cases,
    "uniform": uniform_cases,
    "nosa": nosa_atom_score_cases,
    "selector_init": selector_init_cases,
}

if __name__ == "__main__":
    # With arguments only the named cases are (re)written.
    wanted = sys.argv[1:] or list(CASES)
    for name in wanted:
        torch.manual_seed(0)
        CASES[name]()
    for path in sorted(HERE.glob("*.npz")):
        print(path.name, path.stat().st_size)
