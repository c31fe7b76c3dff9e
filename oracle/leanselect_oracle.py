"""CPU restatement of LeanSelect's prefill hot path -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle for the CUDA kernels in ``leanselect_b200``.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker or the timed CPU
baseline.  The product path never calls it: the CUDA library fails loudly
when it is missing instead of falling back here.

Every function restates the reference algorithm in numpy and cites the
reference file:line it follows (paths relative to the LeanSelect repository).

Numeric policies
----------------
``policy="fp32"``
    Everything in fp32 semantics, like the reference run on fp32 tensors
    (benchmark config 0).  Contractions accumulate in float64 and round to
    float32, which is at least as accurate as torch's fp32 einsum.
``policy="bf16"``
    The rounding points of the reference's bf16 model path:
    ``CompressK`` returns bf16 (minicpm.py:1183-1184), ``fused_weights`` casts
    the fp32 products to the query dtype (selector.py:155-157), the bf16
    ``einsum`` calls of ``project_queries``/``project_atom_keys``
    (selector.py:177, 188-190) return bf16, and so does the scoring
    ``einsum`` (selector.py:203-207): atom scores are rounded to bf16 before
    the max-pool, exactly as the reference rounds them.  Every contraction
    here is computed exactly (float64) and rounded once; an implementation
    that accumulates in fp32 in another order can land one bf16 ulp away
    when the exact value sits next to a rounding midpoint.

Parity pins
-----------
Selection (compression, folding, projections, scoring, pooling, forced
pages, top-k) is pinned against the reference itself: ``tests/golden`` holds
fixtures written by ``tests/golden/make_golden.py``, which imports the
reference in the build container.  Stage-2 attention has no runnable
reference (the InfLLM-v2 CUDA extension is not vendored); its restatement is
pinned against ``torch.nn.functional.scaled_dot_product_attention`` with an
explicit boolean mask built from the page lists, which is an independent
implementation of the same math.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

NEG_INF = np.float32(-np.inf)
POS_INF = np.float32(np.inf)


# ----------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32.

    This is the rounding torch applies in ``Tensor.to(torch.bfloat16)``.
    NaN and infinities pass through unchanged.
    """
    a = np.ascontiguousarray(x, dtype=np.float32)
    bits = a.view(np.uint32)
    # uint32 wrap-around only affects NaN encodings, which are restored below.
    rounded = (bits >> 16) & np.uint32(1)
    rounded += np.uint32(0x7FFF)
    rounded += bits
    rounded &= np.uint32(0xFFFF0000)
    out = rounded.view(np.float32).reshape(a.shape)
    special = ~np.isfinite(a)
    if special.any():
        out = np.where(special, a, out)
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of ``bf16_round(x)``."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """float32 values of bfloat16 bit patterns."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _maybe_round(x: np.ndarray, policy: str) -> np.ndarray:
    if policy == "bf16":
        return bf16_round(x)
    if policy == "fp32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown policy {policy!r}")


# ----------------------------------------------------------------------------
# Geometry (pages.py / minicpm.py)
# ----------------------------------------------------------------------------

def atom_count(seq_len: int, kernel_size: int = 32, kernel_stride: int = 16) -> int:
    """Atoms produced by ``CompressK`` for one sequence.

    ``calc_chunks_with_stride`` (minicpm.py:710-750) keeps windows
    ``[s, s + kernel_size)`` with ``s = i * kernel_stride`` that end inside the
    sequence, so a sequence shorter than ``kernel_size`` has none.  (The
    training helper ``pages.infllm_atom_count`` (pages.py:74-81) returns 1
    there; the serving path used by LeanSelect follows ``CompressK``.)
    """
    if seq_len < kernel_size:
        return 0
    return (seq_len - kernel_size) // kernel_stride + 1


def page_count(seq_len: int, block_size: int = 64) -> int:
    """Pages of a sequence: ``ceil(seq_len / block_size)`` (pages.py:172)."""
    return (seq_len + block_size - 1) // block_size


def compressed_cu_seqlens(cu_seqlens_k: np.ndarray, kernel_size: int = 32,
                          kernel_stride: int = 16) -> np.ndarray:
    """``cu_seqlens_compressed`` of ``calc_chunks_with_stride`` (minicpm.py:736-740)."""
    cu = np.asarray(cu_seqlens_k, dtype=np.int64)
    counts = [atom_count(int(cu[b + 1] - cu[b]), kernel_size, kernel_stride)
              for b in range(len(cu) - 1)]
    out = np.zeros(len(cu), dtype=np.int32)
    out[1:] = np.cumsum(counts)
    return out


# ----------------------------------------------------------------------------
# a1: key compression
# ----------------------------------------------------------------------------

def compress_keys(k: np.ndarray, cu_seqlens_k: np.ndarray, *, kernel_size: int = 32,
                  kernel_stride: int = 16, policy: str = "fp32"):
    """Mean of each window of ``kernel_size`` keys at stride ``kernel_stride``.

    Restates ``CompressK.forward`` (minicpm.py:1169-1185) with
    ``calc_chunks_with_stride`` (minicpm.py:710-750): windows that end inside
    their sequence, packed per sequence, output ``[total_c, G, D]`` plus
    ``cu_seqlens_compressed``.  The same math as ``pages.compress_keys_mean``
    (pages.py:84-101) for sequences of at least ``kernel_size`` tokens.

    Summation order: the window is split into runs of ``run`` tokens, where
    ``run`` is 16 when 16 divides ``kernel_stride`` and ``kernel_stride``
    otherwise; each run is summed sequentially in fp32, the run sums are
    added in order and the total is multiplied by ``1/kernel_size`` (exact
    for powers of two) before the optional bf16 rounding.  The CUDA kernels
    use the same order (16-key runs let one pass serve the 32/16 and 128/64
    compressions together), so in ``bf16`` policy they agree bit for bit.
    """
    k = np.asarray(k, dtype=np.float32)
    if k.ndim != 3:
        raise ValueError("k must be [total_k, G, D]")
    if kernel_size % kernel_stride:
        raise ValueError("kernel_size must be a multiple of kernel_stride")
    cu_c = compressed_cu_seqlens(cu_seqlens_k, kernel_size, kernel_stride)
    total_c = int(cu_c[-1])
    g, d = k.shape[1:]
    out = np.zeros((total_c, g, d), dtype=np.float32)
    run_len = 16 if kernel_stride % 16 == 0 else kernel_stride
    runs = kernel_size // run_len            # runs per window
    step = kernel_stride // run_len          # runs between window starts
    inv = np.float32(1.0 / kernel_size)
    cu = np.asarray(cu_seqlens_k, dtype=np.int64)
    for b in range(len(cu) - 1):
        start = int(cu[b])
        n_atoms = int(cu_c[b + 1] - cu_c[b])
        if n_atoms == 0:
            continue
        n_runs = (n_atoms - 1) * step + runs
        seq = k[start:start + n_runs * run_len]
        # Sequential fp32 sum inside each run of run_len tokens.
        run = np.zeros((n_runs, g, d), dtype=np.float32)
        for i in range(run_len):
            run += seq[i::run_len][:n_runs]
        acc = np.zeros((n_atoms, g, d), dtype=np.float32)
        for j in range(runs):
            acc += run[j:j + (n_atoms - 1) * step + 1:step]
        out[int(cu_c[b]):int(cu_c[b + 1])] = acc * inv
    return _maybe_round(out, policy), cu_c


# ----------------------------------------------------------------------------
# a2-a4: folded selector weights and projections
# ----------------------------------------------------------------------------

@dataclass
class SelectorParams:
    """Canonical selector tensors (selector.py:98-108), float32."""

    head_mix: np.ndarray      # [H, R]
    kv_head_mix: np.ndarray   # [G, R]
    q_proj: np.ndarray        # [R, D, r]
    k_proj: np.ndarray        # [R, D, r]

    @property
    def num_heads(self) -> int:
        return int(self.head_mix.shape[0])

    @property
    def num_kv_heads(self) -> int:
        return int(self.kv_head_mix.shape[0])

    @property
    def head_dim(self) -> int:
        return int(self.q_proj.shape[1])

    @property
    def width(self) -> int:
        return int(self.q_proj.shape[0] * self.q_proj.shape[2])


def fold_weights(params: SelectorParams, policy: str = "fp32"):
    """``LeanSelectSelector.fused_weights`` (selector.py:144-158).

    ``q_fused[h, d, rho*r + j] = head_mix[h, rho] * q_proj[rho, d, j]`` and
    ``kv_fused[g, d, rho*r + j] = kv_head_mix[g, rho] * k_proj[rho, d, j]``:
    one fp32 product per element, then the cast to the query dtype.
    """
    hm = params.head_mix.astype(np.float32)
    km = params.kv_head_mix.astype(np.float32)
    qp = params.q_proj.astype(np.float32)
    kp = params.k_proj.astype(np.float32)
    q_fused = (hm[:, :, None, None] * qp[None]).transpose(0, 2, 1, 3)
    kv_fused = (km[:, :, None, None] * kp[None]).transpose(0, 2, 1, 3)
    q_fused = q_fused.reshape(hm.shape[0], qp.shape[1], -1).astype(np.float32)
    kv_fused = kv_fused.reshape(km.shape[0], kp.shape[1], -1).astype(np.float32)
    return _maybe_round(q_fused, policy), _maybe_round(kv_fused, policy)


def project_queries(q: np.ndarray, q_fused: np.ndarray, num_kv_heads: int,
                    policy: str = "fp32") -> np.ndarray:
    """``project_queries`` (selector.py:160-177): ``[N, H, D] -> [G, N, F]``.

    ``Qs[g, n, f] = sum_{s, d} q[n, g*Hg + s, d] * q_fused[g*Hg + s, d, f]``.
    """
    q = np.asarray(q, dtype=np.float32)
    n, h, d = q.shape
    if q_fused.shape[:2] != (h, d):
        raise ValueError("query must have shape [N, num_heads, head_dim]")
    hg = h // num_kv_heads
    qg = q.reshape(n, num_kv_heads, hg * d).astype(np.float64)
    wf = q_fused.reshape(num_kv_heads, hg * d, -1).astype(np.float64)
    out = np.einsum("ngk,gkf->gnf", qg, wf, optimize=True).astype(np.float32)
    return _maybe_round(out, policy)


def project_atom_keys(kc: np.ndarray, kv_fused: np.ndarray,
                      policy: str = "fp32") -> np.ndarray:
    """``project_atom_keys`` (selector.py:179-190): ``[A, G, D] -> [G, A, F]``."""
    kc = np.asarray(kc, dtype=np.float64)
    out = np.einsum("agd,gdf->gaf", kc, kv_fused.astype(np.float64),
                    optimize=True).astype(np.float32)
    return _maybe_round(out, policy)


def atom_scores(qs: np.ndarray, ks: np.ndarray, policy: str = "fp32") -> np.ndarray:
    """``einsum("gnf,gaf->gna")`` of ``score_pages`` (selector.py:203-207).

    The einsum returns the operands' dtype: bf16 scores under the bf16 policy.
    """
    out = np.einsum("gnf,gaf->gna", qs.astype(np.float64), ks.astype(np.float64),
                    optimize=True).astype(np.float32)
    return _maybe_round(out, policy)


# ----------------------------------------------------------------------------
# a6: atom -> page max-pool
# ----------------------------------------------------------------------------

def pool_atoms_to_pages(scores: np.ndarray, seq_len: int, block_size: int = 64,
                        kernel_stride: int = 16) -> np.ndarray:
    """``pool_atoms_to_pages(reduce="max")`` (pages.py:146-187).

    Page ``p`` is the max over atoms ``[p*s - 1, p*s - 1 + s + 1)`` clipped to
    ``[0, A)`` with ``s = block_size // kernel_stride`` (kernel ``s + 1``,
    stride ``s``, padding 1 with ``-inf``); an empty window gives ``-inf``.
    """
    if block_size % kernel_stride:
        raise ValueError("block_size must be divisible by kernel_stride")
    scores = np.asarray(scores, dtype=np.float32)
    stride = block_size // kernel_stride
    kernel = stride + 1
    n_pages = page_count(seq_len, block_size)
    n_atoms = scores.shape[-1]
    out = np.full(scores.shape[:-1] + (n_pages,), NEG_INF, dtype=np.float32)
    for p in range(n_pages):
        lo = max(p * stride - 1, 0)
        hi = min(p * stride - 1 + kernel, n_atoms)
        if hi > lo:
            out[..., p] = scores[..., lo:hi].max(axis=-1)
    return out


def score_pages(q: np.ndarray, kc: np.ndarray, params: SelectorParams, *, seq_len: int,
                block_size: int = 64, kernel_stride: int = 16,
                policy: str = "fp32") -> np.ndarray:
    """``LeanSelectSelector.score_pages`` (selector.py:192-214): ``[G, N, P]``."""
    q_fused, kv_fused = fold_weights(params, policy)
    qs = project_queries(q, q_fused, params.num_kv_heads, policy)
    ks = project_atom_keys(kc, kv_fused, policy)
    return pool_atoms_to_pages(atom_scores(qs, ks, policy), seq_len, block_size, kernel_stride)


# ----------------------------------------------------------------------------
# a7: visibility, forced pages and top-k
# ----------------------------------------------------------------------------

@dataclass
class Selection:
    """Selected pages of one packed call.

    ``topk_idx``: int32 ``[G, total_q, T]``, each row's pages in ascending
    order followed by ``-1`` padding (the reference's order is unspecified,
    ``torch.topk(sorted=False)``, so comparisons are by set).
    ``boundary``: float32 ``[G, total_q]``, the smallest *finite* score that
    made the cut in each row (``+inf`` when only forced pages were picked,
    ``nan`` when the row is empty); the comparison tolerance is relative to it.
    ``page_scores``: list of ``(q_offset, masked)`` per sequence that was
    scored, ``masked`` being its ``[G, N_b, P_b]`` scores (forced ``+inf``,
    invisible ``-inf``) and ``q_offset`` its first packed query row.
    """

    topk_idx: np.ndarray
    boundary: np.ndarray
    page_scores: list


def select_pages(page_scores: np.ndarray, *, take: int, init_blocks: int,
                 local_blocks: int, block_size: int = 64):
    """Masking + top-k block of ``_lightweight_compressed_attention``.

    Restates minicpm.py:3124-3141: ``visible = p <= t // block_size``;
    ``forced = (p < init_blocks) | (visible & (p + local_blocks >= t // block_size))``;
    invisible pages get ``-inf``, visible forced pages ``+inf``;
    ``topk(min(take, P))``; ``NaN``/``-inf`` picks become ``-1``.  Ties among
    equal finite scores are broken towards the lower page index here (the
    reference leaves the order unspecified).

    Returns ``(idx [G, N, take], boundary [G, N], masked scores [G, N, P])``.
    """
    g, n, p = page_scores.shape
    t_pos = np.arange(n)
    qpage = t_pos // block_size
    pages = np.arange(p)
    visible = pages[None, :] <= qpage[:, None]
    local = visible & (pages[None, :] + local_blocks >= qpage[:, None])
    forced = (pages < init_blocks)[None, :] | local
    masked = np.where(visible[None], page_scores, NEG_INF).astype(np.float32)
    masked = np.where((forced & visible)[None], POS_INF, masked).astype(np.float32)
    k = min(take, p)
    idx = np.full((g, n, take), -1, dtype=np.int32)
    boundary = np.full((g, n), np.nan, dtype=np.float32)
    # Descending by score, ascending page index on ties (stable sort of -score).
    order = np.argsort(-masked, axis=-1, kind="stable")[..., :k]
    vals = np.take_along_axis(masked, order, axis=-1)
    valid = ~(np.isnan(vals) | np.isneginf(vals))
    chosen = np.where(valid, order, -1)
    chosen = np.sort(np.where(chosen < 0, np.iinfo(np.int32).max, chosen), axis=-1)
    chosen = np.where(chosen == np.iinfo(np.int32).max, -1, chosen)
    idx[..., :k] = chosen.astype(np.int32)
    finite_vals = np.where(valid & np.isfinite(vals), vals, POS_INF)
    any_valid = valid.any(axis=-1)
    boundary = np.where(any_valid, finite_vals.min(axis=-1), np.nan).astype(np.float32)
    return idx, boundary, masked


def lightweight_compressed_attention(q: np.ndarray, kc: np.ndarray, cu_seqlens_q: np.ndarray,
                                     cu_seqlens_c: np.ndarray, params: SelectorParams, *,
                                     topk: int, init_blocks: int = 1, local_blocks: int = 2,
                                     block_size: int = 64, kernel_stride: int = 16,
                                     policy: str = "fp32") -> Selection:
    """``MiniCPMInfLLMv2Attention._lightweight_compressed_attention`` (minicpm.py:3061-3142).

    ``topk`` is the reference's ``self.topk`` (= sparse ``topk`` + ``local_blocks``,
    minicpm.py:1965-1966).  Output width ``take = min(topk, max_pages)`` over
    the batch (minicpm.py:3096-3104); each sequence fills
    ``min(take, P_b)`` columns and leaves the rest ``-1``; sequences with no
    queries or no atoms stay all ``-1`` (minicpm.py:3115-3116).
    """
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    cu_c = np.asarray(cu_seqlens_c, dtype=np.int64)
    g = params.num_kv_heads
    total_q = int(q.shape[0])
    max_pages = max((page_count(int(cu_q[b + 1] - cu_q[b]), block_size)
                     for b in range(len(cu_q) - 1)), default=0)
    take = min(topk, max_pages)
    idx = np.full((g, total_q, take), -1, dtype=np.int32)
    boundary = np.full((g, total_q), np.nan, dtype=np.float32)
    scores_out = []
    for b in range(len(cu_q) - 1):
        q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
        c0, c1 = int(cu_c[b]), int(cu_c[b + 1])
        n = q1 - q0
        if n <= 0 or c1 <= c0:
            continue
        scores = score_pages(q[q0:q1], kc[c0:c1], params, seq_len=n, block_size=block_size,
                             kernel_stride=kernel_stride, policy=policy)
        sel, bnd, masked = select_pages(scores, take=take, init_blocks=init_blocks,
                                        local_blocks=local_blocks, block_size=block_size)
        idx[:, q0:q1, :] = sel
        boundary[:, q0:q1] = bnd
        scores_out.append((q0, masked))
    return Selection(idx, boundary, scores_out)


def bf16_ulp(x: float) -> float:
    """Spacing of bfloat16 values at ``|x|`` (2**(e - 7) for 2**e <= |x| < 2**(e+1))."""
    x = abs(float(x))
    if not np.isfinite(x) or x == 0.0:
        return 0.0
    return 2.0 ** (math.floor(math.log2(x)) - 7)


def selection_mismatches(actual: np.ndarray, selection: Selection, *, rel_tol: float = 1e-3,
                         abs_floor: float = 1e-6, ulps: int = 0):
    """Rows whose page set differs from the oracle beyond a boundary tie.

    For each row the symmetric difference between ``actual`` and the oracle
    set must consist only of pages whose oracle score lies within
    ``rel_tol * |boundary|`` (plus ``abs_floor``) of the row's boundary score
    -- or, with ``ulps``, within that many bf16 ulps of it (two bf16-rounded
    scores computed with different fp32 accumulation orders can differ by
    one ulp) -- and both sets must have the same size.  Returns a list of
    ``(g, t, missing, extra)`` for the rows that fail.
    """
    expected = selection.topk_idx
    bad = []
    g_count, n, _ = expected.shape
    score_rows = {}
    for g in range(g_count):
        for t in range(n):
            a = set(int(x) for x in actual[g, t] if x >= 0)
            e = set(int(x) for x in expected[g, t] if x >= 0)
            if a == e:
                continue
            if len(a) != len(e):
                bad.append((g, t, sorted(e - a), sorted(a - e)))
                continue
            bnd = float(selection.boundary[g, t])
            if not np.isfinite(bnd):
                bad.append((g, t, sorted(e - a), sorted(a - e)))
                continue
            if not score_rows:
                score_rows = _score_lookup(selection)
            row = score_rows[(g, t)]
            tol = max(rel_tol * abs(bnd) + abs_floor, ulps * bf16_ulp(bnd))
            if all(abs(float(row[p]) - bnd) <= tol for p in (a ^ e)):
                continue
            bad.append((g, t, sorted(e - a), sorted(a - e)))
    return bad


def _score_lookup(selection: Selection):
    """Map ``(g, packed t)`` to that row's masked page scores."""
    lookup = {}
    for offset, masked in selection.page_scores:
        g_count, n, _ = masked.shape
        for g in range(g_count):
            for t in range(n):
                lookup[(g, offset + t)] = masked[g, t]
    return lookup


# ----------------------------------------------------------------------------
# a9: block-sparse causal attention over selected pages
# ----------------------------------------------------------------------------

def sparse_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens_q: np.ndarray,
                     cu_seqlens_k: np.ndarray, topk_idx: np.ndarray, *,
                     softmax_scale: float | None = None, causal: bool = True,
                     block_size: int = 64, rows=None):
    """Per-token attention over the union of its selected pages.

    Restates the contract of the stage-2 call ``infllmv2_attn_varlen_func(...,
    topk_idx=)`` at minicpm.py:3229-3243: for token ``t`` and head ``h`` (group
    ``g = h // (H/G)``), the keys are the union over ``p in topk_idx[g, t]``,
    ``p >= 0``, of ``[p*block_size, (p+1)*block_size)`` inside the sequence,
    and with ``causal`` only keys at relative position ``<= t + (N_k - N_q)``
    (bottom-right alignment, as FlashAttention-2 varlen).  Duplicate indices
    count once (the extension converts the list to a bitmask,
    paper1.patch topk_to_uint64) and indices at or past the last page are
    ignored.  ``softmax_scale`` defaults to ``D**-0.5``.  A row with no keys
    outputs zeros and ``lse = +inf``.

    Returns ``(out [total_q, H, D] float32, lse [H, total_q] float32)``;
    ``rows`` optionally restricts the work to a list of packed query indices
    (others stay zero / nan).
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    total_q, h, d = q.shape
    g = k.shape[1]
    hg = h // g
    scale = float(d) ** -0.5 if softmax_scale is None else float(softmax_scale)
    out = np.zeros((total_q, h, d), dtype=np.float32)
    lse = np.full((h, total_q), np.nan, dtype=np.float32)
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    cu_k = np.asarray(cu_seqlens_k, dtype=np.int64)
    wanted = None if rows is None else set(int(r) for r in rows)
    for b in range(len(cu_q) - 1):
        q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
        k0, k1 = int(cu_k[b]), int(cu_k[b + 1])
        nq, nk = q1 - q0, k1 - k0
        n_pages = page_count(nk, block_size)
        for t in range(nq):
            row = q0 + t
            if wanted is not None and row not in wanted:
                continue
            limit = nk if not causal else min(nk, t + (nk - nq) + 1)
            for gi in range(g):
                pages = sorted(set(int(p) for p in topk_idx[gi, row] if 0 <= p < n_pages))
                keys = [np.arange(p * block_size, min((p + 1) * block_size, limit))
                        for p in pages if p * block_size < limit]
                heads = slice(gi * hg, (gi + 1) * hg)
                if not keys:
                    out[row, heads] = 0.0
                    lse[heads, row] = np.inf
                    continue
                kk = np.concatenate(keys) + k0
                s = (q[row, heads].astype(np.float64) @ k[kk, gi].astype(np.float64).T) * scale
                m = s.max(axis=-1, keepdims=True)
                e = np.exp(s - m)
                den = e.sum(axis=-1, keepdims=True)
                out[row, heads] = ((e @ v[kk, gi].astype(np.float64)) / den).astype(np.float32)
                lse[heads, row] = (m[:, 0] + np.log(den[:, 0])).astype(np.float32)
    return out, lse


# ----------------------------------------------------------------------------
# Seeded synthetic inputs (benchmark configs)
# ----------------------------------------------------------------------------

@dataclass
class LayerInputs:
    q: np.ndarray            # [total_q, H, D] float32 (bf16-representable when bf16=True)
    k: np.ndarray            # [total_k, G, D]
    v: np.ndarray            # [total_k, G, D]
    cu_seqlens: np.ndarray   # [B+1] int32, q and k share lengths (prefill)
    params: SelectorParams
    hot_pages: list          # per sequence, per group: the shifted page ids


def selector_params(num_heads: int, num_kv_heads: int, head_dim: int, router_heads: int,
                    router_dim: int, rng: np.random.Generator) -> SelectorParams:
    """Selector weights for the synthetic configs.

    ``q_proj``/``k_proj`` follow ``reset_parameters`` (selector.py:112-137):
    an orthonormal frame from a QR of a Gaussian matrix, scaled by
    ``head_dim**-0.25``, reshaped to ``[R, D, r]``.  ``head_mix`` is a seeded
    ``N(0, 1/R)`` matrix (benchmark config 0: "32x32 N(0, 1/32) per group"
    with ``router_heads = 32``) and ``kv_head_mix = 1``.
    """
    width = router_heads * router_dim
    if width <= head_dim:
        frame, _ = np.linalg.qr(rng.standard_normal((head_dim, width)))
    else:
        frame, _ = np.linalg.qr(rng.standard_normal((width, head_dim)))
        frame = frame.T
    frame = (frame * head_dim ** -0.25).astype(np.float32)
    proj = frame.reshape(head_dim, router_heads, router_dim).transpose(1, 0, 2).copy()
    head_mix = (rng.standard_normal((num_heads, router_heads)) / math.sqrt(router_heads))
    return SelectorParams(head_mix.astype(np.float32),
                          np.ones((num_kv_heads, router_heads), dtype=np.float32),
                          proj.astype(np.float32), proj.copy().astype(np.float32))


def synthetic_layer(seq_lens, *, num_heads: int = 32, num_kv_heads: int = 2, head_dim: int = 128,
                    router_heads: int = 32, router_dim: int = 4, hot_pages: int = 24,
                    hot_shift: float = 0.5, block_size: int = 64, seed: int = 0,
                    bf16: bool = False) -> LayerInputs:
    """benchmark config-0/1 generator for a packed batch of sequences.

    Q, K, V ~ N(0, 1).  In each sequence and KV head, ``hot_pages`` distinct
    random pages have their keys shifted by ``hot_shift * u``; every query
    gets the same ``hot_shift * u`` (``u`` a seeded unit vector).  With
    ``bf16`` the tensors are rounded to bf16-representable values.
    """
    rng = np.random.default_rng(seed)
    lens = [int(n) for n in seq_lens]
    total = int(sum(lens))
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    q = rng.standard_normal((total, num_heads, head_dim), dtype=np.float32)
    k = rng.standard_normal((total, num_kv_heads, head_dim), dtype=np.float32)
    v = rng.standard_normal((total, num_kv_heads, head_dim), dtype=np.float32)
    u = rng.standard_normal(head_dim).astype(np.float32)
    u /= np.linalg.norm(u)
    hot = []
    for b, n in enumerate(lens):
        pages = page_count(n, block_size)
        per_group = []
        for g in range(num_kv_heads):
            chosen = rng.choice(pages, size=min(hot_pages, pages), replace=False)
            per_group.append(sorted(int(p) for p in chosen))
            for p in chosen:
                lo = int(cu[b]) + int(p) * block_size
                hi = min(lo + block_size, int(cu[b + 1]))
                k[lo:hi, g] += hot_shift * u
        hot.append(per_group)
    q += hot_shift * u
    params = selector_params(num_heads, num_kv_heads, head_dim, router_heads, router_dim, rng)
    if bf16:
        q, k, v = bf16_round(q), bf16_round(k), bf16_round(v)
    return LayerInputs(q, k, v, cu, params, hot)


def select_for_queries(q_rows: np.ndarray, positions, seq_len: int, kc: np.ndarray,
                       params: SelectorParams, *, take: int, init_blocks: int = 1,
                       local_blocks: int = 2, block_size: int = 64, kernel_stride: int = 16,
                       policy: str = "bf16") -> Selection:
    """The selection of given query rows of ONE sequence of ``seq_len`` tokens.

    ``q_rows [R, H, D]`` are the queries at ``positions`` (relative, length
    ``R``); ``kc [A, G, D]`` are all atoms of the sequence.  Same math as
    :func:`lightweight_compressed_attention` restricted to those rows, so the
    long benchmark configurations can be checked (and timed on the CPU) on a
    sample without scoring every row.  ``take`` is the output width.
    """
    q_fused, kv_fused = fold_weights(params, policy)
    qs = project_queries(q_rows, q_fused, params.num_kv_heads, policy)
    ks = project_atom_keys(kc, kv_fused, policy)
    pages = pool_atoms_to_pages(atom_scores(qs, ks, policy), seq_len, block_size, kernel_stride)
    return select_from_scores(pages, positions, take=take, init_blocks=init_blocks,
                              local_blocks=local_blocks, block_size=block_size)


def select_from_scores(pages: np.ndarray, positions, *, take: int, init_blocks: int = 1,
                       local_blocks: int = 2, block_size: int = 64) -> Selection:
    """Masking + top-k (minicpm.py:3124-3141) of given pooled page scores.

    ``pages [G, R, P]`` are the unmasked page scores of query rows at
    ``positions`` (inside one sequence of ``P`` pages); same rules and tie
    break as :func:`select_pages`.
    """
    positions = np.asarray(positions, dtype=np.int64)
    g, r, p = pages.shape
    qpage = positions // block_size
    page_ids = np.arange(p)
    visible = page_ids[None, :] <= qpage[:, None]
    local = visible & (page_ids[None, :] + local_blocks >= qpage[:, None])
    forced = (page_ids < init_blocks)[None, :] | local
    masked = np.where(visible[None], pages, NEG_INF).astype(np.float32)
    masked = np.where((forced & visible)[None], POS_INF, masked).astype(np.float32)
    k = min(take, p)
    order = np.argsort(-masked, axis=-1, kind="stable")[..., :k]
    vals = np.take_along_axis(masked, order, axis=-1)
    valid = ~(np.isnan(vals) | np.isneginf(vals))
    chosen = np.where(valid, order, -1)
    idx = np.full((g, r, take), -1, dtype=np.int32)
    idx[..., :k] = np.sort(np.where(chosen < 0, np.iinfo(np.int32).max, chosen), axis=-1)
    idx = np.where(idx == np.iinfo(np.int32).max, -1, idx).astype(np.int32)
    finite_vals = np.where(valid & np.isfinite(vals), vals, POS_INF)
    boundary = np.where(valid.any(-1), finite_vals.min(-1), np.nan).astype(np.float32)
    return Selection(idx, boundary, [(0, masked)])


def select_rows(q: np.ndarray, kc: np.ndarray, params: SelectorParams, rows, *, take: int,
                init_blocks: int = 1, local_blocks: int = 2, block_size: int = 64,
                kernel_stride: int = 16, policy: str = "bf16") -> Selection:
    """:func:`select_for_queries` for ``rows`` of a full ``q [N, H, D]``."""
    rows = np.asarray(rows, dtype=np.int64)
    return select_for_queries(q[rows], rows, q.shape[0], kc, params, take=take,
                              init_blocks=init_blocks, local_blocks=local_blocks,
                              block_size=block_size, kernel_stride=kernel_stride, policy=policy)


def attention_for_queries(q_rows: np.ndarray, positions, k: np.ndarray, v: np.ndarray,
                          topk_rows: np.ndarray, *, softmax_scale: float | None = None,
                          block_size: int = 64) -> np.ndarray:
    """Causal sparse attention of given query rows of ONE sequence (prefill).

    ``q_rows [R, H, D]`` at ``positions``; ``k``/``v [N, G, D]`` the whole
    sequence; ``topk_rows [G, R, T]`` their page lists.  Same math as
    :func:`sparse_attention`; returns ``[R, H, D]`` float32.
    """
    positions = np.asarray(positions, dtype=np.int64)
    n, g, d = k.shape
    h = q_rows.shape[1]
    hg = h // g
    scale = float(d) ** -0.5 if softmax_scale is None else float(softmax_scale)
    out = np.zeros((len(positions), h, d), dtype=np.float32)
    n_pages = page_count(n, block_size)
    for i, t in enumerate(positions):
        limit = min(n, int(t) + 1)
        for gi in range(g):
            pages = sorted(set(int(p) for p in topk_rows[gi, i] if 0 <= p < n_pages))
            keys = [np.arange(p * block_size, min((p + 1) * block_size, limit))
                    for p in pages if p * block_size < limit]
            if not keys:
                continue
            kk = np.concatenate(keys)
            qh = q_rows[i, gi * hg:(gi + 1) * hg].astype(np.float64)
            s_ = (qh @ k[kk, gi].astype(np.float64).T) * scale
            e = np.exp(s_ - s_.max(axis=-1, keepdims=True))
            out[i, gi * hg:(gi + 1) * hg] = ((e @ v[kk, gi].astype(np.float64))
                                            / e.sum(-1, keepdims=True)).astype(np.float32)
    return out


def synthetic_keys_and_sample(seq_len: int, rows, *, num_heads: int = 32, num_kv_heads: int = 2,
                              head_dim: int = 128, router_heads: int = 32, router_dim: int = 4,
                              hot_pages: int = 24, hot_shift: float = 0.5, block_size: int = 64,
                              seed: int = 0):
    """Config-0/1 distribution for one sequence, with queries only at ``rows``.

    Returns ``(q_rows [R, H, D], k, v [N, G, D], params)`` rounded to bf16;
    for CPU timing at long lengths without materialising every query.
    """
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((seq_len, num_kv_heads, head_dim), dtype=np.float32)
    v = rng.standard_normal((seq_len, num_kv_heads, head_dim), dtype=np.float32)
    q = rng.standard_normal((len(rows), num_heads, head_dim), dtype=np.float32)
    u = rng.standard_normal(head_dim).astype(np.float32)
    u /= np.linalg.norm(u)
    pages = page_count(seq_len, block_size)
    for g in range(num_kv_heads):
        for p in rng.choice(pages, size=min(hot_pages, pages), replace=False):
            k[int(p) * block_size:min(int(p + 1) * block_size, seq_len), g] += hot_shift * u
    q += hot_shift * u
    params = selector_params(num_heads, num_kv_heads, head_dim, router_heads, router_dim, rng)
    return bf16_round(q), bf16_round(k), bf16_round(v), params


# ----------------------------------------------------------------------------
# Uniform method: the mean-query head mix (ops/uniform.py, ops/head_mix.py)
# ----------------------------------------------------------------------------

def uniform_group_queries(q: np.ndarray, num_kv_heads: int, policy: str = "fp32") -> np.ndarray:
    """``uniform_group_queries`` (pages.py:62-71): mean of each group's heads, ``[N, G, D]``."""
    q = np.asarray(q, dtype=np.float32)
    n, h, d = q.shape
    hg = h // num_kv_heads
    out = q.reshape(n, num_kv_heads, hg, d).astype(np.float64).mean(axis=2).astype(np.float32)
    return _maybe_round(out, policy)


def uniform_atom_scores(q: np.ndarray, kc: np.ndarray, num_kv_heads: int, *,
                        softmax_scale: float | None = None, policy: str = "fp32") -> np.ndarray:
    """Stage-1 scores of the uniform method, ``[G, N, A]`` (head_mix.py:21-77, 80-170).

    ``dots = mean_query . kc`` in the input dtype, then ``* scale`` (default
    ``D**-0.5``) in the input dtype: under the bf16 policy both the matmul
    output and the scaled value are rounded to bf16 (torch computes the
    bf16-tensor-times-scalar product in fp32 and rounds once).
    """
    qg = uniform_group_queries(q, num_kv_heads, policy)
    kc = _maybe_round(np.asarray(kc, dtype=np.float32), policy)
    d = q.shape[-1]
    scale = np.float32(float(d) ** -0.5 if softmax_scale is None else float(softmax_scale))
    dots = np.einsum("ngd,agd->gna", qg.astype(np.float64), kc.astype(np.float64),
                     optimize=True).astype(np.float32)
    dots = _maybe_round(dots, policy)
    return _maybe_round((dots * scale).astype(np.float32), policy)


def uniform_select_rows(atoms: np.ndarray, positions, *, seq_len: int, take: int, topk: int,
                        init_blocks: int, local_blocks: int, block_size: int = 64,
                        kernel_stride: int = 16):
    """Masking, pooling and top-k of the uniform method for rows of ONE sequence.

    Restates ``_uniform_prefill_vectorized_topk`` (uniform.py:68-112) and the
    ragged branch of ``uniform_prefill_topk_idx`` (uniform.py:269-308):
    atoms whose window starts after the query are ``-inf``
    (``apply_atom_causal_mask``, pages.py:199-219); pages are max-pooled
    over ``seq_len``; forced pages (``p < init_blocks`` or
    ``q_page - local_blocks <= p <= q_page``, pages.py:222-240) are ``+inf``;
    ``topk(min(topk, P))`` runs over ALL pages and picks beyond the query's
    page become ``-1`` afterwards.  Such a pick is possible: page
    ``q_page + 1`` sees its first window atom once the query is within one
    stride of the page end, and when it makes the cut it takes a slot that
    no other page gets.  Ties go to the lower page here (the reference's
    order among equal scores is unspecified).

    ``atoms [G, R, A]`` are the rows' uniform atom scores.  Returns
    ``(idx [G, R, take] ascending with -1 padding, boundary [G, R],
    masked page scores [G, R, P])``.
    """
    positions = np.asarray(positions, dtype=np.int64)
    g, r, a = atoms.shape
    atom_start = np.arange(a) * kernel_stride
    vis_atoms = atom_start[None, :] <= positions[:, None]
    masked_atoms = np.where(vis_atoms[None], atoms, NEG_INF).astype(np.float32)
    pages = pool_atoms_to_pages(masked_atoms, max(seq_len, 1), block_size, kernel_stride)
    p = pages.shape[-1]
    qpage = positions // block_size
    page_ids = np.arange(p)
    local = (qpage[:, None] >= page_ids[None, :]) & (qpage[:, None] <= page_ids[None, :] + local_blocks)
    forced = (page_ids < init_blocks)[None, :] | local
    masked = np.where(forced[None], POS_INF, pages).astype(np.float32)
    k = min(topk, p)
    order = np.argsort(-masked, axis=-1, kind="stable")[..., :k]
    vals = np.take_along_axis(masked, order, axis=-1)
    finite_vals = np.where(np.isfinite(vals), vals, POS_INF)
    picked_any = ~np.isneginf(vals)
    boundary = np.where(picked_any.any(-1), finite_vals.min(-1), np.nan).astype(np.float32)
    chosen = np.where(order > qpage[None, :, None], -1, order)
    idx = np.full((g, r, take), -1, dtype=np.int32)
    big = np.iinfo(np.int32).max
    srt = np.sort(np.where(chosen < 0, big, chosen), axis=-1)
    idx[..., :k] = np.where(srt == big, -1, srt).astype(np.int32)
    return idx, boundary, masked


def uniform_prefill_topk_idx(q: np.ndarray, kc: np.ndarray, cu_seqlens_q: np.ndarray,
                             cu_seqlens_c: np.ndarray, *, topk: int, init_blocks: int = 1,
                             local_blocks: int = 2, block_size: int = 64, kernel_stride: int = 16,
                             policy: str = "fp32") -> Selection:
    """``uniform_prefill_topk_idx`` (uniform.py:185-320) on a packed batch.

    Output width ``min(topk, max_pages)``; each sequence fills
    ``min(topk, P_b)`` columns.  A sequence without atoms still selects its
    forced pages (its scores are all ``-inf``, head_mix.py:150-170).  The
    equal-packed, streaming and ragged branches of the reference compute the
    same selection; this follows the ragged one.  The reference rejects
    query lengths <= 1 (uniform.py:203-204).
    """
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    cu_c = np.asarray(cu_seqlens_c, dtype=np.int64)
    lens = np.diff(cu_q)
    if lens.size == 0 or (lens <= 1).any():
        raise ValueError("Uniform is prefill-only; decode must use vanilla Sparse")
    g = kc.shape[1]
    total_q = int(q.shape[0])
    max_pages = max(page_count(int(n), block_size) for n in lens)
    take = min(topk, max_pages)
    idx = np.full((g, total_q, take), -1, dtype=np.int32)
    boundary = np.full((g, total_q), np.nan, dtype=np.float32)
    scores_out = []
    for b in range(len(lens)):
        q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
        c0, c1 = int(cu_c[b]), int(cu_c[b + 1])
        n = q1 - q0
        if c1 > c0:
            atoms = uniform_atom_scores(q[q0:q1], kc[c0:c1], g, policy=policy)
        else:
            atoms = np.full((g, n, 1), NEG_INF, dtype=np.float32)
        sel, bnd, masked = uniform_select_rows(atoms, np.arange(n), seq_len=n, take=take,
                                               topk=topk, init_blocks=init_blocks,
                                               local_blocks=local_blocks, block_size=block_size,
                                               kernel_stride=kernel_stride)
        idx[:, q0:q1] = sel
        boundary[:, q0:q1] = bnd
        scores_out.append((q0, masked))
    return Selection(idx, boundary, scores_out)


def uniform_selection_mismatches(actual: np.ndarray, selection: Selection, *,
                                 block_size: int = 64, rel_tol: float = 1e-3,
                                 abs_floor: float = 1e-6, positions=None):
    """:func:`selection_mismatches` for the uniform method.

    The one difference: a row's pick of page ``q_page + 1`` is dropped from
    its output, so two selections that differ only by a boundary tie
    involving that page have different sizes.  Each row's sets are therefore
    compared after adding that page back to whichever side has one page
    fewer than the number of picks the row made.  ``positions[t]`` is row
    ``t``'s position in its sequence (default: from the packed offsets).
    """
    expected = selection.topk_idx
    scores = _score_lookup(selection)
    bad = []
    g_count, n, _ = expected.shape
    for g in range(g_count):
        for t in range(n):
            a = set(int(x) for x in actual[g, t] if x >= 0)
            e = set(int(x) for x in expected[g, t] if x >= 0)
            if a == e:
                continue
            row = scores[(g, t)]
            if positions is not None:
                pos = int(positions[t])
            else:
                pos = t - max(o for o, _ in selection.page_scores if o <= t)
            future = pos // block_size + 1
            width = min(expected.shape[2], row.shape[0])
            picks = int(np.count_nonzero(~np.isneginf(np.sort(row)[::-1][:width])))
            if future < row.shape[0]:
                if len(a) + 1 == picks and future not in a:
                    a = a | {future}
                if len(e) + 1 == picks and future not in e:
                    e = e | {future}
            bnd = float(selection.boundary[g, t])
            if len(a) != len(e) or not np.isfinite(bnd):
                bad.append((g, t, sorted(e - a), sorted(a - e)))
                continue
            tol = rel_tol * abs(bnd) + abs_floor
            if all(abs(float(row[p]) - bnd) <= tol for p in (a ^ e)):
                continue
            bad.append((g, t, sorted(e - a), sorted(a - e)))
    return bad
