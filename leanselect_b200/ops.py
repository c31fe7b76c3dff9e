"""Torch-tensor wrappers over the C ABI (device memory and streams come from PyTorch).

Every function takes CUDA tensors, launches on the current stream and returns
new tensors; nothing here computes on the CPU.  bf16 is the compute type of
the kernels: other floating inputs are cast to bf16 at the boundary.

A per-device int32 *status word* collects device-side error bits
(``LS_DEVERR_*``).  It is only read (a stream synchronisation) by
:func:`check_status`, which the tests and ``smoke()`` call.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import torch

from . import _native
from ._native import LS_MAX_ATTN_SPLITS, LS_MAX_TOPK, LeanSelectError

_STATUS: dict[int, torch.Tensor] = {}


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("leanselect_b200 operates on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _call(dev: torch.device, name: str, *args) -> None:
    """One C-ABI call with ``dev`` as the current device (the kernels launch on
    the calling thread's current device; the reference guards the same way)."""
    with torch.cuda.device(dev):
        _native.call(name, *args)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def status_word(device: torch.device) -> torch.Tensor:
    """The device's status word (int32, accumulates LS_DEVERR_* bits)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    word = _STATUS.get(idx)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = word
    return word


def check_status(device: torch.device | int | None = None, reset: bool = True) -> int:
    """Synchronise, return the status bits and raise if any is set."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    word = status_word(device)
    bits = int(word.item())
    if reset and bits:
        word.zero_()
    if bits:
        names = [n for n, b in (("TIMEOUT", _native.LS_DEVERR_TIMEOUT),
                                ("PAGE_INDEX", _native.LS_DEVERR_PAGE_INDEX),
                                ("SEQLENS", _native.LS_DEVERR_SEQLENS)) if bits & b]
        raise LeanSelectError(-bits, f"device status bits set: {'|'.join(names)}")
    return bits


def _bf16(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    return t.contiguous()


def _i32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


def host_lengths(cu_seqlens: torch.Tensor | Sequence[int]) -> list[int]:
    """Sequence lengths on the host (one device->host copy, as the reference does)."""
    cu = cu_seqlens.detach().to("cpu").tolist() if torch.is_tensor(cu_seqlens) else list(cu_seqlens)
    return [int(cu[i + 1]) - int(cu[i]) for i in range(len(cu) - 1)]


def atom_count(n: int, kernel_size: int = 32, kernel_stride: int = 16) -> int:
    """Atoms ``CompressK`` keeps for a sequence of ``n`` keys (minicpm.py:710-750)."""
    return 0 if n < kernel_size else (n - kernel_size) // kernel_stride + 1


# ---------------------------------------------------------------------------
# a2: folded weights
# ---------------------------------------------------------------------------

@dataclass
class FoldedWeights:
    """Selector weights in the layouts the kernels consume."""

    wq_t: torch.Tensor   # [G, F, Hg*D] bf16
    wk_t: torch.Tensor   # [G, F, D] bf16
    num_heads: int
    num_kv_heads: int
    head_dim: int
    width: int


def fold_weights(head_mix: torch.Tensor, kv_head_mix: torch.Tensor, q_proj: torch.Tensor,
                 k_proj: torch.Tensor, *, reference_layout: bool = False,
                 dtype: torch.dtype | None = None):
    """``LeanSelectSelector.fused_weights`` (selector.py:144-158) on the GPU.

    With ``reference_layout`` returns ``(q_fused [H, D, F], kv_fused [G, D, F])``
    in fp32 (``dtype=None``) or bf16; otherwise a :class:`FoldedWeights`.
    """
    dev = _require_cuda(head_mix, kv_head_mix, q_proj, k_proj)
    hm, km = head_mix.detach().float().contiguous(), kv_head_mix.detach().float().contiguous()
    qp, kp = q_proj.detach().float().contiguous(), k_proj.detach().float().contiguous()
    H, R = hm.shape
    G = km.shape[0]
    _, D, r = qp.shape
    F = R * r
    if H % G:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    s = _stream(dev)
    if reference_layout:
        if dtype in (None, torch.float32):
            qf = torch.empty(H, D, F, dtype=torch.float32, device=dev)
            kf = torch.empty(G, D, F, dtype=torch.float32, device=dev)
            _call(dev, "ls_fold_weights", hm.data_ptr(), km.data_ptr(), qp.data_ptr(),
                       kp.data_ptr(), H, G, D, R, r, qf.data_ptr(), kf.data_ptr(), None, None,
                       None, None, s)
            if dtype is None or dtype == torch.float32:
                return qf, kf
        if dtype == torch.bfloat16:
            qb = torch.empty(H, D, F, dtype=torch.bfloat16, device=dev)
            kb = torch.empty(G, D, F, dtype=torch.bfloat16, device=dev)
            _call(dev, "ls_fold_weights", hm.data_ptr(), km.data_ptr(), qp.data_ptr(),
                       kp.data_ptr(), H, G, D, R, r, None, None, qb.data_ptr(), kb.data_ptr(),
                       None, None, s)
            return qb, kb
        # Other dtypes: the reference casts the fp32 product (selector.py:155-157).
        qf = torch.empty(H, D, F, dtype=torch.float32, device=dev)
        kf = torch.empty(G, D, F, dtype=torch.float32, device=dev)
        _call(dev, "ls_fold_weights", hm.data_ptr(), km.data_ptr(), qp.data_ptr(),
                   kp.data_ptr(), H, G, D, R, r, qf.data_ptr(), kf.data_ptr(), None, None,
                   None, None, s)
        return qf.to(dtype), kf.to(dtype)
    hg = H // G
    wq_t = torch.empty(G, F, hg * D, dtype=torch.bfloat16, device=dev)
    wk_t = torch.empty(G, F, D, dtype=torch.bfloat16, device=dev)
    _call(dev, "ls_fold_weights", hm.data_ptr(), km.data_ptr(), qp.data_ptr(), kp.data_ptr(),
               H, G, D, R, r, None, None, None, None, wq_t.data_ptr(), wk_t.data_ptr(), s)
    return FoldedWeights(wq_t, wk_t, H, G, D, F)


# ---------------------------------------------------------------------------
# a1: compression
# ---------------------------------------------------------------------------

def compressed_seqlens(cu_seqlens_k: torch.Tensor, kernel_size: int = 32,
                       kernel_stride: int = 16) -> torch.Tensor:
    """``cu_seqlens_compressed`` of ``calc_chunks_with_stride`` (minicpm.py:710-750)."""
    dev = _require_cuda(cu_seqlens_k)
    cu = _i32(cu_seqlens_k)
    out = torch.empty_like(cu)
    _call(dev, "ls_compressed_seqlens", cu.data_ptr(), cu.numel() - 1, kernel_size,
               kernel_stride, out.data_ptr(), status_word(dev).data_ptr(), _stream(dev))
    return out


def compress_keys(k: torch.Tensor, cu_seqlens_k: torch.Tensor, *, kernel_size: int = 32,
                  kernel_stride: int = 16, lengths: Sequence[int] | None = None,
                  total_c: int | None = None):
    """``CompressK.forward`` (minicpm.py:1169-1185): ``k [total_k, G, D] -> (kc, cu_c)``.

    ``lengths`` (host sequence lengths) or ``total_c`` (the number of atoms)
    avoids the device->host copy of ``cu_seqlens_k`` that sizing the output
    otherwise needs.
    """
    dev = _require_cuda(k, cu_seqlens_k)
    if k.ndim != 3:
        raise ValueError("k must be [total_k, num_kv_heads, head_dim]")
    cu = _i32(cu_seqlens_k)
    if total_c is None:
        lens = list(lengths) if lengths is not None else host_lengths(cu)
        total_c = sum(atom_count(n, kernel_size, kernel_stride) for n in lens)
    if k.dtype == torch.float32:
        # fp32 keys stay fp32, as CompressK keeps the input dtype.
        kf = k.contiguous()
        kc = torch.empty(total_c, k.shape[1], k.shape[2], dtype=torch.float32, device=dev)
        cu_c = torch.empty_like(cu)
        _call(dev, "ls_compress_keys_f32", kf.data_ptr(), cu.data_ptr(), cu.numel() - 1,
              kf.shape[0], k.shape[1], k.shape[2], kernel_size, kernel_stride,
              _ptr(kc) if total_c else None, cu_c.data_ptr(), total_c,
              status_word(dev).data_ptr(), _stream(dev))
        return kc, cu_c
    kb = _bf16(k)
    kc = torch.empty(total_c, k.shape[1], k.shape[2], dtype=torch.bfloat16, device=dev)
    cu_c = torch.empty_like(cu)
    _call(dev, "ls_compress_keys", kb.data_ptr(), cu.data_ptr(), cu.numel() - 1, kb.shape[0],
               k.shape[1], k.shape[2], kernel_size, kernel_stride, _ptr(kc) if total_c else None,
               cu_c.data_ptr(), total_c, status_word(dev).data_ptr(), _stream(dev))
    return kc, cu_c


def compress_keys_dual(k: torch.Tensor, cu_seqlens_k: torch.Tensor, *,
                       lengths: Sequence[int] | None = None):
    """``compress_k`` (32/16) and ``compress_k2`` (128/64) of one prefill in one pass over K.

    Returns ``(kc, cu_c, kc2, cu_c2)``, bit for bit what :func:`compress_keys`
    gives for the two geometries (minicpm.py:2785-2792).
    """
    dev = _require_cuda(k, cu_seqlens_k)
    if k.ndim != 3:
        raise ValueError("k must be [total_k, num_kv_heads, head_dim]")
    kb = _bf16(k)
    cu = _i32(cu_seqlens_k)
    lens = list(lengths) if lengths is not None else host_lengths(cu)
    total_c = sum(atom_count(n, 32, 16) for n in lens)
    total_c2 = sum(atom_count(n, 128, 64) for n in lens)
    g, d = k.shape[1], k.shape[2]
    kc = torch.empty(total_c, g, d, dtype=torch.bfloat16, device=dev)
    kc2 = torch.empty(total_c2, g, d, dtype=torch.bfloat16, device=dev)
    cu_c, cu_c2 = torch.empty_like(cu), torch.empty_like(cu)
    _call(dev, "ls_compress_keys_dual", kb.data_ptr(), cu.data_ptr(), cu.numel() - 1,
          max(lens, default=0), kb.shape[0], g, d, _ptr(kc) if total_c else None,
          cu_c.data_ptr(), total_c, _ptr(kc2) if total_c2 else None, cu_c2.data_ptr(), total_c2,
          status_word(dev).data_ptr(), _stream(dev))
    return kc, cu_c, kc2, cu_c2


# ---------------------------------------------------------------------------
# a3/a4: projections
# ---------------------------------------------------------------------------

def project_atom_keys(kc: torch.Tensor, wk_t: torch.Tensor) -> torch.Tensor:
    """``project_atom_keys`` (selector.py:179-190): ``[A, G, D] -> [G, A, F]`` bf16."""
    dev = _require_cuda(kc, wk_t)
    kcb = _bf16(kc)
    A, G, D = kcb.shape
    F = wk_t.shape[1]
    ks = torch.empty(G, A, F, dtype=torch.bfloat16, device=dev)
    if A:
        _call(dev, "ls_project_atom_keys", kcb.data_ptr(), A, G, D, wk_t.data_ptr(), F,
                   ks.data_ptr(), _stream(dev))
    return ks


def project_queries(q: torch.Tensor, wq_t: torch.Tensor, num_kv_heads: int) -> torch.Tensor:
    """``project_queries`` (selector.py:160-177): ``[N, H, D] -> [G, N, F]`` bf16."""
    dev = _require_cuda(q, wq_t)
    qb = _bf16(q)
    N, H, D = qb.shape
    F = wq_t.shape[1]
    qs = torch.empty(num_kv_heads, N, F, dtype=torch.bfloat16, device=dev)
    if N:
        _call(dev, "ls_project_queries", qb.data_ptr(), N, H, num_kv_heads, D, wq_t.data_ptr(),
                   F, qs.data_ptr(), status_word(dev).data_ptr(), _stream(dev))
    return qs


# ---------------------------------------------------------------------------
# a5-a7: scoring and selection
# ---------------------------------------------------------------------------

def score_pages(q: torch.Tensor, weights: FoldedWeights, ks: torch.Tensor,
                cu_seqlens_q: torch.Tensor, cu_seqlens_c: torch.Tensor, max_seqlen_q: int,
                *, block_size: int = 64, kernel_stride: int = 16) -> torch.Tensor:
    """Pooled page scores ``[G, total_q, ceil(max_seqlen_q/64)]`` (no causal mask).

    Stored as fp32; every value is a bf16 number, because the atom scores are
    rounded to bf16 as the reference's bf16 einsum rounds them
    (selector.py:203-207).  These are the scores :func:`select_pages` ranks.
    """
    dev = _require_cuda(q, ks, cu_seqlens_q, cu_seqlens_c)
    qb = _bf16(q)
    total_q = qb.shape[0]
    G = weights.num_kv_heads
    total_c = ks.shape[1]
    pages = (int(max_seqlen_q) + block_size - 1) // block_size
    out = torch.empty(G, total_q, pages, dtype=torch.float32, device=dev)
    cu_q, cu_c = _i32(cu_seqlens_q), _i32(cu_seqlens_c)
    _call(dev, "ls_score_pages", qb.data_ptr(), weights.wq_t.data_ptr(),
               _ptr(ks) if total_c else None, cu_q.data_ptr(), cu_c.data_ptr(),
               cu_q.numel() - 1, int(max_seqlen_q), total_q, total_c, weights.num_heads, G,
               weights.head_dim, weights.width, block_size, kernel_stride, out.data_ptr(),
               status_word(dev).data_ptr(), _stream(dev))
    return out


def score_pages_single(q: torch.Tensor, weights: FoldedWeights, ks: torch.Tensor, seq_len: int,
                       *, block_size: int = 64, kernel_stride: int = 16) -> torch.Tensor:
    """Page scores ``[G, N, ceil(seq_len/64)]`` of query rows against one sequence's atoms.

    The reference's ``score_pages`` with its own ``seq_len`` (selector.py:192-214):
    the page count follows ``seq_len``, not the number of query rows.
    """
    dev = _require_cuda(q, ks)
    qb = _bf16(q)
    total_q = qb.shape[0]
    G = weights.num_kv_heads
    total_c = ks.shape[1]
    pages = (int(seq_len) + block_size - 1) // block_size
    out = torch.empty(G, total_q, pages, dtype=torch.float32, device=dev)
    if total_q == 0 or pages == 0:
        return out
    _call(dev, "ls_score_pages_single", qb.data_ptr(), weights.wq_t.data_ptr(),
          _ptr(ks) if total_c else None, total_q, total_c, int(seq_len), weights.num_heads, G,
          weights.head_dim, weights.width, block_size, kernel_stride, out.data_ptr(),
          status_word(dev).data_ptr(), _stream(dev))
    return out


def atom_scores(q: torch.Tensor, weights: FoldedWeights, ks: torch.Tensor,
                cu_seqlens_q: torch.Tensor, cu_seqlens_c: torch.Tensor, max_seqlen_q: int,
                max_atoms: int) -> torch.Tensor:
    """Raw atom scores ``[G, total_q, max_atoms]`` bf16 (-inf past each sequence's atoms)."""
    dev = _require_cuda(q, ks, cu_seqlens_q, cu_seqlens_c)
    qb = _bf16(q)
    total_q = qb.shape[0]
    G = weights.num_kv_heads
    total_c = ks.shape[1]
    out = torch.empty(G, total_q, int(max_atoms), dtype=torch.bfloat16, device=dev)
    if total_q == 0 or max_atoms == 0:
        return out
    cu_q, cu_c = _i32(cu_seqlens_q), _i32(cu_seqlens_c)
    _call(dev, "ls_atom_scores", qb.data_ptr(), weights.wq_t.data_ptr(),
               _ptr(ks) if total_c else None, cu_q.data_ptr(), cu_c.data_ptr(),
               cu_q.numel() - 1, int(max_seqlen_q), total_q, total_c, weights.num_heads, G,
               weights.head_dim, weights.width, int(max_atoms), out.data_ptr(),
               status_word(dev).data_ptr(), _stream(dev))
    return out


def select_pages(q: torch.Tensor, weights: FoldedWeights, ks: torch.Tensor,
                 cu_seqlens_q: torch.Tensor, cu_seqlens_c: torch.Tensor, max_seqlen_q: int, *,
                 take: int, init_blocks: int = 1, local_blocks: int = 2, block_size: int = 64,
                 kernel_stride: int = 16) -> torch.Tensor:
    """Fused score + pool + forced + top-T: ``topk_idx [G, total_q, take]`` int32."""
    dev = _require_cuda(q, ks, cu_seqlens_q, cu_seqlens_c)
    qb = _bf16(q)
    total_q = qb.shape[0]
    G = weights.num_kv_heads
    total_c = ks.shape[1]
    if take > LS_MAX_TOPK:
        raise ValueError(f"take={take} exceeds LS_MAX_TOPK={LS_MAX_TOPK}")
    idx = torch.empty(G, total_q, take, dtype=torch.int32, device=dev)
    if take == 0 or total_q == 0:
        return idx
    cu_q, cu_c = _i32(cu_seqlens_q), _i32(cu_seqlens_c)
    ws = _workspace(dev, total_q, G, int(max_seqlen_q))
    _call(dev, "ls_select_pages", qb.data_ptr(), weights.wq_t.data_ptr(),
               _ptr(ks) if total_c else None, cu_q.data_ptr(), cu_c.data_ptr(),
               cu_q.numel() - 1, int(max_seqlen_q), total_q, total_c, weights.num_heads, G,
               weights.head_dim, weights.width, int(take), int(init_blocks), int(local_blocks),
               block_size, kernel_stride, idx.data_ptr(), ws.data_ptr(), ws.numel(),
               status_word(dev).data_ptr(), _stream(dev))
    return idx


def select_pages_f32(q: torch.Tensor, q_fused: torch.Tensor, kc: torch.Tensor,
                     kv_fused: torch.Tensor, cu_seqlens_q: torch.Tensor,
                     cu_seqlens_c: torch.Tensor, max_seqlen_q: int, *, take: int,
                     init_blocks: int = 1, local_blocks: int = 2, block_size: int = 64,
                     kernel_stride: int = 16) -> torch.Tensor:
    """Selection of fp32 inputs in fp32 (the reference's fp32 einsums): ``[G, total_q, take]``.

    ``q_fused [H, D, F]`` / ``kv_fused [G, D, F]`` are the fp32 folded
    weights (``fused_weights()``), ``kc [total_c, G, D]`` the fp32 atoms.
    """
    dev = _require_cuda(q, q_fused, kc, kv_fused, cu_seqlens_q, cu_seqlens_c)
    qf = q.float().contiguous()
    kcf = kc.float().contiguous()
    wq, wk = q_fused.float().contiguous(), kv_fused.float().contiguous()
    total_q, H, D = qf.shape
    total_c, G = kcf.shape[0], kcf.shape[1]
    if take > LS_MAX_TOPK:
        raise ValueError(f"take={take} exceeds LS_MAX_TOPK={LS_MAX_TOPK}")
    idx = torch.empty(G, total_q, take, dtype=torch.int32, device=dev)
    if take == 0 or total_q == 0:
        return idx
    cu_q, cu_c = _i32(cu_seqlens_q), _i32(cu_seqlens_c)
    nbytes = _native.load().ls_select_pages_f32_workspace_bytes(total_q, total_c, G,
                                                                int(max_seqlen_q))
    ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
    _call(dev, "ls_select_pages_f32", qf.data_ptr(), wq.data_ptr(),
          kcf.data_ptr() if total_c else None, wk.data_ptr(), cu_q.data_ptr(), cu_c.data_ptr(),
          cu_q.numel() - 1, int(max_seqlen_q), total_q, total_c, H, G, D, wq.shape[-1], int(take),
          int(init_blocks), int(local_blocks), block_size, kernel_stride, idx.data_ptr(),
          ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(), _stream(dev))
    return idx


def uniform_select_pages(q: torch.Tensor, kc: torch.Tensor, cu_seqlens_q: torch.Tensor,
                         cu_seqlens_c: torch.Tensor, max_seqlen_q: int, *, take: int,
                         init_blocks: int = 1, local_blocks: int = 2, block_size: int = 64,
                         kernel_stride: int = 16,
                         softmax_scale: float | None = None) -> torch.Tensor:
    """Uniform-method selection (ops/uniform.py:185-320): ``[G, total_q, take]`` int32.

    ``kc [total_c, G, D]`` are the compressed keys themselves.
    """
    dev = _require_cuda(q, kc, cu_seqlens_q, cu_seqlens_c)
    qb, kcb = _bf16(q), _bf16(kc)
    total_q, H, D = qb.shape
    total_c, G = kcb.shape[0], kcb.shape[1]
    if take > LS_MAX_TOPK:
        raise ValueError(f"take={take} exceeds LS_MAX_TOPK={LS_MAX_TOPK}")
    idx = torch.empty(G, total_q, take, dtype=torch.int32, device=dev)
    if take == 0 or total_q == 0:
        return idx
    cu_q, cu_c = _i32(cu_seqlens_q), _i32(cu_seqlens_c)
    nbytes = _native.load().ls_uniform_select_workspace_bytes(total_q, total_c, H, G,
                                                              int(max_seqlen_q))
    ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
    _call(dev, "ls_uniform_select_pages", qb.data_ptr(), kcb.data_ptr() if total_c else None,
               cu_q.data_ptr(), cu_c.data_ptr(), cu_q.numel() - 1, int(max_seqlen_q), total_q,
               total_c, H, G, D, int(take), int(init_blocks), int(local_blocks), block_size,
               kernel_stride, float(softmax_scale or 0.0), idx.data_ptr(), ws.data_ptr(),
               ws.numel(), status_word(dev).data_ptr(), _stream(dev))
    return idx


def _workspace(dev: torch.device, rows: int, groups: int, seq_len: int) -> torch.Tensor:
    """Scratch for the selection kernels, from PyTorch's caching allocator."""
    nbytes = _native.load().ls_select_pages_workspace_bytes(rows, groups, seq_len)
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)


def select_pages_chunk(q: torch.Tensor, weights: FoldedWeights, ks: torch.Tensor, *,
                       q_position: int, seq_len: int, take: int, init_blocks: int = 1,
                       local_blocks: int = 2, block_size: int = 64,
                       kernel_stride: int = 16) -> torch.Tensor:
    """Selection for query rows at ``[q_position, q_position + len(q))`` of one sequence.

    ``ks [G, A, F]`` holds the atoms of the whole sequence (sequence-parallel
    prefill: each rank selects for its own query chunks).
    """
    dev = _require_cuda(q, ks)
    qb = _bf16(q)
    n = qb.shape[0]
    G = weights.num_kv_heads
    total_c = ks.shape[1]
    if take > LS_MAX_TOPK:
        raise ValueError(f"take={take} exceeds LS_MAX_TOPK={LS_MAX_TOPK}")
    idx = torch.empty(G, n, take, dtype=torch.int32, device=dev)
    if take == 0 or n == 0:
        return idx
    ws = _workspace(dev, n, G, int(seq_len))
    _call(dev, "ls_select_pages_chunk", qb.data_ptr(), weights.wq_t.data_ptr(),
               _ptr(ks) if total_c else None, n, int(q_position), int(seq_len), total_c,
               weights.num_heads, G, weights.head_dim, weights.width, int(take),
               int(init_blocks), int(local_blocks), block_size, kernel_stride, idx.data_ptr(),
               ws.data_ptr(), ws.numel(), status_word(dev).data_ptr(), _stream(dev))
    return idx


# ---------------------------------------------------------------------------
# a9: sparse attention
# ---------------------------------------------------------------------------

def attn_splits(rows: int, max_seqlen_q: int, max_seqlen_k: int, topk: int,
                device: torch.device) -> int:
    """Page-list slices per row for :func:`sparse_attn` (1 = one CTA per row).

    Only decode-shaped calls (one query per sequence) are split: with fewer
    (token, group) rows than SMs, one CTA per row leaves SMs idle, so each
    row's pages are cut into slices of at least 4 pages, up to about one CTA
    per SM (more slices cost more in per-CTA set-up than they gain: measured
    on 128K-token caches, batch 64 runs 70 us unsplit and 79 us in 3 slices).
    Prefill keeps one CTA per row, so its results do not depend on how the
    rows are batched.
    """
    if max_seqlen_q != 1 or rows <= 0:
        return 1
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    pages = min(topk, -(-max(max_seqlen_k, 0) // 64))
    want = sms // rows
    return max(1, min(want, pages // 4, LS_MAX_ATTN_SPLITS))


def sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                cu_seqlens_k: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int,
                topk_idx: torch.Tensor, *, softmax_scale: float | None = None,
                causal: bool = True, return_lse: bool = False, block_size: int = 64,
                out: torch.Tensor | None = None, splits: int | None = None):
    """Block-sparse attention over per-token page lists (minicpm.py:3229-3243).

    ``splits`` cuts each row's page list into that many slices, one CTA each,
    combined by a second kernel (``ls_sparse_attn_split``); ``None`` picks
    it with :func:`attn_splits` (decode calls only).
    """
    dev = _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, topk_idx)
    qb, kb, vb = _bf16(q), _bf16(k), _bf16(v)
    total_q, H, D = qb.shape
    total_k, G, _ = kb.shape
    idx = _i32(topk_idx)
    if idx.ndim != 3 or idx.shape[0] != G or idx.shape[1] != total_q:
        raise ValueError("topk_idx must be [num_kv_heads, total_q, T]")
    if out is None:
        out = torch.empty(total_q, H, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(H, total_q, dtype=torch.float32, device=dev) if return_lse else None
    cu_q, cu_k = _i32(cu_seqlens_q), _i32(cu_seqlens_k)
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(D)
    if splits is None:
        splits = attn_splits(total_q * G, int(max_seqlen_q), int(max_seqlen_k), idx.shape[2], dev)
    if splits > 1 and total_q:
        nbytes = _native.load().ls_sparse_attn_split_workspace_bytes(total_q, H, int(splits))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _call(dev, "ls_sparse_attn_split", qb.data_ptr(), kb.data_ptr(), vb.data_ptr(),
              cu_q.data_ptr(), cu_k.data_ptr(), cu_q.numel() - 1, int(max_seqlen_q),
              int(max_seqlen_k), total_q, total_k, H, G, D, idx.data_ptr(), idx.shape[2],
              block_size, scale, 1 if causal else 0, int(splits), ws.data_ptr(), nbytes,
              out.data_ptr(), _ptr(lse), status_word(dev).data_ptr(), _stream(dev))
    else:
        _call(dev, "ls_sparse_attn", qb.data_ptr(), kb.data_ptr(), vb.data_ptr(),
              cu_q.data_ptr(), cu_k.data_ptr(), cu_q.numel() - 1, int(max_seqlen_q),
              int(max_seqlen_k), total_q, total_k, H, G, D, idx.data_ptr(), idx.shape[2],
              block_size, scale, 1 if causal else 0, out.data_ptr(), _ptr(lse),
              status_word(dev).data_ptr(), _stream(dev))
    if q.dtype != torch.bfloat16:
        out = out.to(q.dtype)
    return (out, lse) if return_lse else out


def sparse_attn_gather_only(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                            max_seqlen_q: int, max_seqlen_k: int, topk_idx: torch.Tensor, *,
                            causal: bool = True, block_size: int = 64) -> None:
    """The data movement of :func:`sparse_attn` alone (measured gather roofline).

    Same launch geometry, page lists and TMA ring; no math, no output.  Its
    duration is the L2 -> shared-memory gather time of that attention call.
    """
    dev = _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, topk_idx)
    qb, kb, vb = _bf16(q), _bf16(k), _bf16(v)
    total_q, H, D = qb.shape
    total_k, G, _ = kb.shape
    idx = _i32(topk_idx)
    if idx.ndim != 3 or idx.shape[0] != G or idx.shape[1] != total_q:
        raise ValueError("topk_idx must be [num_kv_heads, total_q, T]")
    cu_q, cu_k = _i32(cu_seqlens_q), _i32(cu_seqlens_k)
    _call(dev, "ls_sparse_attn_gather_only", qb.data_ptr(), kb.data_ptr(), vb.data_ptr(),
               cu_q.data_ptr(), cu_k.data_ptr(), cu_q.numel() - 1, int(max_seqlen_q),
               int(max_seqlen_k), total_q, total_k, H, G, D, idx.data_ptr(), idx.shape[2],
               block_size, 1 if causal else 0, status_word(dev).data_ptr(), _stream(dev))
