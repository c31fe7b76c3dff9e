"""Sequence-parallel prefill of one long sequence across the GPUs of a box.

Partition (causal-balanced zig-zag): the sequence is cut into ``2W`` equal
page-aligned chunks; rank ``r`` owns chunks ``r`` and ``2W-1-r``, so every
rank holds one early and one late chunk.  Embedding, QKV, RoPE (at the true
positions), the output projection and the MLP are token-local.  Per layer the
post-RoPE K and V of all ranks are all-gathered over NCCL into the full
sequence; each rank compresses the full K (cheap), then selects pages and runs
the sparse attention for its own two query chunks only
(``ls_select_pages_chunk`` with the chunk's position offset; ``ls_sparse_attn``
over the causal key prefix of the chunk).  The last token lives in chunk
``2W-1``, i.e. on rank 0, which computes the logits.

The partition and gather/reorder helpers are plain host logic over
``torch.distributed`` and work on any backend (tested with ``gloo`` on CPU).
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.distributed as dist

from . import ops
from .attention import _LayerView, count_attended_keys, lightweight_compressed_attention  # noqa: F401
from .model import MiniCPMShape, PrefillModel


def zigzag_chunks(seq_len: int, world: int, rank: int, align: int = 64):
    """``[(start, length), (start, length)]`` of the two chunks rank ``rank`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if seq_len % (2 * world * align):
        raise ValueError(f"seq_len={seq_len} must be a multiple of 2*world*{align}")
    c = seq_len // (2 * world)
    return [(rank * c, c), ((2 * world - 1 - rank) * c, c)]


def local_positions(seq_len: int, world: int, rank: int, device=None) -> torch.Tensor:
    parts = [torch.arange(s, s + n, device=device) for s, n in zigzag_chunks(seq_len, world, rank)]
    return torch.cat(parts)


def gather_sequence(local: torch.Tensor, seq_len: int, group=None) -> torch.Tensor:
    """All-gather every rank's ``[2C, ...]`` rows and return them in sequence order.

    Rank ``r`` contributes chunks ``r`` and ``2W-1-r`` (in that order).  The
    result is ``[seq_len, ...]`` with chunk ``c`` at rows ``[cC, (c+1)C)``.
    """
    world = dist.get_world_size(group)
    c = seq_len // (2 * world)
    if local.shape[0] != 2 * c:
        raise ValueError("local rows must be two chunks of seq_len / (2 * world)")
    local = local.contiguous()
    flat = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(flat, local, group=group)
    gathered = flat.view((world,) + tuple(local.shape))
    first = gathered[:, :c]                     # chunk r of rank r      -> chunks 0 .. W-1
    second = gathered[:, c:].flip(0)            # chunk 2W-1-r of rank r -> chunks W .. 2W-1
    return torch.cat((first.reshape((-1,) + tuple(local.shape[1:])),
                      second.reshape((-1,) + tuple(local.shape[1:]))), dim=0)


def lpt_shards(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of sequences to ranks.

    Returns, per rank, the indices of its sequences (in input order).  Work is
    taken as proportional to length (the dense layers are token-linear and the
    page budget caps the attention per token).
    """
    loads = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: (-int(lengths[j]), j)):
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += int(lengths[i])
    return [sorted(s) for s in shards]


class RankFailure(RuntimeError):
    """A rank did not reach a step: it died, left, or stalled past the limit."""

    def __init__(self, step: int, missing: Sequence[int]):
        super().__init__(f"ranks {list(missing)} did not reach step {step}")
        self.step = step
        self.missing = list(missing)


class StepPresence:
    """Host-side presence check between prefill steps.

    Before each step every rank posts ``step/rank`` to the process group's
    key-value store and waits, up to ``timeout_s``, for all ranks' posts of
    that step.  A rank that died, left between steps or stalls past the limit
    makes the others raise :class:`RankFailure` naming it, before they launch
    a kernel or a collective of the step, so no NCCL collective is left
    waiting for a peer that will never come.  This plays the role of the
    reference trainer's per-step presence all-reduce and error broadcast
    (train.py:270-275, 140), on the store instead of the data path.
    """

    def __init__(self, group=None, timeout_s: float = 60.0, store=None, prefix: str = "leanselect"):
        from datetime import timedelta

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.timeout = timedelta(seconds=float(timeout_s))
        self.prefix = prefix
        self.step = 0

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/step{step}/rank{rank}"

    def arrive(self) -> int:
        """Post this rank's presence for the next step and wait for every rank's."""
        step = self.step
        self.step += 1
        self.store.set(self._key(step, self.rank), "1")
        keys = [self._key(step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception as exc:  # the store raises its own timeout / connection errors
            missing = []
            for r, key in enumerate(keys):
                try:
                    present = self.store.check([key])
                except Exception:
                    present = False
                if not present:
                    missing.append(r)
            raise RankFailure(step, missing or list(range(self.world))) from exc
        return step


_CU_CACHE: dict[tuple, torch.Tensor] = {}


_COMM_STREAMS: dict[int, torch.cuda.Stream] = {}
_OVERLAP_MIN_CHUNK = 4096  # tokens per zig-zag chunk from which the late gather is overlapped


def _comm_stream(dev: torch.device) -> torch.cuda.Stream:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    stream = _COMM_STREAMS.get(idx)
    if stream is None:
        stream = _COMM_STREAMS[idx] = torch.cuda.Stream(device=dev)
    return stream


def sequence_parallel_layer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int,
                            selector, cfg, group=None, timers: list | None = None,
                            key_counts: list | None = None,
                            capture: dict | None = None) -> torch.Tensor:
    """The hot path of one layer for this rank's two zig-zag query chunks.

    ``q [2C, H, D]``, ``k``/``v [2C, G, D]`` are this rank's rows (chunk ``r``
    then chunk ``2W-1-r``, post-RoPE).  Returns the local attention output
    ``[2C, H, D]``.

    The early chunks of all ranks are sequence chunks ``0 .. W-1`` in rank
    order, so they are all-gathered straight into the front half of the full
    K/V.  That half is all the early chunk ``r`` needs (its keys end at
    ``(r+1)C <= WC``, and so do the atoms its candidate pages pool), so its
    compression, selection and attention run while the late chunks are
    all-gathered on a second stream (for chunks of at least
    ``_OVERLAP_MIN_CHUNK`` tokens; shorter ones gather everything first); the
    late half is then put in sequence order, the whole K compressed, and the
    late chunk selected and attended.
    The result equals gathering everything first.  ``timers`` receives
    ``(stage, start, end)`` CUDA events for "gather", "compress", "select" and
    "attn" (two spans per stage: early chunk, late chunk); ``capture``
    (optional dict) receives the page lists of the two chunks as ``idx``
    ``[G, 2C, T]`` (this rank's rows, in its local order).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = int(seq_len)
    chunks = zigzag_chunks(n, world, rank)
    c = chunks[0][1]
    half = world * c
    g, d = k.shape[1], k.shape[2]
    dev = q.device
    compute = torch.cuda.current_stream(dev)
    comm = _comm_stream(dev)

    def mark():
        if timers is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def cu(*values):
        key = (str(dev),) + values
        t = _CU_CACHE.get(key)
        if t is None:
            t = _CU_CACHE[key] = torch.tensor(values, dtype=torch.int32, device=dev)
        return t

    k, v = k.contiguous(), v.contiguous()
    k_full = torch.empty(n, g, d, dtype=k.dtype, device=dev)
    v_full = torch.empty_like(k_full)
    k_late = torch.empty(half, g, d, dtype=k.dtype, device=dev)
    v_late = torch.empty_like(k_late)
    pages = (n + cfg.block_size - 1) // cfg.block_size
    take = min(cfg.topk, pages)
    weights = selector.kernel_weights()

    # Chunks of a few thousand tokens finish their gathers faster than the
    # overlap saves (measured: 0.68 vs 0.25 ms at 2K-token chunks on 8 GPUs).
    overlap = c >= _OVERLAP_MIN_CHUNK
    e_g0 = mark()
    dist.all_gather_into_tensor(k_full[:half], k[:c], group=group)
    dist.all_gather_into_tensor(v_full[:half], v[:c], group=group)
    if overlap:
        comm.wait_stream(compute)
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(k_late, k[c:], group=group)
            dist.all_gather_into_tensor(v_late, v[c:], group=group)
        for t in (k, v, k_late, v_late):
            t.record_stream(comm)
    else:
        dist.all_gather_into_tensor(k_late, k[c:], group=group)
        dist.all_gather_into_tensor(v_late, v[c:], group=group)

    def place_late():
        # Rank r's late chunk is sequence chunk 2W-1-r: reverse the rank order.
        k_full[half:].view(world, c, g, d).copy_(k_late.view(world, c, g, d).flip(0))
        v_full[half:].view(world, c, g, d).copy_(v_late.view(world, c, g, d).flip(0))

    def chunk_work(i, kc_len):
        """Compress K[:kc_len], select and attend query chunk i."""
        start, length = chunks[i]
        e0 = mark()
        kc, _ = ops.compress_keys(k_full[:kc_len], cu(0, kc_len), kernel_size=cfg.kernel_size,
                                  kernel_stride=cfg.kernel_stride, lengths=[kc_len])
        e1 = mark()
        ks = ops.project_atom_keys(kc, weights.wk_t)
        idx = ops.select_pages_chunk(
            q[i * c:(i + 1) * c], weights, ks, q_position=start, seq_len=n, take=take,
            init_blocks=cfg.init_blocks, local_blocks=cfg.local_blocks,
            block_size=cfg.block_size, kernel_stride=cfg.kernel_stride)
        e2 = mark()
        ops.sparse_attn(q[i * c:(i + 1) * c], k_full, v_full, cu(0, length),
                        cu(0, start + length), length, start + length, idx, causal=True,
                        out=attn[i * c:(i + 1) * c])
        e3 = mark()
        if timers is not None:
            timers.extend([("compress", e0, e1), ("select", e1, e2), ("attn", e2, e3)])
        return idx

    attn = torch.empty_like(q)
    if not overlap:
        place_late()
    e_g1 = mark()
    if timers is not None:
        timers.append(("gather", e_g0, e_g1))
    idx0 = chunk_work(0, half)
    if overlap:
        e_w0 = mark()
        compute.wait_stream(comm)
        place_late()
        e_w1 = mark()
        if timers is not None:
            timers.append(("gather", e_w0, e_w1))
    idx1 = chunk_work(1, n)
    if capture is not None:
        capture["idx"] = torch.cat((idx0, idx1), dim=1)
    if key_counts is not None:
        positions = local_positions(n, world, rank, device=dev)
        total = 0
        for i, idx in enumerate((idx0, idx1)):
            total += count_attended_keys(idx, None, cfg.block_size,
                                         positions=positions[i * c:(i + 1) * c])
        key_counts.append(total)
    return attn


class DataParallelRunner:
    """Batched prefill (benchmark config 4): sequences sharded over ranks, no collectives.

    Every rank holds the whole model (same seed), takes its LPT shard of the
    batch, and prefills it as one packed varlen batch; ranks never exchange
    data.  ``prefill_device`` returns this rank's ``(sequence indices, logits)``.
    """

    def __init__(self, shape: MiniCPMShape, device: torch.device | str, seed: int = 0,
                 group=None, presence_timeout_s: float | None = 300.0):
        self.device = torch.device(device)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.model = PrefillModel(shape, self.device, seed=seed)
        self.presence = (StepPresence(group, presence_timeout_s)
                         if self.world > 1 and presence_timeout_s else None)

    def prefill_device(self, ids: torch.Tensor, lengths: Sequence[int]):
        if self.presence is not None:
            self.presence.arrive()
        lengths = [int(n) for n in lengths]
        mine = lpt_shards(lengths, self.world)[self.rank]
        if not mine:
            return mine, None
        offsets = [0]
        for n in lengths:
            offsets.append(offsets[-1] + n)
        local_ids = torch.cat([ids[offsets[i]:offsets[i + 1]] for i in mine])
        local_lens = [lengths[i] for i in mine]
        cu = torch.zeros(len(mine) + 1, dtype=torch.int32)
        cu[1:] = torch.tensor(local_lens).cumsum(0)
        logits = self.model.prefill(local_ids, cu.to(self.device), local_lens)
        return mine, logits


class SequenceParallelRunner:
    """One sequence prefilled by all ranks of the default process group."""

    def __init__(self, shape: MiniCPMShape, device: torch.device | str, seed: int = 0,
                 group=None, presence_timeout_s: float | None = 300.0):
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        # Same seed on every rank: identical random weights everywhere.
        self.model = PrefillModel(shape, self.device, seed=seed)
        self._cu_cache: dict[tuple, torch.Tensor] = {}
        # Every rank checks that all ranks reached the step before launching it.
        self.presence = StepPresence(group, presence_timeout_s) if presence_timeout_s else None

    def _cu(self, *values: int) -> torch.Tensor:
        key = tuple(values)
        t = self._cu_cache.get(key)
        if t is None:
            t = torch.tensor(values, dtype=torch.int32, device=self.device)
            self._cu_cache[key] = t
        return t

    def prefill_device(self, ids: torch.Tensor, lengths: Sequence[int], timers: list | None = None,
                       key_counts: list | None = None):
        """``ids`` holds the whole sequence on every rank; rank 0 returns ``[1, vocab]`` logits."""
        if len(lengths) != 1:
            raise ValueError("sequence-parallel prefill takes one sequence")
        if self.presence is not None:
            self.presence.arrive()
        m, s = self.model, self.model.shape
        n = int(lengths[0])
        chunks = zigzag_chunks(n, self.world, self.rank)
        c = chunks[0][1]
        local_ids = torch.cat([ids[a:a + c] for a, _ in chunks])
        positions = local_positions(n, self.world, self.rank, device=self.device)
        freqs = m.rope.frequencies(n)
        h = m.embed[local_ids] * s.scale_emb
        layer_timers = [] if timers is not None else None
        for layer in m.layers:
            q, k, v = m.qkv(layer, h, positions, freqs)
            attn = sequence_parallel_layer(q, k, v, n, layer.selector, s.sparse, self.group,
                                           timers=layer_timers, key_counts=key_counts)
            del q, k, v
            h.addmm_(attn.view(h.shape[0], -1), layer.w_o.t(), alpha=m.residual_scale)
            del attn
            m.mlp_residual(layer, h)
        if timers is not None:
            timers.extend(layer_timers)
        if self.rank == 0:
            return m.logits(h[-1:])
        return None

    def __call__(self, ids_host: torch.Tensor, lengths: Sequence[int]):
        ids = ids_host.to(self.device, non_blocking=True)
        logits = self.prefill_device(ids, lengths)
        if logits is None:
            torch.cuda.current_stream(self.device).synchronize()
            return None
        out = torch.empty(logits.shape, dtype=logits.dtype, pin_memory=True)
        out.copy_(logits, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out
