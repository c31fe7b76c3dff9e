"""Public prefill entry point: host token ids in, last-token logits out.

``PrefillRunner`` owns a :class:`~leanselect_b200.model.PrefillModel` (or its
sequence-parallel form) and exposes the call a user makes:
``logits = runner(token_ids_on_host, lengths)`` copies the ids to the GPU,
runs the packed prefill and copies the logits back.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .model import MiniCPMShape, PrefillModel


class PrefillRunner:
    def __init__(self, shape: MiniCPMShape, device: torch.device | str = "cuda", seed: int = 0,
                 model: PrefillModel | None = None):
        self.device = torch.device(device)
        self.model = model if model is not None else PrefillModel(shape, self.device, seed=seed)

    def prefill_device(self, ids: torch.Tensor, lengths: Sequence[int], timers=None,
                       key_counts=None, capture=None):
        """Prefill with ids already on the device; returns device logits ``[B, vocab]``."""
        lengths = [int(n) for n in lengths]
        cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
        cu[1:] = torch.tensor(lengths).cumsum(0)
        cu = cu.to(self.device, non_blocking=True)
        return self.model.prefill(ids, cu, lengths, timers=timers, key_counts=key_counts,
                                  capture=capture)

    def __call__(self, ids_host: torch.Tensor, lengths: Sequence[int]) -> torch.Tensor:
        """Host ids (ideally pinned) -> host logits ``[B, vocab]`` fp32."""
        ids = ids_host.to(self.device, non_blocking=True)
        logits = self.prefill_device(ids, lengths)
        out = torch.empty(logits.shape, dtype=logits.dtype, pin_memory=True)
        out.copy_(logits, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out
