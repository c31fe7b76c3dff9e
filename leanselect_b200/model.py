"""A MiniCPM4.1-shaped prefill model hosting the LeanSelect hot path.

The benchmark workloads (random-init MiniCPM4.1-8B shape at 128K tokens, and
the batched 24-layer small model) need a backbone around the hot path.  This
module is that host: token embedding scaled by ``scale_emb``, per layer
RMSNorm -> fused QKV projection -> LongRoPE -> **LeanSelect hot path**
(compress, select, sparse attention; this package's kernels) -> output
projection, and a SiLU-gated MLP, each added to the residual with
``scale_depth / sqrt(num_layers)``; a final RMSNorm and the LM head on the
last token of each sequence, scaled by ``hidden / dim_model_base``
(minicpm.py:3526-3634, 3676-3958, 3987-4080).

The dense projections are plain cuBLAS GEMMs through PyTorch; the backbone is
not the product, the hot path is.  Weights are random (seeded): there are no
checkpoints on the benchmark machines.  The LongRoPE per-frequency factors of
the real checkpoint are likewise replaced by a seeded monotone ramp.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import torch

from . import host_kernels as hk
from .attention import LayerConfig, count_attended_keys, prefill_layer_attention
from .selector import LeanSelectSelector


@dataclass
class MiniCPMShape:
    """Architecture numbers (MiniCPM4.1-8B by default)."""

    vocab_size: int = 73448
    hidden_size: int = 4096
    intermediate_size: int = 16384
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 2
    head_dim: int = 128
    rope_theta: float = 10000.0
    original_max_position: int = 65536
    max_position: int = 131072
    scale_emb: float = 12.0
    scale_depth: float = 1.4
    dim_model_base: int = 256
    rms_eps: float = 1e-6
    router_heads: int = 32
    router_dim: int = 4
    sparse: LayerConfig = field(default_factory=LayerConfig)

    @classmethod
    def minicpm41_8b(cls, **kw) -> "MiniCPMShape":
        return cls(**kw)

    @classmethod
    def small_24l(cls, **kw) -> "MiniCPMShape":
        """benchmark config 4: 24 layers, hidden 2048, 16/2 heads, head_dim 128."""
        base = dict(hidden_size=2048, intermediate_size=8192, num_layers=24, num_heads=16,
                    num_kv_heads=2, max_position=32768, original_max_position=32768,
                    router_heads=4, router_dim=32)
        base.update(kw)
        return cls(**base)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Torch reference of the fused RMSNorm kernel (minicpm.py:772-798)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * weight.float()).to(x.dtype)


class LongRoPE:
    """Rotary frequencies with LongRoPE divisors (minicpm.py:895-940)."""

    def __init__(self, shape: MiniCPMShape, device: torch.device, seed: int = 0):
        d = shape.head_dim
        self.inv_freq = 1.0 / shape.rope_theta ** (
            torch.arange(0, d, 2, dtype=torch.float32, device=device) / d)
        # Seeded monotone divisors in [1, 16): the real checkpoint ships 64 measured values.
        gen = torch.Generator(device="cpu").manual_seed(seed)
        ramp = torch.linspace(0.0, 1.0, d // 2) + 0.01 * torch.rand(d // 2, generator=gen)
        self.long_factor = (16.0 ** ramp.clamp(0, 0.999)).to(device)
        self.orig = shape.original_max_position
        scale = shape.max_position / shape.original_max_position
        self.scaling = math.sqrt(1 + math.log(scale) / math.log(self.orig)) if scale > 1 else 1.0

    def frequencies(self, seq_len: int) -> torch.Tensor:
        """Per-frequency inverse wavelengths for a sequence of ``seq_len`` tokens."""
        ext = self.long_factor if seq_len > self.orig else torch.ones_like(self.long_factor)
        return self.inv_freq / ext

    def tables(self, positions: torch.Tensor, seq_len: int):
        """``cos, sin [N, D]`` (fp32, scaled) for integer ``positions`` (torch reference)."""
        freqs = positions.float()[:, None] * self.frequencies(seq_len)[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos() * self.scaling, emb.sin() * self.scaling


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x * cos + rotate_half(x) * sin`` for ``x [N, heads, D]`` (torch reference)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    rot = torch.cat((-x2, x1), dim=-1)
    return (x.float() * cos[:, None].float() + rot.float() * sin[:, None].float()).to(x.dtype)


class Layer:
    """Weights of one decoder layer."""

    def __init__(self, shape: MiniCPMShape, device, gen: torch.Generator, std: float = 0.02):
        h, H, G, D, I = (shape.hidden_size, shape.num_heads, shape.num_kv_heads, shape.head_dim,
                         shape.intermediate_size)

        def w(*dims):
            return (torch.randn(*dims, device=device, generator=gen) * std).bfloat16()

        self.w_qkv = w((H + 2 * G) * D, h)
        self.w_o = w(h, H * D)
        self.w_gate_up = w(2 * I, h)
        self.w_down = w(h, I)
        self.norm_in = torch.ones(h, device=device, dtype=torch.bfloat16)
        self.norm_post = torch.ones(h, device=device, dtype=torch.bfloat16)
        sel = LeanSelectSelector(num_heads=H, num_kv_heads=G, head_dim=D,
                                 router_heads=shape.router_heads, router_dim=shape.router_dim)
        sel = sel.to(device)
        with torch.no_grad():
            # Every selector tensor comes from the model's seeded generator, so
            # two models built with one seed (e.g. on different ranks) agree.
            width = shape.router_heads * shape.router_dim
            raw = torch.randn(max(D, width), min(D, width), device=device, generator=gen)
            frame = torch.linalg.qr(raw.float().cpu(), mode="reduced").Q
            frame = frame if width <= D else frame.T
            proj = (frame * D ** -0.25).reshape(D, shape.router_heads, shape.router_dim)
            sel.q_proj.copy_(proj.permute(1, 0, 2))
            sel.k_proj.copy_(proj.permute(1, 0, 2))
            sel.head_mix.copy_(torch.randn(H, shape.router_heads, device=device, generator=gen)
                               / math.sqrt(shape.router_heads))
        self.selector = sel


class PrefillModel:
    """Random-init MiniCPM-shaped model: ``prefill(token ids) -> last-token logits``."""

    def __init__(self, shape: MiniCPMShape, device: torch.device | str = "cuda", seed: int = 0,
                 mlp_chunk_tokens: int = 16384):
        self.shape = shape
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device).manual_seed(seed)
        std = 0.02
        self.embed = (torch.randn(shape.vocab_size, shape.hidden_size, device=self.device,
                                  generator=gen) * std).bfloat16()
        self.lm_head = (torch.randn(shape.vocab_size, shape.hidden_size, device=self.device,
                                    generator=gen) * std).bfloat16()
        self.norm_final = torch.ones(shape.hidden_size, device=self.device, dtype=torch.bfloat16)
        self.layers = [Layer(shape, self.device, gen, std) for _ in range(shape.num_layers)]
        self.rope = LongRoPE(shape, self.device, seed)
        self.mlp_chunk = int(mlp_chunk_tokens)
        self.residual_scale = shape.scale_depth / math.sqrt(shape.num_layers)

    # -- pieces ----------------------------------------------------------------------

    def qkv(self, layer: Layer, h: torch.Tensor, positions: torch.Tensor, freqs: torch.Tensor):
        """RMSNorm -> fused QKV GEMM -> LongRoPE (fused kernel): contiguous q, k, v."""
        s = self.shape
        x = hk.rms_norm(h, layer.norm_in, s.rms_eps)
        qkv = x @ layer.w_qkv.t()
        del x
        return hk.rope_split(qkv, positions, freqs, self.rope.scaling, s.num_heads,
                             s.num_kv_heads, s.head_dim)

    def mlp_residual(self, layer: Layer, h: torch.Tensor) -> torch.Tensor:
        """``h += scale * down(silu(gate(x)) * up(x))``, chunked over tokens."""
        s = self.shape
        for start in range(0, h.shape[0], self.mlp_chunk):
            hc = h[start:start + self.mlp_chunk]
            x = hk.rms_norm(hc, layer.norm_post, s.rms_eps)
            act = hk.silu_mul(x @ layer.w_gate_up.t())
            hc.addmm_(act, layer.w_down.t(), alpha=self.residual_scale)
        return h

    def logits(self, h_last: torch.Tensor) -> torch.Tensor:
        s = self.shape
        x = hk.rms_norm(h_last, self.norm_final, s.rms_eps)
        return (x @ self.lm_head.t()).float() / (s.hidden_size / s.dim_model_base)

    # -- single-device prefill ---------------------------------------------------------

    def prefill(self, input_ids: torch.Tensor, cu_seqlens: torch.Tensor,
                lengths: Sequence[int], timers: list | None = None,
                key_counts: list | None = None, capture: dict | None = None) -> torch.Tensor:
        """Packed prefill of ``len(lengths)`` sequences; returns ``[B, vocab]`` fp32 logits.

        ``timers`` (optional) collects per-layer hot-path stage events (see
        ``prefill_layer_attention``); ``key_counts`` (optional, adds host
        syncs) collects each layer's attended-key count; ``capture``
        (optional dict) receives the last layer's attention inputs
        (``q``, ``k``, ``v``, ``idx``, ``cu``, ``max_len``) for profiling.
        """
        s = self.shape
        lengths = [int(n) for n in lengths]
        positions = torch.cat([torch.arange(n, device=self.device) for n in lengths])
        freqs = self.rope.frequencies(max(lengths))
        h = self.embed[input_ids] * s.scale_emb
        max_len = max(lengths)
        for layer in self.layers:
            q, k, v = self.qkv(layer, h, positions, freqs)
            attn, idx = prefill_layer_attention(q, k, v, cu_seqlens, max_len, layer.selector,
                                                s.sparse, lengths=lengths, return_topk=True,
                                                timers=timers)
            if key_counts is not None:
                key_counts.append(count_attended_keys(idx, lengths, s.sparse.block_size))
            if capture is not None and layer is self.layers[-1]:
                capture.update(q=q, k=k, v=v, idx=idx, cu=cu_seqlens, max_len=max_len)
            del q, k, v, idx
            h.addmm_(attn.view(h.shape[0], -1), layer.w_o.t(), alpha=self.residual_scale)
            del attn
            self.mlp_residual(layer, h)
        last = cu_seqlens[1:].long() - 1
        return self.logits(h[last])
