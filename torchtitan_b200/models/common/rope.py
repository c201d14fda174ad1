"""Rotary position embedding tables (llama-3 frequency scaling, YaRN).

Tables are ``cos, sin: fp32 [max_seq_len, head_dim/2]``; the kernel rotates
interleaved (even, odd) pairs, i.e. the complex-multiplication convention of
the reference's ``backend="complex"`` (``models/common/rope.py:330``).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn


def _llama3_scale(freqs: torch.Tensor, factor: float = 8.0, low: float = 1.0, high: float = 4.0,
                  orig_ctx: int = 8192) -> torch.Tensor:
    low_wavelen, high_wavelen = orig_ctx / low, orig_ctx / high
    wavelen = 2 * math.pi / freqs
    smooth = (orig_ctx / wavelen - low) / (high - low)
    scaled = torch.where(wavelen > low_wavelen, freqs / factor, freqs)
    mid = (1 - smooth) * freqs / factor + smooth * freqs
    is_mid = (wavelen <= low_wavelen) & (wavelen >= high_wavelen)
    return torch.where(is_mid, mid, scaled)


def _yarn_scale(freqs: torch.Tensor, dim: int, theta: float, factor: float, orig_ctx: int,
                beta_fast: float = 32.0, beta_slow: float = 1.0, truncate: bool = True) -> torch.Tensor:
    """YaRN (Peng et al. 2023) frequency interpolation: a linear ramp between the
    correction dims of ``beta_fast`` and ``beta_slow`` rotations blends interpolated
    (``freq / factor``) and original frequencies.  ``truncate`` rounds the ramp ends
    to whole dims (DeepSeek-V3); GPT-OSS keeps them fractional."""
    def corr_dim(n_rot):
        return dim * math.log(orig_ctx / (n_rot * 2 * math.pi)) / (2 * math.log(theta))

    lo, hi = corr_dim(beta_fast), corr_dim(beta_slow)
    if truncate:
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, dim - 1)
    ramp = ((torch.arange(dim // 2, dtype=torch.float32) - lo) / max(hi - lo, 1e-3)).clamp(0, 1)
    smooth = 1 - ramp
    return freqs / factor * (1 - smooth) + freqs * smooth


def precompute_rope(head_dim: int, max_seq_len: int, theta: float = 10000.0, scaling: str | None = None,
                    scaling_factor: float = 8.0, original_max_seq_len: int = 8192,
                    yarn_truncate: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim))
    if scaling == "llama":
        freqs = _llama3_scale(freqs, factor=scaling_factor, orig_ctx=original_max_seq_len)
    elif scaling == "yarn":
        freqs = _yarn_scale(freqs, head_dim, theta, scaling_factor, original_max_seq_len, truncate=yarn_truncate)
    t = torch.arange(max_seq_len, dtype=torch.float32)
    ang = torch.outer(t, freqs)
    return ang.cos(), ang.sin()


class RotaryEmbedding(nn.Module):
    """Holds the cos/sin tables as non-persistent buffers."""

    def __init__(self, head_dim: int, max_seq_len: int, theta: float, scaling: str | None = None,
                 scaling_factor: float = 8.0, original_max_seq_len: int = 8192, yarn_truncate: bool = True):
        super().__init__()
        self.args = (head_dim, max_seq_len, theta, scaling, scaling_factor, original_max_seq_len, yarn_truncate)
        self.register_buffer("cos", torch.empty(max_seq_len, head_dim // 2), persistent=False)
        self.register_buffer("sin", torch.empty(max_seq_len, head_dim // 2), persistent=False)

    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        c, s = precompute_rope(*self.args)
        dev = buffer_device or self.cos.device
        self.cos = c.to(dev)
        self.sin = s.to(dev)

    def tables(self, seq_len: int, positions: torch.Tensor | None = None):
        if positions is None:
            return self.cos[:seq_len], self.sin[:seq_len]
        if positions.dim() == 2 and positions.shape[0] == 1:
            positions = positions[0]
        # [S] -> [S, D/2]; per-row positions [B, S] -> [B, S, D/2]
        return self.cos[positions], self.sin[positions]
