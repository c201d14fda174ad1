"""Llama 3 / 3.1 dense decoder (parity: ``models/llama3/model.py:21-146``)."""
from __future__ import annotations

import dataclasses
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200.protocols import BaseModelArgs
from ..common import Decoder, Embedding, FeedForward, GQAttention, Linear, RMSNorm, RotaryEmbedding
from ..common.layers import compute_ffn_hidden_dim, depth_init_std


@dataclasses.dataclass(kw_only=True)
class Llama3ModelArgs(BaseModelArgs):
    dim: int = 4096
    n_layers: int = 32
    n_heads: int = 32
    n_kv_heads: int | None = None
    vocab_size: int = 128256
    multiple_of: int = 256
    ffn_dim_multiplier: float | None = None
    norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: str | None = "llama"
    rope_scaling_factor: float = 8.0
    max_seq_len: int = 131072
    depth_init: bool = True
    mask_type: str = "causal"  # or "block_causal" (document masking)
    enable_weight_tying: bool = False

    def update_from_config(self, trainer_config: Any) -> None:
        seq = trainer_config.training.seq_len
        if seq > self.max_seq_len:
            self.max_seq_len = seq

    def build(self) -> "Llama3Model":
        return Llama3Model(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        return dense_nparams_and_flops(model, self.n_layers, self.n_heads, 2 * (self.dim // self.n_heads), seq_len,
                                       self.enable_weight_tying)


def dense_nparams_and_flops(model: nn.Module, n_layers: int, n_heads: int, head_dims: int, seq_len: int,
                            tied: bool = False) -> tuple[int, float]:
    """Training FLOPs/token = 6 * non-embedding params + 6 * L * H * (d_qk + d_v) * S.

    Same convention as the reference (``models/utils.py:389-434``): causal
    sparsity is not discounted and recomputation is not counted, so MFU is
    comparable between the two frameworks.
    """
    nparams = sum(p.numel() for p in model.parameters())
    emb = sum(p.numel() for m in model.children() if isinstance(m, Embedding) for p in m.parameters())
    flops = 6 * (nparams - emb) + 6 * n_layers * n_heads * head_dims * seq_len
    return (nparams - emb if tied else nparams), flops


class Llama3TransformerBlock(nn.Module):
    def __init__(self, layer_id: int, a: Llama3ModelArgs):
        super().__init__()
        self.layer_id = layer_id
        self.attention_norm = RMSNorm(a.dim, a.norm_eps)
        self.attention = GQAttention(a.dim, a.n_heads, a.n_kv_heads, mask_type=a.mask_type)
        self.ffn_norm = RMSNorm(a.dim, a.norm_eps)
        hidden = compute_ffn_hidden_dim(a.dim, a.multiple_of, a.ffn_dim_multiplier)
        self.feed_forward = FeedForward(a.dim, hidden)
        self.weight_init_std = depth_init_std(layer_id, a.n_layers, a.depth_init)
        self.moe_enabled = False

    def forward(self, x, cos, sin, attention_masks=None):
        h = x + self.attention(self.attention_norm(x), cos, sin, attention_masks)
        return h + self.feed_forward(self.ffn_norm(h))

    def init_weights(self) -> None:
        self.attention_norm.init_weights()
        self.ffn_norm.init_weights()
        self.attention.init_weights(self.weight_init_std)
        self.feed_forward.init_weights(self.weight_init_std)


class Llama3Model(Decoder):
    def __init__(self, a: Llama3ModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        self.rope = RotaryEmbedding(a.dim // a.n_heads, a.max_seq_len, a.rope_theta, a.rope_scaling,
                                    a.rope_scaling_factor)
        self.layers = nn.ModuleDict({str(i): Llama3TransformerBlock(i, a) for i in range(a.n_layers)})
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)
        if a.enable_weight_tying:
            self.output.weight = self.tok_embeddings.weight

    @torch.no_grad()
    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        self.rope.init_weights(buffer_device)
        if self.tok_embeddings is not None:
            self.tok_embeddings.init_weights()
        for layer in self.layers.values():
            if layer is not None:
                layer.init_weights()
        if self.norm is not None:
            self.norm.init_weights()
        if self.output is not None:
            s = self.model_args.dim ** -0.5
            self.output.init_cutoff = 3 * s
            self.output.init_weights(s)
