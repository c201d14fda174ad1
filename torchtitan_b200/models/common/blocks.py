"""Pre-norm decoder block shared by the newer families, and FLOPs counting
for dense and MoE models (parity: ``models/common/decoder.py:38-198`` block
structure; ``models/utils.py:389-434`` FLOPs convention)."""
from __future__ import annotations

import torch
import torch.nn as nn

from .layers import Embedding, RMSNorm


class DecoderBlock(nn.Module):
    """``h = x + attn(norm(x)); out = h + mlp(norm(h))`` where ``mlp`` is a dense
    ``feed_forward`` or a ``moe``; FQNs match the reference families."""

    def __init__(self, layer_id: int, dim: int, attention: nn.Module, norm_eps: float, *,
                 feed_forward: nn.Module | None = None, moe: nn.Module | None = None, init_std: float = 0.02):
        super().__init__()
        self.layer_id = layer_id
        self.attention_norm = RMSNorm(dim, norm_eps)
        self.attention = attention
        self.ffn_norm = RMSNorm(dim, norm_eps)
        if moe is not None:
            self.moe = moe
        else:
            self.feed_forward = feed_forward
        self.moe_enabled = moe is not None
        self.weight_init_std = init_std

    def forward(self, x, cos, sin, attention_masks=None):
        h = x + self.attention(self.attention_norm(x), cos, sin, attention_masks)
        return h + (self.moe if self.moe_enabled else self.feed_forward)(self.ffn_norm(h))

    def init_weights(self) -> None:
        self.attention_norm.init_weights()
        self.ffn_norm.init_weights()
        self.attention.init_weights(self.weight_init_std)
        (self.moe if self.moe_enabled else self.feed_forward).init_weights(self.weight_init_std)


def nparams_and_flops(model: nn.Module, n_layers: int, n_heads: int, head_dims: int, seq_len: int,
                      tied: bool = False) -> tuple[int, float]:
    """Training FLOPs/token = 6 * active non-embedding params + 6 * L * H * (d_qk + d_v) * S.

    Routed experts count with the fraction ``top_k / num_experts`` of their
    parameters (the ones a token actually uses).  Causal sparsity is not
    discounted and recomputation is not counted, as in the reference.
    """
    from .moe import MoE

    nparams = sum(p.numel() for p in model.parameters())
    emb = sum(p.numel() for m in model.modules() if isinstance(m, Embedding) for p in m.parameters())
    inactive = 0
    for m in model.modules():
        if isinstance(m, MoE):
            ex = sum(p.numel() for p in m.experts.parameters())
            inactive += ex - ex * m.top_k // m.num_experts
    flops = 6 * (nparams - emb - inactive) + 6 * n_layers * n_heads * head_dims * seq_len
    return (nparams - emb if tied else nparams), float(flops)


def init_output(model: nn.Module, dim: int) -> None:
    if getattr(model, "output", None) is not None:
        s = dim ** -0.5
        model.output.init_cutoff = 3 * s
        model.output.init_weights(s)


@torch.no_grad()
def init_decoder(model: nn.Module, dim: int, buffer_device=None) -> None:
    """Reference init order: rope tables, embedding, blocks, final norm, output."""
    model.rope.init_weights(buffer_device)
    if model.tok_embeddings is not None:
        model.tok_embeddings.init_weights()
    for layer in model.layers.values():
        if layer is not None:
            layer.init_weights()
    if model.norm is not None:
        model.norm.init_weights()
    init_output(model, dim)
