"""Llama 4 (parity: reference ``models/llama4/``): MoE with a shared expert
and top-1 sigmoid routing (scores applied before the experts), interleaved
with dense layers every ``interleave_moe_layer_step`` layers, and iRoPE:
every ``every_n_layers_nope``-th layer uses no positional encoding and full
causal attention (with position-dependent query temperature for long contexts), the others use RoPE with chunked attention (causal within
blocks of ``fixed_attn_block_size`` tokens) and optional weightless q/k RMS
normalisation.

Chunked attention is exact with the causal kernel: the sequence is folded
into ``S / block`` independent sequences of ``block`` tokens.
"""
from __future__ import annotations

import dataclasses
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.protocols import BaseModelArgs
from ..common import Decoder, Embedding, FeedForward, GQAttention, Linear, RMSNorm, RotaryEmbedding
from ..common.blocks import DecoderBlock, init_decoder, nparams_and_flops
from ..common.layers import compute_ffn_hidden_dim, depth_init_std
from ..common.moe import MoE


@dataclasses.dataclass(kw_only=True)
class Llama4ModelArgs(BaseModelArgs):
    dim: int = 5120
    n_layers: int = 48
    n_heads: int = 40
    n_kv_heads: int = 8
    vocab_size: int = 202048
    multiple_of: int = 2048
    ffn_dim_multiplier: float | None = 1.2
    norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling_factor: float = 16.0
    max_seq_len: int = 1048576
    depth_init: bool = True
    every_n_layers_nope: int | None = 4
    fixed_attn_block_size: int = 8192
    use_qk_norm: bool = True
    attn_temperature_tuning: bool = True
    floor_scale: float = 8192.0
    attn_scale: float = 0.1
    # MoE
    interleave_moe_layer_step: int = 1
    num_experts: int = 16
    top_k: int = 1
    moe_hidden_dim: int | None = None
    load_balance_coeff: float | None = 1e-3
    aux_loss_coeff: float = 0.0

    def update_from_config(self, trainer_config: Any) -> None:
        self.max_seq_len = max(min(self.max_seq_len, 131072), trainer_config.training.seq_len)

    def build(self) -> "Llama4Model":
        return Llama4Model(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        return nparams_and_flops(model, self.n_layers, self.n_heads, 2 * (self.dim // self.n_heads), seq_len)


def _rms(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


class Llama4Attention(GQAttention):
    def __init__(self, a: Llama4ModelArgs, use_rope: bool):
        super().__init__(a.dim, a.n_heads, a.n_kv_heads)
        self.use_rope = use_rope
        self.block = a.fixed_attn_block_size if use_rope else 0
        self.qk_l2 = a.use_qk_norm and use_rope
        # NoPE layers: queries scaled by 1 + attn_scale * log(1 + floor((pos + 1) / floor_scale))
        self.temp = (a.floor_scale, a.attn_scale) if (a.attn_temperature_tuning and not use_rope) else None

    def inner_attention(self, q, k, v, attention_masks=None):
        B, S = q.shape[:2]
        if self.block and S > self.block:
            # block-diagonal causal: fold the chunks into the batch (padding the last chunk at its
            # end, where causal masking keeps it away from every real query)
            pad = (-S) % self.block
            if pad:
                q, k, v = (torch.nn.functional.pad(t, (0, 0, 0, 0, 0, pad)) for t in (q, k, v))
            n = (S + pad) // self.block
            fold = lambda t: t.reshape(B * n, self.block, *t.shape[2:])  # noqa: E731
            o = ops.attention(fold(q), fold(k), fold(v), causal=True)
            return o.reshape(B, S + pad, *o.shape[2:])[:, :S]
        return ops.attention(q, k, v, causal=True)

    def forward(self, x, cos, sin, attention_masks=None):
        B = x.shape[0]
        q, k, v = self.wq(x), self.wk(x), self.wv(x)
        S = q.shape[1]  # the full sequence under sequence parallelism (the projections gather it)
        q = q.view(B, S, -1, self.head_dim)
        k = k.view(B, S, -1, self.head_dim)
        v = v.view(B, S, -1, self.head_dim)
        if self.use_rope:
            q, k = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
        if self.qk_l2:
            q, k = _rms(q), _rms(k)
        if self.temp is not None:
            floor_scale, attn_scale = self.temp
            pos = torch.arange(S, device=x.device, dtype=torch.float32)
            scale = torch.log(torch.floor((pos + 1) / floor_scale) + 1) * attn_scale + 1
            q = (q.float() * scale.view(1, S, 1, 1)).to(q.dtype)
        if self.cp_hook is not None:
            o = self.cp_hook(self.inner_attention, q, k, v, attention_masks)
        else:
            o = self.inner_attention(q, k, v, attention_masks)
        return self.wo(o.reshape(B, S, -1))


class Llama4Model(Decoder):
    def __init__(self, a: Llama4ModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        self.rope = RotaryEmbedding(a.dim // a.n_heads, a.max_seq_len, a.rope_theta, "llama", a.rope_scaling_factor)
        hidden = compute_ffn_hidden_dim(a.dim, a.multiple_of, a.ffn_dim_multiplier)
        moe_hidden = a.moe_hidden_dim or hidden
        layers = {}
        for i in range(a.n_layers):
            nope = a.every_n_layers_nope is not None and (i + 1) % a.every_n_layers_nope == 0
            att = Llama4Attention(a, use_rope=not nope)
            std = depth_init_std(i, a.n_layers, a.depth_init)
            if (i + 1) % a.interleave_moe_layer_step == 0:
                moe = MoE(a.dim, moe_hidden, a.num_experts, a.top_k, score_func="sigmoid", route_norm=False,
                          shared_hidden_dim=moe_hidden, load_balance_coeff=a.load_balance_coeff,
                          aux_loss_coeff=a.aux_loss_coeff, score_before_experts=True)
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, moe=moe, init_std=std)
            else:
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, feed_forward=FeedForward(a.dim, hidden),
                                              init_std=std)
        self.layers = nn.ModuleDict(layers)
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)

    def init_weights(self, buffer_device=None) -> None:
        init_decoder(self, self.model_args.dim, buffer_device)
