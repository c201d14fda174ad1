"""Qwen3 dense and MoE decoders (parity: reference ``models/qwen3/``).

Differences from Llama 3: an explicit ``head_dim`` (128, independent of
``dim / n_heads``), RMSNorm on every query and key head before RoPE
(``qk_norm``), RoPE theta 1e6, optional tied embeddings, and for the MoE
flavors softmax routing with top-k renormalisation (``norm_topk_prob``) and
no shared expert.
"""
from __future__ import annotations

import dataclasses
from typing import Any

import torch.nn as nn

from torchtitan_b200.protocols import BaseModelArgs
from ..common import Decoder, Embedding, FeedForward, GQAttention, Linear, RMSNorm, RotaryEmbedding
from ..common.blocks import DecoderBlock, init_decoder, nparams_and_flops
from ..common.layers import depth_init_std
from ..common.moe import MoE


@dataclasses.dataclass(kw_only=True)
class Qwen3ModelArgs(BaseModelArgs):
    dim: int = 4096
    n_layers: int = 36
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    hidden_dim: int = 12288
    vocab_size: int = 151936
    norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_seq_len: int = 40960
    qk_norm: bool = True
    enable_weight_tying: bool = False
    depth_init: bool = True
    # MoE
    moe_enabled: bool = False
    num_experts: int = 128
    top_k: int = 8
    moe_hidden_dim: int = 768
    decoder_sparse_step: int = 1
    route_norm: bool = True
    load_balance_coeff: float | None = 1e-3
    aux_loss_coeff: float = 0.0

    def update_from_config(self, trainer_config: Any) -> None:
        self.max_seq_len = max(self.max_seq_len, trainer_config.training.seq_len)

    def build(self) -> "Qwen3Model":
        return Qwen3Model(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        return nparams_and_flops(model, self.n_layers, self.n_heads, 2 * self.head_dim, seq_len,
                                 self.enable_weight_tying)


class Qwen3Model(Decoder):
    def __init__(self, a: Qwen3ModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        self.rope = RotaryEmbedding(a.head_dim, a.max_seq_len, a.rope_theta, None)
        layers = {}
        for i in range(a.n_layers):
            att = GQAttention(a.dim, a.n_heads, a.n_kv_heads, head_dim=a.head_dim, qk_norm=a.qk_norm,
                              norm_eps=a.norm_eps)
            std = depth_init_std(i, a.n_layers, a.depth_init)
            if a.moe_enabled and (i + 1) % a.decoder_sparse_step == 0:
                moe = MoE(a.dim, a.moe_hidden_dim, a.num_experts, a.top_k, score_func="softmax",
                          route_norm=a.route_norm, load_balance_coeff=a.load_balance_coeff,
                          aux_loss_coeff=a.aux_loss_coeff, score_before_experts=False)
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, moe=moe, init_std=std)
            else:
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, feed_forward=FeedForward(a.dim, a.hidden_dim),
                                              init_std=std)
        self.layers = nn.ModuleDict(layers)
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)
        if a.enable_weight_tying:
            self.output.weight = self.tok_embeddings.weight

    def init_weights(self, buffer_device=None) -> None:
        init_decoder(self, self.model_args.dim, buffer_device)
