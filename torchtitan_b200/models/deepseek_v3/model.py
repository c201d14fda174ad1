"""DeepSeek-V3 (parity: reference ``models/deepseek_v3/model.py:29-262``).

Multi-head latent attention: queries come from ``wq`` or, with q-LoRA,
``wq_b(q_norm(wq_a(x)))``; keys/values from a compressed latent
``wkv_a(x) = [c_kv (kv_lora_rank), k_pe (rope dim)]`` expanded by
``wkv_b(kv_norm(c_kv)) = [k_nope, v]`` per head.  RoPE (YaRN-scaled) rotates
only the ``qk_rope_head_dim`` slice; the single ``k_pe`` head is shared by all
heads.  Attention runs with d_qk = nope + rope (192) and d_v = 128 on the
tcgen05 MLA path of ``ops.attention``; the softmax scale carries YaRN's
``mscale**2``.  The first ``n_dense_layers`` blocks have a dense SwiGLU MLP,
the rest a token-choice MoE with shared experts and (node-)group-limited routing.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.protocols import BaseModelArgs
from ..common import Decoder, Embedding, FeedForward, Linear, RMSNorm, RotaryEmbedding
from ..common.blocks import DecoderBlock, init_decoder, nparams_and_flops
from ..common.moe import MoE


@dataclasses.dataclass(kw_only=True)
class DeepSeekV3ModelArgs(BaseModelArgs):
    vocab_size: int = 102400
    dim: int = 2048
    inter_dim: int = 10944
    moe_inter_dim: int = 1408
    n_layers: int = 27
    n_dense_layers: int = 1
    n_heads: int = 16
    norm_eps: float = 1e-5
    # MoE
    n_routed_experts: int = 64
    n_shared_experts: int = 2
    n_activated_experts: int = 6
    n_expert_groups: int = 1
    n_limited_groups: int = 1
    score_func: str = "softmax"
    route_norm: bool = False
    route_scale: float = 1.0
    load_balance_coeff: float | None = 1e-3
    aux_loss_coeff: float = 0.0
    # MLA
    q_lora_rank: int = 0
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    # YaRN
    max_seq_len: int = 4096
    original_seq_len: int = 4096
    rope_theta: float = 10000.0
    rope_factor: float = 40.0
    beta_fast: int = 32
    beta_slow: int = 1
    mscale: float = 1.0

    def update_from_config(self, trainer_config: Any) -> None:
        self.max_seq_len = max(self.max_seq_len, trainer_config.training.seq_len)

    def build(self) -> "DeepSeekV3Model":
        return DeepSeekV3Model(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        return nparams_and_flops(model, self.n_layers, self.n_heads,
                                 self.qk_nope_head_dim + self.qk_rope_head_dim + self.v_head_dim, seq_len)

    @property
    def softmax_scale(self) -> float:
        s = (self.qk_nope_head_dim + self.qk_rope_head_dim) ** -0.5
        if self.max_seq_len > self.original_seq_len:
            m = 0.1 * self.mscale * math.log(self.rope_factor) + 1.0
            s = s * m * m
        return s


class MLAttention(nn.Module):
    def __init__(self, a: DeepSeekV3ModelArgs):
        super().__init__()
        self.n_heads = a.n_heads
        self.nope, self.rope_dim, self.vd = a.qk_nope_head_dim, a.qk_rope_head_dim, a.v_head_dim
        self.qk_dim = self.nope + self.rope_dim
        self.q_lora_rank, self.kv_lora_rank = a.q_lora_rank, a.kv_lora_rank
        if a.q_lora_rank == 0:
            self.wq = Linear(a.dim, a.n_heads * self.qk_dim)
        else:
            self.wq_a = Linear(a.dim, a.q_lora_rank)
            self.q_norm = RMSNorm(a.q_lora_rank, a.norm_eps)
            self.wq_b = Linear(a.q_lora_rank, a.n_heads * self.qk_dim)
        self.wkv_a = Linear(a.dim, a.kv_lora_rank + self.rope_dim)
        self.kv_norm = RMSNorm(a.kv_lora_rank, a.norm_eps)
        self.wkv_b = Linear(a.kv_lora_rank, a.n_heads * (self.nope + self.vd))
        self.wo = Linear(a.n_heads * self.vd, a.dim)
        self.softmax_scale = a.softmax_scale
        self.cp_hook = None
        self.kv_cache: dict | None = None  # set by generation (keys/values of earlier positions)

    def init_weights(self, init_std: float) -> None:
        lins = [self.wkv_a, self.wkv_b] + ([self.wq] if self.q_lora_rank == 0 else [self.wq_a, self.wq_b])
        for lin in lins:
            lin.init_weights(0.02)
        self.wo.init_weights(init_std)
        self.kv_norm.init_weights()
        if self.q_lora_rank:
            self.q_norm.init_weights()

    def inner_attention(self, q, k, v, attention_masks=None):
        return ops.attention(q, k, v, causal=True, scale=self.softmax_scale)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, attention_masks=None) -> torch.Tensor:
        B = x.shape[0]
        q = self.wq(x) if self.q_lora_rank == 0 else self.wq_b(self.q_norm(self.wq_a(x)))
        S = q.shape[1]  # the full sequence under sequence parallelism (the projections gather it)
        q = q.view(B, S, -1, self.qk_dim)
        H = q.shape[2]
        q_nope, q_pe = q.split([self.nope, self.rope_dim], dim=-1)
        q_pe = ops.rope(q_pe.contiguous(), cos, sin)
        kv = self.wkv_a(x)
        c_kv, k_pe = kv.split([self.kv_lora_rank, self.rope_dim], dim=-1)
        k_pe = ops.rope(k_pe.contiguous().view(B, S, 1, self.rope_dim), cos, sin)
        kv = self.wkv_b(self.kv_norm(c_kv.contiguous())).view(B, S, H, self.nope + self.vd)
        k_nope, v = kv.split([self.nope, self.vd], dim=-1)
        q = torch.cat([q_nope, q_pe], dim=-1)
        k = torch.cat([k_nope, k_pe.expand(B, S, H, self.rope_dim)], dim=-1)
        v = v.contiguous()
        if self.kv_cache is not None:  # incremental decoding: attend to every cached position too
            if self.kv_cache:
                k = torch.cat([self.kv_cache["k"], k], 1)
                v = torch.cat([self.kv_cache["v"], v], 1)
            self.kv_cache["k"], self.kv_cache["v"] = k, v
        if self.cp_hook is not None:
            o = self.cp_hook(self.inner_attention, q, k, v, attention_masks)
        else:
            o = self.inner_attention(q, k, v, attention_masks)
        return self.wo(o.reshape(B, S, -1))


class DeepSeekV3Model(Decoder):
    def __init__(self, a: DeepSeekV3ModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        scaling = "yarn" if a.max_seq_len > a.original_seq_len else None
        self.rope = RotaryEmbedding(a.qk_rope_head_dim, a.max_seq_len, a.rope_theta, scaling, a.rope_factor,
                                    a.original_seq_len)
        layers = {}
        for i in range(a.n_layers):
            std = 0.02 / (2 * (i + 1)) ** 0.5
            att = MLAttention(a)
            if i < a.n_dense_layers:
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, feed_forward=FeedForward(a.dim, a.inter_dim),
                                              init_std=std)
            else:
                moe = MoE(a.dim, a.moe_inter_dim, a.n_routed_experts, a.n_activated_experts,
                          score_func=a.score_func, route_norm=a.route_norm, route_scale=a.route_scale,
                          num_expert_groups=a.n_expert_groups if a.n_expert_groups > 1 else None,
                          num_limited_groups=a.n_limited_groups if a.n_expert_groups > 1 else None,
                          shared_hidden_dim=a.moe_inter_dim * a.n_shared_experts or None,
                          load_balance_coeff=a.load_balance_coeff, aux_loss_coeff=a.aux_loss_coeff,
                          score_before_experts=False)
                layers[str(i)] = DecoderBlock(i, a.dim, att, a.norm_eps, moe=moe, init_std=std)
        self.layers = nn.ModuleDict(layers)
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)

    def init_weights(self, buffer_device=None) -> None:
        init_decoder(self, self.model_args.dim, buffer_device)
