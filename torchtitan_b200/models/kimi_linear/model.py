"""Kimi-Linear hybrid: KDA linear attention + MLA (NoPE) + sigmoid top-8 MoE.

Structure and parameter names follow the reference port
(``experiments/attention_residual/kimi_linear/model.py:83-1115``) so DCP
checkpoints and the HF adapter line up: ``embed_tokens``,
``layers.<i>.{input_layernorm, self_attn, post_attention_layernorm, ffn}``,
``norm``, ``lm_head``; MoE params under ``ffn._moe``.

Block Attention Residuals (``attn_res_blocks > 0``; reference
``experiments/attention_residual/attn_res.py`` and ``kimi_linear/attn_res_model.py``):
each sub-layer reads a softmax mixture (over the block axis, with a learned
zero-initialised pseudo-query and RMSNorm-ed keys) of the committed block
outputs plus the current partial sum instead of a plain residual stream.
``attn_res_blocks == num_hidden_layers`` is Full AttnRes.

FLOPs: routed-expert parameters count as active only for the top_k of
num_experts experts each token uses (the reference counts every expert as
active because its name filter misses ``ffn._moe.experts``).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Any

import torch
import torch.nn as nn

from torchtitan_b200 import ops
from torchtitan_b200.ops import kda as K
from torchtitan_b200.protocols import BaseModel, BaseModelArgs

from ..common.attn_res import block_attn_res
from ..common.layers import Embedding, Linear, RMSNorm, _local
from ..common.moe import MoE


@dataclasses.dataclass(kw_only=True)
class KimiLinearModelArgs(BaseModelArgs):
    vocab_size: int = 163840
    hidden_size: int = 2304
    tie_word_embeddings: bool = False
    num_hidden_layers: int = 27
    intermediate_size: int = 9216
    num_attention_heads: int = 32
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    kda_num_heads: int = 32
    kda_head_dim: int = 128
    kda_short_conv_kernel_size: int = 4
    kda_chunk_size: int = 64
    kda_layers: list[int] = dataclasses.field(default_factory=list)  # 1-indexed
    full_attn_layers: list[int] = dataclasses.field(default_factory=list)  # 1-indexed
    num_experts: int = 256
    num_experts_per_token: int = 8
    moe_intermediate_size: int = 1024
    moe_renormalize: bool = True
    moe_router_activation_func: str = "sigmoid"
    num_shared_experts: int = 1
    routed_scaling_factor: float = 2.446
    first_k_dense_replace: int = 1
    moe_layer_freq: int = 1
    use_grouped_topk: bool = True
    num_expert_group: int = 1
    topk_group: int = 1
    load_balance_coeff: float | None = 1e-3
    aux_loss_coeff: float = 0.0
    rms_norm_eps: float = 1e-5
    initializer_range: float = 0.02
    attn_res_blocks: int = 0  # 0 = standard residuals
    max_seq_len: int = 4096

    def update_from_config(self, trainer_config: Any) -> None:
        self.max_seq_len = max(self.max_seq_len, trainer_config.training.seq_len)

    def is_kda_layer(self, i: int) -> bool:
        return (i + 1) in self.kda_layers

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.first_k_dense_replace and i % self.moe_layer_freq == 0

    def build(self) -> "KimiLinearModel":
        return KimiLinearModel(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        total = sum(p.numel() for p in model.parameters())
        emb = sum(p.numel() for n, p in model.named_parameters() if "embed_tokens" in n)
        routed = sum(p.numel() for n, p in model.named_parameters() if "_moe.experts." in n)
        active_routed = routed * self.num_experts_per_token / max(self.num_experts, 1)
        active = total - emb - routed + active_routed
        n_mla = sum(1 for i in range(self.num_hidden_layers) if not self.is_kda_layer(i))
        qk = self.qk_nope_head_dim + self.qk_rope_head_dim
        attn = 6 * n_mla * self.num_attention_heads * (qk + self.v_head_dim) * seq_len
        # KDA: per token per head ~ chunk-local C*(K+V) pair terms + K*V state update; x3 for fwd+bwd
        n_kda = self.num_hidden_layers - n_mla
        C, Kd = self.kda_chunk_size, self.kda_head_dim
        kda = 6 * n_kda * self.kda_num_heads * (2 * C * Kd + 2 * Kd * Kd)
        return total, 6 * active + attn + kda


class KimiMLP(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.gate_proj = Linear(dim, hidden)
        self.up_proj = Linear(dim, hidden)
        self.down_proj = Linear(hidden, dim)

    def forward(self, x):
        return self.down_proj(ops.swiglu(self.gate_proj(x), self.up_proj(x)))

    def init_weights(self, std):
        for l in (self.gate_proj, self.up_proj, self.down_proj):
            l.init_weights(std)


class KimiMLAAttention(nn.Module):
    """MLA without q compression and without RoPE (mla_use_nope): the 'rope'
    slice of K is shared by all heads (broadcast, not re-projected)."""

    def __init__(self, a: KimiLinearModelArgs):
        super().__init__()
        self.h = a.num_attention_heads
        self.nope, self.rope, self.vd = a.qk_nope_head_dim, a.qk_rope_head_dim, a.v_head_dim
        self.kv_lora_rank = a.kv_lora_rank
        self.q_head_dim = self.nope + self.rope
        self.scaling = self.q_head_dim ** -0.5
        self.q_proj = Linear(a.hidden_size, self.h * self.q_head_dim)
        self.kv_a_proj_with_mqa = Linear(a.hidden_size, a.kv_lora_rank + self.rope)
        self.kv_a_layernorm = RMSNorm(a.kv_lora_rank, a.rms_norm_eps)
        self.kv_b_proj = Linear(a.kv_lora_rank, self.h * (self.nope + self.vd))
        self.o_proj = Linear(self.h * self.vd, a.hidden_size)
        self.cp_hook = None

    def init_weights(self, std):
        for l in (self.q_proj, self.kv_a_proj_with_mqa, self.kv_b_proj, self.o_proj):
            l.init_weights(std)
        self.kv_a_layernorm.init_weights()

    def _attn(self, q, k, v, masks=None):
        return ops.attention(q, k, v, causal=True, scale=self.scaling)

    def forward(self, x):
        B, T, _ = x.shape
        q = self.q_proj(x).view(B, T, -1, self.q_head_dim)
        H = q.shape[2]
        ckv = self.kv_a_proj_with_mqa(x)
        k_pass, k_rot = ckv.split([self.kv_lora_rank, self.rope], dim=-1)
        if getattr(self, "tp_group", None) is not None:
            # the shared key slice feeds only this rank's heads: its gradient is a partial sum
            from torchtitan_b200.parallel.tensor_parallel import grad_all_reduce

            k_rot = grad_all_reduce(k_rot, self.tp_group)
        kv = self.kv_b_proj(self.kv_a_layernorm(k_pass.contiguous())).view(B, T, H, self.nope + self.vd)
        k_nope, v = kv.split([self.nope, self.vd], dim=-1)
        k = torch.cat([k_nope, k_rot[:, :, None, :].expand(B, T, H, self.rope)], dim=-1)
        v = v.contiguous()
        if self.cp_hook is not None:
            o = self.cp_hook(self._attn, q.contiguous(), k.contiguous(), v, None)
        else:
            o = self._attn(q.contiguous(), k.contiguous(), v)
        return self.o_proj(o.reshape(B, o.shape[1], -1))


class ShortConv(nn.Module):
    """Causal depthwise conv + SiLU; ``weight`` [C, 1, W] (nn.Conv1d layout)."""

    def __init__(self, channels: int, width: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(channels, 1, width))

    def init_weights(self):
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))

    def forward(self, x, channel_slice: slice | None = None):
        w = _local(self.weight)
        if channel_slice is not None:
            w = w[channel_slice]
        return K.short_conv_silu(x, w)


class KimiDeltaAttention(nn.Module):
    def __init__(self, a: KimiLinearModelArgs):
        super().__init__()
        self.h, self.d = a.kda_num_heads, a.kda_head_dim
        proj = self.h * self.d
        D = a.hidden_size
        self.chunk = a.kda_chunk_size
        self.eps = a.rms_norm_eps
        self.q_proj, self.k_proj, self.v_proj = Linear(D, proj), Linear(D, proj), Linear(D, proj)
        self.q_conv1d = ShortConv(proj, a.kda_short_conv_kernel_size)
        self.k_conv1d = ShortConv(proj, a.kda_short_conv_kernel_size)
        self.v_conv1d = ShortConv(proj, a.kda_short_conv_kernel_size)
        self.A_log = nn.Parameter(torch.empty(self.h, dtype=torch.float32))
        self.dt_bias = nn.Parameter(torch.empty(proj, dtype=torch.float32))
        self.f_a_proj, self.f_b_proj = Linear(D, self.d), Linear(self.d, proj)
        self.g_a_proj, self.g_b_proj = Linear(D, self.d), Linear(self.d, proj)
        self.b_proj = Linear(D, self.h)
        self.o_norm = RMSNorm(self.d, a.rms_norm_eps)
        self.o_proj = Linear(proj, D)
        self.cp_group = None  # Ulysses: sequence <-> head all-to-all around the recurrence

    def init_weights(self, std):
        for l in (self.q_proj, self.k_proj, self.v_proj, self.f_a_proj, self.f_b_proj, self.g_a_proj,
                  self.g_b_proj, self.b_proj, self.o_proj):
            l.init_weights(std)
        for c in (self.q_conv1d, self.k_conv1d, self.v_conv1d):
            c.init_weights()
        with torch.no_grad():
            self.A_log.copy_(torch.empty_like(self.A_log).uniform_(1, 16).log())
            self.dt_bias.zero_()
        self.o_norm.init_weights()

    def forward(self, x):
        B, T, _ = x.shape
        q, k, v = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        g_raw = self.f_b_proj(self.f_a_proj(x))
        beta = torch.sigmoid(self.b_proj(x).float())
        g_out = self.g_b_proj(self.g_a_proj(x))
        H, Dh = self.h, self.d
        chan = None
        A_log, dt_bias = _local(self.A_log), _local(self.dt_bias)
        if self.cp_group is not None:
            import torch.distributed as dist

            from torchtitan_b200.parallel.context_parallel import seq_to_head

            cp, r = dist.get_world_size(self.cp_group), dist.get_rank(self.cp_group)
            hl = H // cp
            # [B, T/cp, H, D] -> [B, T, H/cp, D] for every per-head stream
            q, k, v, g_raw, g_out = (seq_to_head(t.reshape(B, T, H, -1).contiguous(), self.cp_group)
                                     for t in (q, k, v, g_raw, g_out))
            beta = seq_to_head(beta.reshape(B, T, H, 1).contiguous(), self.cp_group)[..., 0]
            T_full = q.shape[1]
            q, k, v, g_raw, g_out = (t.reshape(B, T_full, hl * Dh) for t in (q, k, v, g_raw, g_out))
            chan = slice(r * hl * Dh, (r + 1) * hl * Dh)
            A_log = A_log[r * hl:(r + 1) * hl]
            dt_bias = dt_bias[chan]
            H, T = hl, T_full
        q = self.q_conv1d(q, chan).reshape(B, T, H, Dh)
        k = self.k_conv1d(k, chan).reshape(B, T, H, Dh)
        v = self.v_conv1d(v, chan).reshape(B, T, H, Dh)
        g = K.kda_gate(g_raw.reshape(B, T, H, Dh), A_log, dt_bias)
        o, _ = K.chunk_kda(q, k, v, g, beta, chunk_size=self.chunk)
        o = K.gated_rms_norm(o, g_out.reshape(B, T, H, Dh), _local(self.o_norm.weight), self.eps)
        if self.cp_group is not None:
            from torchtitan_b200.parallel.context_parallel import head_to_seq

            o = head_to_seq(o.contiguous(), self.cp_group)
            T = o.shape[1]
        return self.o_proj(o.reshape(B, T, -1))


class KimiMoE(nn.Module):
    def __init__(self, a: KimiLinearModelArgs):
        super().__init__()
        groups = a.num_expert_group if (a.use_grouped_topk and a.num_expert_group > 1) else None
        self._moe = MoE(a.hidden_size, a.moe_intermediate_size, a.num_experts, a.num_experts_per_token,
                        score_func=a.moe_router_activation_func, route_norm=a.moe_renormalize,
                        route_scale=a.routed_scaling_factor, num_expert_groups=groups,
                        num_limited_groups=a.topk_group if groups else None,
                        shared_hidden_dim=a.moe_intermediate_size * a.num_shared_experts or None,
                        load_balance_coeff=a.load_balance_coeff, aux_loss_coeff=a.aux_loss_coeff)

    def forward(self, x):
        return self._moe(x)


class KimiDecoderLayer(nn.Module):
    def __init__(self, a: KimiLinearModelArgs, i: int):
        super().__init__()
        self.layer_idx = i
        self.is_linear_attn = a.is_kda_layer(i)
        self.self_attn = KimiDeltaAttention(a) if self.is_linear_attn else KimiMLAAttention(a)
        self.is_moe = a.is_moe_layer(i)
        self.moe_enabled = self.is_moe
        self.ffn = KimiMoE(a) if self.is_moe else KimiMLP(a.hidden_size, a.intermediate_size)
        self.input_layernorm = RMSNorm(a.hidden_size, a.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(a.hidden_size, a.rms_norm_eps)
        self.attn_res = a.attn_res_blocks > 0
        if self.attn_res:
            self.layers_per_block = max(1, a.num_hidden_layers // a.attn_res_blocks)
            self.attn_res_proj = Linear(a.hidden_size, 1)
            self.attn_res_norm = RMSNorm(a.hidden_size, a.rms_norm_eps)
            self.mlp_res_proj = Linear(a.hidden_size, 1)
            self.mlp_res_norm = RMSNorm(a.hidden_size, a.rms_norm_eps)
        self.std = a.initializer_range

    @property
    def moe(self):
        return self.ffn._moe if self.is_moe else None

    def init_weights(self):
        self.self_attn.init_weights(self.std)
        if self.is_moe:
            self.ffn._moe.init_weights(self.std)
        else:
            self.ffn.init_weights(self.std)
        self.input_layernorm.init_weights()
        self.post_attention_layernorm.init_weights()
        if self.attn_res:
            with torch.no_grad():
                self.attn_res_proj.weight.zero_()
                self.mlp_res_proj.weight.zero_()
            self.attn_res_norm.init_weights()
            self.mlp_res_norm.init_weights()

    def forward(self, x, cos=None, sin=None, attention_masks=None):
        if not self.attn_res:
            x = x + self.self_attn(self.input_layernorm(x))
            return x + self.ffn(self.post_attention_layernorm(x))
        blocks, partial = x
        h = block_attn_res(blocks, partial, self.attn_res_proj.weight, self.attn_res_norm)
        if self.layer_idx % self.layers_per_block == 0:
            blocks = blocks + [partial]
            partial = None
        a = self.self_attn(self.input_layernorm(h))
        partial = a if partial is None else partial + a
        h = block_attn_res(blocks, partial, self.mlp_res_proj.weight, self.mlp_res_norm)
        partial = partial + self.ffn(self.post_attention_layernorm(h))
        return blocks, partial


class KimiLinearModel(BaseModel):
    # names used by the pipeline splitter
    pp_first_module = "embed_tokens"

    @property
    def attn_res_layers_per_block(self) -> int | None:
        a = self.model_args
        return max(1, a.num_hidden_layers // a.attn_res_blocks) if a.attn_res_blocks > 0 else None

    @property
    def pp_last_modules(self) -> tuple[str, ...]:
        extra = ("final_res_proj", "final_res_norm") if self.model_args.attn_res_blocks > 0 else ()
        return ("norm", "lm_head", *extra)

    def __init__(self, a: KimiLinearModelArgs):
        super().__init__()
        self.model_args = a
        self.embed_tokens = Embedding(a.vocab_size, a.hidden_size, init_std=a.initializer_range)
        self.layers = nn.ModuleDict({str(i): KimiDecoderLayer(a, i) for i in range(a.num_hidden_layers)})
        self.norm = RMSNorm(a.hidden_size, a.rms_norm_eps)
        self.lm_head = Linear(a.hidden_size, a.vocab_size)
        if a.tie_word_embeddings:
            self.lm_head.weight = self.embed_tokens.weight
        if a.attn_res_blocks > 0:
            self.final_res_proj = Linear(a.hidden_size, 1)
            self.final_res_norm = RMSNorm(a.hidden_size, a.rms_norm_eps)

    @torch.no_grad()
    def init_weights(self, buffer_device: torch.device | None = None) -> None:
        if self.embed_tokens is not None:
            self.embed_tokens.init_weights()
        for layer in self.layers.values():
            layer.init_weights()
        if self.norm is not None:
            self.norm.init_weights()
        if self.lm_head is not None and not self.model_args.tie_word_embeddings:
            self.lm_head.init_weights(self.model_args.initializer_range)
        if getattr(self, "final_res_proj", None) is not None:
            self.final_res_proj.weight.zero_()
            self.final_res_norm.init_weights()

    def forward(self, tokens, attention_masks=None, positions=None, inputs_embeds=None, **kw):
        if inputs_embeds is not None:
            h = inputs_embeds
        else:
            h = self.embed_tokens(tokens) if self.embed_tokens is not None else tokens
        if self.model_args.attn_res_blocks > 0:
            from ..common.attn_res import stage_enter, stage_exit

            # a pipeline stage after the first receives the residual state packed as one tensor
            first = self.embed_tokens is not None or inputs_embeds is not None
            state = stage_enter(self, state=([], h)) if first else stage_enter(self, h)
            for layer in self.layers.values():
                state = layer(state)
            if self.lm_head is None:  # not the last pipeline stage: hand the state on
                return stage_exit(self, state)
            blocks, partial = state
            if getattr(self, "final_res_proj", None) is not None:
                h = block_attn_res(blocks, partial, self.final_res_proj.weight, self.final_res_norm)
            else:
                h = partial
        else:
            for layer in self.layers.values():
                h = layer(h)
        if self.norm is not None:
            h = self.norm(h)
        return self.lm_head(h) if self.lm_head is not None else h
