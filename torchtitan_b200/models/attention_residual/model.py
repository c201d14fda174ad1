"""Dense transformer with Block / Full Attention Residuals (parity: reference
``experiments/attention_residual/model.py:73-503``): Llama 3 blocks whose
residual connections are replaced by ``block_attn_res`` mixtures (two
pseudo-queries and two key norms per layer, one before attention and one
before the MLP; a final mixture before the output norm).

The residual state threaded through the layers is ``(blocks, partial)``:
the list of completed block sums and the running sum of the current block.
A new block starts at every ``layers_per_block``-th layer.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.nn as nn

from ..common import Decoder, Embedding, FeedForward, GQAttention, Linear, RMSNorm, RotaryEmbedding
from ..common.attn_res import block_attn_res
from ..common.blocks import init_output
from ..common.layers import compute_ffn_hidden_dim, depth_init_std
from ..llama3.model import Llama3ModelArgs, dense_nparams_and_flops


@dataclasses.dataclass(kw_only=True)
class AttnResModelArgs(Llama3ModelArgs):
    attn_res_blocks: int = 8
    """Number of residual blocks; ``n_layers`` = Full AttnRes."""

    def build(self) -> "AttnResModel":
        return AttnResModel(self)

    def get_nparams_and_flops(self, model: nn.Module, seq_len: int) -> tuple[int, float]:
        return dense_nparams_and_flops(model, self.n_layers, self.n_heads, 2 * (self.dim // self.n_heads), seq_len,
                                       self.enable_weight_tying)


class AttnResBlock(nn.Module):
    def __init__(self, layer_id: int, a: AttnResModelArgs):
        super().__init__()
        self.layer_id = layer_id
        self.layers_per_block = max(1, a.n_layers // a.attn_res_blocks)
        self.attention_norm = RMSNorm(a.dim, a.norm_eps)
        self.attention = GQAttention(a.dim, a.n_heads, a.n_kv_heads, mask_type=a.mask_type)
        self.ffn_norm = RMSNorm(a.dim, a.norm_eps)
        self.feed_forward = FeedForward(a.dim, compute_ffn_hidden_dim(a.dim, a.multiple_of, a.ffn_dim_multiplier))
        self.attn_res_query = Linear(a.dim, 1)
        self.attn_res_norm = RMSNorm(a.dim, a.norm_eps)
        self.mlp_res_query = Linear(a.dim, 1)
        self.mlp_res_norm = RMSNorm(a.dim, a.norm_eps)
        self.weight_init_std = depth_init_std(layer_id, a.n_layers, a.depth_init)
        self.moe_enabled = False

    def forward(self, state, cos, sin, attention_masks=None):
        blocks, partial = state
        h = block_attn_res(blocks, partial, self.attn_res_query.weight, self.attn_res_norm)
        if self.layer_id % self.layers_per_block == 0:
            blocks, partial = blocks + [partial], None
        a = self.attention(self.attention_norm(h), cos, sin, attention_masks)
        partial = a if partial is None else partial + a
        h = block_attn_res(blocks, partial, self.mlp_res_query.weight, self.mlp_res_norm)
        return blocks, partial + self.feed_forward(self.ffn_norm(h))

    def init_weights(self) -> None:
        for n in (self.attention_norm, self.ffn_norm, self.attn_res_norm, self.mlp_res_norm):
            n.init_weights()
        self.attention.init_weights(self.weight_init_std)
        self.feed_forward.init_weights(self.weight_init_std)
        with torch.no_grad():  # zero queries: every mixture starts uniform
            self.attn_res_query.weight.zero_()
            self.mlp_res_query.weight.zero_()


class AttnResModel(Decoder):
    # pipeline stages: the last one also holds the final residual aggregation
    pp_last_modules = ("final_res_query", "final_res_norm", "norm", "output")

    @property
    def attn_res_layers_per_block(self) -> int:
        a = self.model_args
        return max(1, a.n_layers // a.attn_res_blocks)

    def __init__(self, a: AttnResModelArgs):
        super().__init__()
        self.model_args = a
        self.tok_embeddings = Embedding(a.vocab_size, a.dim)
        self.rope = RotaryEmbedding(a.dim // a.n_heads, a.max_seq_len, a.rope_theta, a.rope_scaling,
                                    a.rope_scaling_factor)
        self.layers = nn.ModuleDict({str(i): AttnResBlock(i, a) for i in range(a.n_layers)})
        self.final_res_query = Linear(a.dim, 1)
        self.final_res_norm = RMSNorm(a.dim, a.norm_eps)
        self.norm = RMSNorm(a.dim, a.norm_eps)
        self.output = Linear(a.dim, a.vocab_size)

    @torch.no_grad()
    def init_weights(self, buffer_device=None) -> None:
        self.rope.init_weights(buffer_device)
        if self.tok_embeddings is not None:
            self.tok_embeddings.init_weights()
        for layer in self.layers.values():
            layer.init_weights()
        if self.final_res_query is not None:
            self.final_res_query.weight.zero_()
            self.final_res_norm.init_weights()
        if self.norm is not None:
            self.norm.init_weights()
        init_output(self, self.model_args.dim)

    def forward(self, tokens, attention_masks=None, positions=None):
        from ..common.attn_res import stage_enter, stage_exit

        if self.tok_embeddings is not None:
            state = stage_enter(self, state=([], self.tok_embeddings(tokens)))
        else:  # a later pipeline stage: the residual state arrives packed as one tensor
            state = stage_enter(self, tokens)
        cos, sin = self._rope_tables(state[1].shape[1], positions)
        for layer in self.layers.values():
            state = layer(state, cos, sin, attention_masks)
        if self.output is None:
            return stage_exit(self, state)
        blocks, partial = state
        h = block_attn_res(blocks, partial, self.final_res_query.weight, self.final_res_norm)
        return self.output(self.norm(h))
