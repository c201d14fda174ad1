"""Llama 3 <-> Hugging Face ``LlamaForCausalLM`` names.

HF stores q/k projections with the rotary pairs split into halves (rotate-half
convention); this framework rotates interleaved pairs, so q/k rows are
permuted on conversion (parity: ``models/llama3/state_dict_adapter.py:18-153``).
"""
from __future__ import annotations

import torch

from torchtitan_b200.protocols import StateDictAdapter


class Llama3StateDictAdapter(StateDictAdapter):
    from_hf_map = {
        "model.embed_tokens.weight": "tok_embeddings.weight",
        "model.layers.{}.self_attn.q_proj.weight": "layers.{}.attention.wq.weight",
        "model.layers.{}.self_attn.k_proj.weight": "layers.{}.attention.wk.weight",
        "model.layers.{}.self_attn.v_proj.weight": "layers.{}.attention.wv.weight",
        "model.layers.{}.self_attn.o_proj.weight": "layers.{}.attention.wo.weight",
        "model.layers.{}.self_attn.rotary_emb.inv_freq": None,
        "model.layers.{}.mlp.gate_proj.weight": "layers.{}.feed_forward.w1.weight",
        "model.layers.{}.mlp.up_proj.weight": "layers.{}.feed_forward.w3.weight",
        "model.layers.{}.mlp.down_proj.weight": "layers.{}.feed_forward.w2.weight",
        "model.layers.{}.input_layernorm.weight": "layers.{}.attention_norm.weight",
        "model.layers.{}.post_attention_layernorm.weight": "layers.{}.ffn_norm.weight",
        "model.norm.weight": "norm.weight",
        "lm_head.weight": "output.weight",
    }

    def _heads(self, key: str) -> int | None:
        a = self.model_args
        if a is None:
            return None
        if key.endswith("attention.wq.weight"):
            return a.n_heads
        if key.endswith("attention.wk.weight"):
            return a.n_kv_heads or a.n_heads
        return None

    @staticmethod
    def interleaved_to_halves(w: torch.Tensor, n_heads: int) -> torch.Tensor:
        hd = w.shape[0] // n_heads
        return w.view(n_heads, hd // 2, 2, -1).transpose(1, 2).reshape(w.shape)

    @staticmethod
    def halves_to_interleaved(w: torch.Tensor, n_heads: int) -> torch.Tensor:
        hd = w.shape[0] // n_heads
        return w.view(n_heads, 2, hd // 2, -1).transpose(1, 2).reshape(w.shape)

    def to_hf_tensor(self, native_key, t):
        h = self._heads(native_key)
        return self.interleaved_to_halves(t, h) if h else t

    def from_hf_tensor(self, native_key, t):
        h = self._heads(native_key)
        return self.halves_to_interleaved(t, h) if h else t
