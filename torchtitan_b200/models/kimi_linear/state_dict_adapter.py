"""Kimi-Linear <-> Hugging Face ``KimiLinearForCausalLM`` names.

HF keeps one module per expert (``block_sparse_moe.experts.<e>.{w1,w2,w3}``);
this framework stacks them into ``ffn._moe.experts.w{1,2,3}`` of shape
``[E, ...]``.  Parity: ``models/utils.py:19-386`` (MoE adapter) and the Kimi
HF blueprint ``kimi_linear/reference/modeling_kimi.py``.
"""
from __future__ import annotations

import re

import torch

from torchtitan_b200.protocols import StateDictAdapter


class KimiLinearStateDictAdapter(StateDictAdapter):
    from_hf_map = {
        "model.embed_tokens.weight": "embed_tokens.weight",
        "model.norm.weight": "norm.weight",
        "lm_head.weight": "lm_head.weight",
        "model.layers.{}.input_layernorm.weight": "layers.{}.input_layernorm.weight",
        "model.layers.{}.post_attention_layernorm.weight": "layers.{}.post_attention_layernorm.weight",
        "model.layers.{}.block_sparse_moe.gate.weight": "layers.{}.ffn._moe.router.gate.weight",
        "model.layers.{}.block_sparse_moe.gate.e_score_correction_bias": "layers.{}.ffn._moe.expert_bias",
        "model.layers.{}.block_sparse_moe.shared_experts.gate_proj.weight": "layers.{}.ffn._moe.shared_experts.w1.weight",
        "model.layers.{}.block_sparse_moe.shared_experts.up_proj.weight": "layers.{}.ffn._moe.shared_experts.w3.weight",
        "model.layers.{}.block_sparse_moe.shared_experts.down_proj.weight": "layers.{}.ffn._moe.shared_experts.w2.weight",
        "model.layers.{}.mlp.gate_proj.weight": "layers.{}.ffn.gate_proj.weight",
        "model.layers.{}.mlp.up_proj.weight": "layers.{}.ffn.up_proj.weight",
        "model.layers.{}.mlp.down_proj.weight": "layers.{}.ffn.down_proj.weight",
    }
    _ATTN = ("q_proj", "k_proj", "v_proj", "o_proj", "kv_a_proj_with_mqa", "kv_b_proj", "f_a_proj", "f_b_proj",
             "g_a_proj", "g_b_proj", "b_proj")
    _ATTN_PARAMS = ("kv_a_layernorm.weight", "o_norm.weight", "q_conv1d.weight", "k_conv1d.weight",
                    "v_conv1d.weight", "A_log", "dt_bias")

    def __init__(self, model_args=None, hf_assets_path=None):
        self.from_hf_map = dict(type(self).from_hf_map)
        for n in self._ATTN:
            self.from_hf_map[f"model.layers.{{}}.self_attn.{n}.weight"] = f"layers.{{}}.self_attn.{n}.weight"
        for n in self._ATTN_PARAMS:
            self.from_hf_map[f"model.layers.{{}}.self_attn.{n}"] = f"layers.{{}}.self_attn.{n}"
        super().__init__(model_args, hf_assets_path)

    def to_hf(self, sd):
        out = {}
        for k, v in sd.items():
            m = re.fullmatch(r"layers\.(\d+)\.ffn\._moe\.experts\.(w[123])", k)
            if m:
                for e in range(v.shape[0]):
                    out[f"model.layers.{m.group(1)}.block_sparse_moe.experts.{e}.{m.group(2)}.weight"] = v[e]
                continue
            nk = self._apply(k, self._to_hf)
            if nk is not None:
                out[nk] = v
        return out

    def from_hf(self, hf):
        out, experts = {}, {}
        for k, v in hf.items():
            m = re.fullmatch(r"model\.layers\.(\d+)\.block_sparse_moe\.experts\.(\d+)\.(w[123])\.weight", k)
            if m:
                experts.setdefault((m.group(1), m.group(3)), {})[int(m.group(2))] = v
                continue
            nk = self._apply(k, self.from_hf_map)
            if nk is not None:
                out[nk] = v
        for (layer, w), per in experts.items():
            out[f"layers.{layer}.ffn._moe.experts.{w}"] = torch.stack([per[e] for e in sorted(per)])
        return out
