"""Llama 4 <-> Hugging Face ``Llama4ForCausalLM`` (text) names.  Both rotate
interleaved RoPE pairs, so q/k rows are not permuted; HF stacks each layer's
experts transposed with gate and up concatenated (``gate_up_proj [E, D, 2I]``,
``down_proj [E, I, D]``)."""
from __future__ import annotations

import re

import torch

from torchtitan_b200.protocols import StateDictAdapter


class Llama4StateDictAdapter(StateDictAdapter):
    from_hf_map = {
        "model.embed_tokens.weight": "tok_embeddings.weight",
        "model.layers.{}.self_attn.q_proj.weight": "layers.{}.attention.wq.weight",
        "model.layers.{}.self_attn.k_proj.weight": "layers.{}.attention.wk.weight",
        "model.layers.{}.self_attn.v_proj.weight": "layers.{}.attention.wv.weight",
        "model.layers.{}.self_attn.o_proj.weight": "layers.{}.attention.wo.weight",
        "model.layers.{}.input_layernorm.weight": "layers.{}.attention_norm.weight",
        "model.layers.{}.post_attention_layernorm.weight": "layers.{}.ffn_norm.weight",
        "model.layers.{}.feed_forward.gate_proj.weight": "layers.{}.feed_forward.w1.weight",
        "model.layers.{}.feed_forward.up_proj.weight": "layers.{}.feed_forward.w3.weight",
        "model.layers.{}.feed_forward.down_proj.weight": "layers.{}.feed_forward.w2.weight",
        "model.layers.{}.feed_forward.router.weight": "layers.{}.moe.router.gate.weight",
        "model.layers.{}.feed_forward.shared_expert.gate_proj.weight": "layers.{}.moe.shared_experts.w1.weight",
        "model.layers.{}.feed_forward.shared_expert.up_proj.weight": "layers.{}.moe.shared_experts.w3.weight",
        "model.layers.{}.feed_forward.shared_expert.down_proj.weight": "layers.{}.moe.shared_experts.w2.weight",
        "model.norm.weight": "norm.weight",
        "lm_head.weight": "output.weight",
    }

    def to_hf(self, state_dict: dict) -> dict:
        rest, out = {}, {}
        for k, v in state_dict.items():
            m = re.fullmatch(r"layers\.(\d+)\.moe\.experts\.w([123])", k)
            if m is None:
                rest[k] = v
                continue
            pre = f"model.layers.{m.group(1)}.feed_forward.experts"
            if m.group(2) == "2":
                out[f"{pre}.down_proj"] = v.transpose(1, 2).contiguous()
            elif m.group(2) == "1":
                w3 = state_dict[f"layers.{m.group(1)}.moe.experts.w3"]
                out[f"{pre}.gate_up_proj"] = torch.cat([v, w3], 1).transpose(1, 2).contiguous()
        out.update(super().to_hf(rest))
        return out

    def from_hf(self, hf_state_dict: dict) -> dict:
        rest, out = {}, {}
        for k, v in hf_state_dict.items():
            m = re.fullmatch(r"model\.layers\.(\d+)\.feed_forward\.experts\.(gate_up_proj|down_proj)", k)
            if m is None:
                rest[k] = v
                continue
            pre = f"layers.{m.group(1)}.moe.experts"
            if m.group(2) == "down_proj":
                out[f"{pre}.w2"] = v.transpose(1, 2).contiguous()
            else:
                w1, w3 = v.transpose(1, 2).chunk(2, dim=1)
                out[f"{pre}.w1"], out[f"{pre}.w3"] = w1.contiguous(), w3.contiguous()
        out.update(super().from_hf(rest))
        return out
