"""DeepSeek-V3 <-> Hugging Face ``DeepseekV3ForCausalLM`` names (parity:
reference ``models/deepseek_v3/model/state_dict_adapter.py``).  Both sides rotate
interleaved pairs in the rope slice, so no row permutation is needed; HF's
per-expert 2-D tensors are stacked into ``[E, out, in]``."""
from __future__ import annotations

import re

import torch

from torchtitan_b200.protocols import StateDictAdapter

_EXPERT = re.compile(r"model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight")
_NATIVE = {"gate_proj": "w1", "up_proj": "w3", "down_proj": "w2"}


class DeepSeekV3StateDictAdapter(StateDictAdapter):
    from_hf_map = {
        "model.embed_tokens.weight": "tok_embeddings.weight",
        "model.layers.{}.self_attn.q_proj.weight": "layers.{}.attention.wq.weight",
        "model.layers.{}.self_attn.q_a_proj.weight": "layers.{}.attention.wq_a.weight",
        "model.layers.{}.self_attn.q_a_layernorm.weight": "layers.{}.attention.q_norm.weight",
        "model.layers.{}.self_attn.q_b_proj.weight": "layers.{}.attention.wq_b.weight",
        "model.layers.{}.self_attn.kv_a_proj_with_mqa.weight": "layers.{}.attention.wkv_a.weight",
        "model.layers.{}.self_attn.kv_a_layernorm.weight": "layers.{}.attention.kv_norm.weight",
        "model.layers.{}.self_attn.kv_b_proj.weight": "layers.{}.attention.wkv_b.weight",
        "model.layers.{}.self_attn.o_proj.weight": "layers.{}.attention.wo.weight",
        "model.layers.{}.mlp.gate_proj.weight": "layers.{}.feed_forward.w1.weight",
        "model.layers.{}.mlp.up_proj.weight": "layers.{}.feed_forward.w3.weight",
        "model.layers.{}.mlp.down_proj.weight": "layers.{}.feed_forward.w2.weight",
        "model.layers.{}.mlp.gate.weight": "layers.{}.moe.router.gate.weight",
        "model.layers.{}.mlp.gate.e_score_correction_bias": "layers.{}.moe.expert_bias",
        "model.layers.{}.mlp.shared_experts.gate_proj.weight": "layers.{}.moe.shared_experts.w1.weight",
        "model.layers.{}.mlp.shared_experts.up_proj.weight": "layers.{}.moe.shared_experts.w3.weight",
        "model.layers.{}.mlp.shared_experts.down_proj.weight": "layers.{}.moe.shared_experts.w2.weight",
        "model.layers.{}.input_layernorm.weight": "layers.{}.attention_norm.weight",
        "model.layers.{}.post_attention_layernorm.weight": "layers.{}.ffn_norm.weight",
        "model.norm.weight": "norm.weight",
        "lm_head.weight": "output.weight",
    }

    def from_hf(self, hf_state_dict: dict) -> dict:
        experts: dict[tuple[int, str], dict[int, torch.Tensor]] = {}
        rest = {}
        for k, v in hf_state_dict.items():
            m = _EXPERT.fullmatch(k)
            if m:
                experts.setdefault((int(m.group(1)), _NATIVE[m.group(3)]), {})[int(m.group(2))] = v
            else:
                rest[k] = v
        out = super().from_hf(rest)
        for (layer, name), per in experts.items():
            out[f"layers.{layer}.moe.experts.{name}"] = torch.stack([per[e] for e in sorted(per)])
        return out

    def to_hf(self, state_dict: dict) -> dict:
        inv = {v: k for k, v in _NATIVE.items()}
        rest, out = {}, {}
        for k, v in state_dict.items():
            m = re.fullmatch(r"layers\.(\d+)\.moe\.experts\.(w1|w2|w3)", k)
            if m:
                for e in range(v.shape[0]):
                    out[f"model.layers.{m.group(1)}.mlp.experts.{e}.{inv[m.group(2)]}.weight"] = v[e]
            else:
                rest[k] = v
        out.update(super().to_hf(rest))
        return out
