"""Qwen3 <-> Hugging Face ``Qwen3ForCausalLM`` / ``Qwen3MoeForCausalLM`` names.

q/k rows are permuted between HF's rotate-half layout and this framework's
interleaved RoPE pairs (as for Llama 3); the per-head q/k norm weights are
permuted the same way because they scale the same head-dim features.  HF MoE
stores one 2-D tensor per expert; they are stacked into ``[E, out, in]``.
"""
from __future__ import annotations

import re

import torch

from torchtitan_b200.models.llama3.state_dict_adapter import Llama3StateDictAdapter

_EXPERT = re.compile(r"model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.weight")
_NATIVE_EXPERT = {"gate_proj": "w1", "up_proj": "w3", "down_proj": "w2"}


class Qwen3StateDictAdapter(Llama3StateDictAdapter):
    from_hf_map = dict(Llama3StateDictAdapter.from_hf_map)
    from_hf_map.update({
        "model.layers.{}.self_attn.q_norm.weight": "layers.{}.attention.q_norm.weight",
        "model.layers.{}.self_attn.k_norm.weight": "layers.{}.attention.k_norm.weight",
        "model.layers.{}.mlp.gate.weight": "layers.{}.moe.router.gate.weight",
    })

    def _heads(self, key: str) -> int | None:
        if key.endswith(("attention.q_norm.weight", "attention.k_norm.weight")):
            return 1
        return super()._heads(key)

    def to_hf_tensor(self, native_key, t):
        h = self._heads(native_key)
        if h == 1:
            return self.interleaved_to_halves(t[:, None], 1)[:, 0]
        return super().to_hf_tensor(native_key, t)

    def from_hf_tensor(self, native_key, t):
        h = self._heads(native_key)
        if h == 1:
            return self.halves_to_interleaved(t[:, None], 1)[:, 0]
        return super().from_hf_tensor(native_key, t)

    def from_hf(self, hf_state_dict: dict) -> dict:
        experts: dict[tuple[int, str], dict[int, torch.Tensor]] = {}
        rest = {}
        for k, v in hf_state_dict.items():
            m = _EXPERT.fullmatch(k)
            if m:
                experts.setdefault((int(m.group(1)), _NATIVE_EXPERT[m.group(3)]), {})[int(m.group(2))] = v
            else:
                rest[k] = v
        out = super().from_hf(rest)
        for (layer, name), per in experts.items():
            out[f"layers.{layer}.moe.experts.{name}"] = torch.stack([per[e] for e in sorted(per)])
        return out

    def to_hf(self, state_dict: dict) -> dict:
        rest, out = {}, {}
        inv = {v: k for k, v in _NATIVE_EXPERT.items()}
        for k, v in state_dict.items():
            m = re.fullmatch(r"layers\.(\d+)\.moe\.experts\.(w1|w2|w3)", k)
            if m:
                for e in range(v.shape[0]):
                    out[f"model.layers.{m.group(1)}.mlp.experts.{e}.{inv[m.group(2)]}.weight"] = v[e]
            elif k.endswith("moe.expert_bias"):
                continue
            else:
                rest[k] = v
        out.update(super().to_hf(rest))
        return out
