"""FLUX transformer <-> Hugging Face ``diffusers`` ``FluxTransformer2DModel`` names
(parity: reference ``models/flux/model/state_dict_adapter.py``).

* diffusers splits the fused projections: image/text ``qkv`` into ``to_q/k/v`` and
  ``add_q/k/v_proj``, the single-stream ``linear1`` into ``to_q/k/v`` + ``proj_mlp``;
* the final adaptive norm stores (scale, shift) where this model stores (shift, scale).
"""
from __future__ import annotations

import re

import torch

from torchtitan_b200.protocols import StateDictAdapter

_DIRECT = {  # HF key (``{}`` = block index) -> native key
    "x_embedder.{w}": "img_in.{w}",
    "context_embedder.{w}": "txt_in.{w}",
    "time_text_embed.timestep_embedder.linear_1.{w}": "time_in.in_layer.{w}",
    "time_text_embed.timestep_embedder.linear_2.{w}": "time_in.out_layer.{w}",
    "time_text_embed.text_embedder.linear_1.{w}": "vector_in.in_layer.{w}",
    "time_text_embed.text_embedder.linear_2.{w}": "vector_in.out_layer.{w}",
    "norm_out.linear.{w}": "final_layer.adaLN_modulation.{w}",
    "proj_out.{w}": "final_layer.linear.{w}",
    "transformer_blocks.{}.norm1.linear.{w}": "double_blocks.{}.img_mod.lin.{w}",
    "transformer_blocks.{}.norm1_context.linear.{w}": "double_blocks.{}.txt_mod.lin.{w}",
    "transformer_blocks.{}.attn.to_out.0.{w}": "double_blocks.{}.img_attn.proj.{w}",
    "transformer_blocks.{}.attn.to_add_out.{w}": "double_blocks.{}.txt_attn.proj.{w}",
    "transformer_blocks.{}.ff.net.0.proj.{w}": "double_blocks.{}.img_mlp.fc1.{w}",
    "transformer_blocks.{}.ff.net.2.{w}": "double_blocks.{}.img_mlp.fc2.{w}",
    "transformer_blocks.{}.ff_context.net.0.proj.{w}": "double_blocks.{}.txt_mlp.fc1.{w}",
    "transformer_blocks.{}.ff_context.net.2.{w}": "double_blocks.{}.txt_mlp.fc2.{w}",
    "transformer_blocks.{}.attn.norm_q.weight": "double_blocks.{}.img_attn.norm.query_norm.weight",
    "transformer_blocks.{}.attn.norm_k.weight": "double_blocks.{}.img_attn.norm.key_norm.weight",
    "transformer_blocks.{}.attn.norm_added_q.weight": "double_blocks.{}.txt_attn.norm.query_norm.weight",
    "transformer_blocks.{}.attn.norm_added_k.weight": "double_blocks.{}.txt_attn.norm.key_norm.weight",
    "single_transformer_blocks.{}.norm.linear.{w}": "single_blocks.{}.modulation.lin.{w}",
    "single_transformer_blocks.{}.proj_out.{w}": "single_blocks.{}.linear2.{w}",
    "single_transformer_blocks.{}.attn.norm_q.weight": "single_blocks.{}.norm.query_norm.weight",
    "single_transformer_blocks.{}.attn.norm_k.weight": "single_blocks.{}.norm.key_norm.weight",
}
_FUSED = {  # native key -> HF parts in concatenation order
    "double_blocks.{}.img_attn.qkv.{w}": ["transformer_blocks.{}.attn.to_q.{w}", "transformer_blocks.{}.attn.to_k.{w}",
                                          "transformer_blocks.{}.attn.to_v.{w}"],
    "double_blocks.{}.txt_attn.qkv.{w}": ["transformer_blocks.{}.attn.add_q_proj.{w}",
                                          "transformer_blocks.{}.attn.add_k_proj.{w}",
                                          "transformer_blocks.{}.attn.add_v_proj.{w}"],
    "single_blocks.{}.linear1.{w}": ["single_transformer_blocks.{}.attn.to_q.{w}",
                                     "single_transformer_blocks.{}.attn.to_k.{w}",
                                     "single_transformer_blocks.{}.attn.to_v.{w}",
                                     "single_transformer_blocks.{}.proj_mlp.{w}"],
}
_SWAP = "final_layer.adaLN_modulation."


def _pattern(template: str) -> re.Pattern:
    p = re.escape(template).replace(r"\{\}", r"(?P<i>\d+)").replace(r"\{w\}", r"(?P<w>weight|bias)")
    return re.compile(p + "$")


def _fill(template: str, m: re.Match) -> str:
    d = m.groupdict()
    return template.replace("{}", d.get("i") or "").replace("{w}", d.get("w") or "")


def _swap_halves(t: torch.Tensor) -> torch.Tensor:
    a, b = t.chunk(2, dim=0)
    return torch.cat([b, a], 0)


class FluxStateDictAdapter(StateDictAdapter):
    def _sizes(self, native_template: str) -> list[int]:
        a = self.model_args
        h = a.hidden_size
        return [h, h, h, int(h * a.mlp_ratio)] if native_template.startswith("single") else [h, h, h]

    def to_hf(self, state_dict: dict) -> dict:
        out = {}
        direct = [(_pattern(n), hf) for hf, n in _DIRECT.items()]
        fused = [(_pattern(n), n, parts) for n, parts in _FUSED.items()]
        for k, v in state_dict.items():
            for pat, hf in direct:
                m = pat.match(k)
                if m:
                    out[_fill(hf, m)] = _swap_halves(v) if k.startswith(_SWAP) else v
                    break
            else:
                for pat, n, parts in fused:
                    m = pat.match(k)
                    if m:
                        for part, t in zip(parts, torch.split(v, self._sizes(n), 0)):
                            out[_fill(part, m)] = t
                        break
                else:
                    raise KeyError(f"flux: no Hugging Face name for {k}")
        return out

    def from_hf(self, hf_state_dict: dict) -> dict:
        out = {}
        direct = [(_pattern(hf), n) for hf, n in _DIRECT.items()]
        for k, v in hf_state_dict.items():
            for pat, n in direct:
                m = pat.match(k)
                if m:
                    nk = _fill(n, m)
                    out[nk] = _swap_halves(v) if nk.startswith(_SWAP) else v
                    break
        for n, parts in _FUSED.items():
            first = _pattern(parts[0])
            for k in hf_state_dict:
                m = first.match(k)
                if m:
                    out[_fill(n, m)] = torch.cat([hf_state_dict[_fill(p, m)] for p in parts], 0)
        return out
