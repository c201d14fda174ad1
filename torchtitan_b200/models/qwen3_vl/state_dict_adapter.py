"""Qwen3-VL <-> Hugging Face ``Qwen3VLForConditionalGeneration`` names (parity:
reference ``models/qwen3_vl/state_dict_adapter.py``).

* Decoder keys are the Qwen3 ones under ``model.language_model.`` (``lm_head`` at the top).
* The vision patch embedding is HF's stride-equals-kernel Conv3d ``[D, C, T, P, P]``;
  here it is the equivalent ``[D, C*T*P*P]`` linear map.
* Both rotary embeddings rotate interleaved pairs here and half-split pairs in HF, so
  the query and key rows (weights and biases) of the vision ``qkv`` projection are
  permuted per head, as the decoder's q/k projections are.
"""
from __future__ import annotations

import re

import torch

from ..qwen3.state_dict_adapter import Qwen3StateDictAdapter

# vision key renames under model.visual. (HF) / vision_encoder. (native)
_TO_NATIVE = [
    (r"^blocks\.(\d+)\.attn\.(qkv|proj)\.", r"blocks.\1.\2."),
    (r"^blocks\.(\d+)\.mlp\.linear_(fc1|fc2)\.", r"blocks.\1.\2."),
    (r"^merger\.linear_(fc1|fc2)\.", r"merger.\1."),
    (r"^deepstack_merger_list\.(\d+)\.linear_(fc1|fc2)\.", r"deepstack_mergers.\1.\2."),
    (r"^deepstack_merger_list\.(\d+)\.norm\.", r"deepstack_mergers.\1.norm."),
]
_TO_HF = [
    (r"^blocks\.(\d+)\.(qkv|proj)\.", r"blocks.\1.attn.\2."),
    (r"^blocks\.(\d+)\.(fc1|fc2)\.", r"blocks.\1.mlp.linear_\2."),
    (r"^merger\.(fc1|fc2)\.", r"merger.linear_\1."),
    (r"^deepstack_mergers\.(\d+)\.(fc1|fc2)\.", r"deepstack_merger_list.\1.linear_\2."),
    (r"^deepstack_mergers\.(\d+)\.norm\.", r"deepstack_merger_list.\1.norm."),
]


def _rename(key: str, rules) -> str:
    for pat, rep in rules:
        new, n = re.subn(pat, rep, key)
        if n:
            return new
    return key


class Qwen3VLStateDictAdapter(Qwen3StateDictAdapter):
    def _qkv_permute(self, t: torch.Tensor, to_hf: bool) -> torch.Tensor:
        a = self.model_args
        dim, h = a.vision_dim, a.vision_heads
        f = self.interleaved_to_halves if to_hf else self.halves_to_interleaved
        t2 = t if t.dim() == 2 else t[:, None]
        q, k, v = t2[:dim], t2[dim:2 * dim], t2[2 * dim:]
        out = torch.cat([f(q, h), f(k, h), v])
        return out if t.dim() == 2 else out[:, 0]

    def from_hf(self, hf_state_dict: dict) -> dict:
        text, out = {}, {}
        for k, v in hf_state_dict.items():
            if k.startswith("model.language_model."):
                text["model." + k[len("model.language_model."):]] = v
            elif k == "lm_head.weight":
                text[k] = v
            elif k.startswith("model.visual."):
                sub = k[len("model.visual."):]
                if sub == "patch_embed.proj.weight":
                    out["vision_encoder.patch_embed.weight"] = v.reshape(v.shape[0], -1)
                    continue
                if sub == "patch_embed.proj.bias":
                    out["vision_encoder.patch_embed.bias"] = v
                    continue
                nk = "vision_encoder." + _rename(sub, _TO_NATIVE)
                out[nk] = self._qkv_permute(v, False) if ".qkv." in nk else v
        out.update(super().from_hf(text))
        return out

    def to_hf(self, state_dict: dict) -> dict:
        a = self.model_args
        text, out = {}, {}
        for k, v in state_dict.items():
            if not k.startswith("vision_encoder."):
                text[k] = v
                continue
            sub = k[len("vision_encoder."):]
            if sub == "patch_embed.weight":
                P, T = a.patch_size, a.temporal_patch_size
                out["model.visual.patch_embed.proj.weight"] = v.reshape(v.shape[0], -1, T, P, P)
                continue
            if sub == "patch_embed.bias":
                out["model.visual.patch_embed.proj.bias"] = v
                continue
            out["model.visual." + _rename(sub, _TO_HF)] = self._qkv_permute(v, True) if ".qkv." in sub else v
        for k, v in super().to_hf(text).items():
            out[k if k == "lm_head.weight" else "model.language_model." + k[len("model."):]] = v
        return out
