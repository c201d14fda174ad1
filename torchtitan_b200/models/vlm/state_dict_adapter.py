"""Llama 3 + SigLIP2 <-> Hugging Face names: the decoder as ``LlamaForCausalLM``, the
encoder as ``Siglip2VisionModel`` (``vision_model.*``), the projector under
``multi_modal_projector.*``."""
from __future__ import annotations

from ..llama3.state_dict_adapter import Llama3StateDictAdapter

_ENC = [  # native suffix under encoder. <-> HF suffix under vision_model.
    ("patch_embedding.", "embeddings.patch_embedding."),
    ("position_embedding.", "embeddings.position_embedding."),
    ("post_layernorm.", "post_layernorm."),
]
_BLK = [("layer_norm1.", "layer_norm1."), ("layer_norm2.", "layer_norm2."), ("q_proj.", "self_attn.q_proj."),
        ("k_proj.", "self_attn.k_proj."), ("v_proj.", "self_attn.v_proj."), ("out_proj.", "self_attn.out_proj."),
        ("fc1.", "mlp.fc1."), ("fc2.", "mlp.fc2.")]


def _enc_to_hf(sub: str) -> str:
    for a, b in _ENC:
        if sub.startswith(a):
            return "vision_model." + b + sub[len(a):]
    _, i, rest = sub.split(".", 2)
    for a, b in _BLK:
        if rest.startswith(a):
            return f"vision_model.encoder.layers.{i}.{b}{rest[len(a):]}"
    raise KeyError(sub)


class Llama3Siglip2StateDictAdapter(Llama3StateDictAdapter):
    def to_hf(self, state_dict: dict) -> dict:
        out, text = {}, {}
        for k, v in state_dict.items():
            if k.startswith("encoder."):
                out[_enc_to_hf(k[len("encoder."):])] = v
            elif k.startswith("projector."):
                out["multi_modal_projector." + k[len("projector."):]] = v
            else:
                text[k] = v
        out.update(super().to_hf(text))
        return out

    def from_hf(self, hf_state_dict: dict) -> dict:
        a = self.model_args
        inv = {_enc_to_hf(n): "encoder." + n for n in _native_encoder_keys(a)}
        out, text = {}, {}
        for k, v in hf_state_dict.items():
            if k in inv:
                out[inv[k]] = v
            elif k.startswith("multi_modal_projector."):
                out["projector." + k[len("multi_modal_projector."):]] = v
            elif not k.startswith("vision_model."):
                text[k] = v
        out.update(super().from_hf(text))
        return out


def _native_encoder_keys(a) -> list[str]:
    keys = ["patch_embedding.weight", "patch_embedding.bias", "position_embedding.weight",
            "post_layernorm.weight", "post_layernorm.bias"]
    for i in range(a.vit_layers):
        for n, _ in _BLK:
            keys += [f"layers.{i}.{n}weight", f"layers.{i}.{n}bias"]
    return keys
