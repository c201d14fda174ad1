"""Llama 3 + SigLIP2 vision-language models (parity: reference ``experiments/vlm``).
``debugmodel`` matches the reference's debug sizes; ``8B_so400m`` pairs Llama 3 8B with
the SigLIP2 so400m/16 encoder."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.protocols import ModelSpec

from .model import Llama3Siglip2, Llama3Siglip2Args
from .parallelize import parallelize_vlm
from .state_dict_adapter import Llama3Siglip2StateDictAdapter

A = Llama3Siglip2Args
vlm_args = {
    "debugmodel": A(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048, image_token_id=2047,
                    vit_dim=128, vit_ffn_dim=256, vit_layers=4, vit_heads=2, patch_size=16, n_pos_embs=16),
    "8B_so400m": A(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim_multiplier=1.3, multiple_of=1024,
                   image_token_id=128256 - 1, vit_dim=1152, vit_ffn_dim=4304, vit_layers=27, vit_heads=16,
                   patch_size=16, n_pos_embs=16),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in vlm_args:
        raise ValueError(f"unknown vlm flavor '{flavor}', available: {sorted(vlm_args)}")
    return ModelSpec(name="vlm", flavor=flavor, model=copy.deepcopy(vlm_args[flavor]),
                     parallelize_fn=parallelize_vlm, pipelining_fn=None, build_loss_fn=build_cross_entropy_loss,
                     state_dict_adapter=Llama3Siglip2StateDictAdapter)


__all__ = ["Llama3Siglip2", "Llama3Siglip2Args", "model_registry", "vlm_args"]
