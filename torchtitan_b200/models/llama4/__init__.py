"""Llama 4 family: flavors and the ``ModelSpec`` registry (parity: reference
``models/llama4/__init__.py``; 17bx16e = Scout, 17bx128e = Maverick shapes)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.parallel.parallelize_decoder import parallelize_decoder
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import Llama4Model, Llama4ModelArgs
from .state_dict_adapter import Llama4StateDictAdapter

A = Llama4ModelArgs
llama4_args = {
    "debugmodel": A(dim=256, n_layers=8, n_heads=16, n_kv_heads=8, vocab_size=2048, multiple_of=256,
                    ffn_dim_multiplier=None, rope_scaling_factor=8.0, max_seq_len=4096, fixed_attn_block_size=256,
                    num_experts=8, interleave_moe_layer_step=2),
    "17bx16e": A(dim=5120, n_layers=48, n_heads=40, n_kv_heads=8, ffn_dim_multiplier=1.2, multiple_of=2048,
                 rope_theta=500000, num_experts=16, interleave_moe_layer_step=1),
    "17bx128e": A(dim=5120, n_layers=48, n_heads=40, n_kv_heads=8, ffn_dim_multiplier=1.2, multiple_of=2048,
                  rope_theta=500000, num_experts=128, interleave_moe_layer_step=2),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in llama4_args:
        raise ValueError(f"unknown llama4 flavor '{flavor}', available: {sorted(llama4_args)}")
    from torchtitan_b200.components.optimizer import build_optimizers_with_moe_load_balancing

    return ModelSpec(name="llama4", flavor=flavor, model=copy.deepcopy(llama4_args[flavor]),
                     parallelize_fn=parallelize_decoder, pipelining_fn=pipeline_llm,
                     build_loss_fn=build_cross_entropy_loss,
                     post_optimizer_build_fn=build_optimizers_with_moe_load_balancing,
                     state_dict_adapter=Llama4StateDictAdapter)


__all__ = ["Llama4Model", "Llama4ModelArgs", "model_registry", "llama4_args"]
