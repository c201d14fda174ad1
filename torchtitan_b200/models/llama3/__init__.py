"""Llama 3 family: flavors and the ``ModelSpec`` registry
(parity: ``models/llama3/__init__.py:43-412``)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import Llama3Model, Llama3ModelArgs
from .parallelize import parallelize_llama
from .state_dict_adapter import Llama3StateDictAdapter

llama3_args = {
    "debugmodel": Llama3ModelArgs(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048, rope_theta=500000),
    "debugmodel_flex_attn": Llama3ModelArgs(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048,
                                            rope_theta=500000, mask_type="block_causal"),
    "debugmodel_varlen_attn": Llama3ModelArgs(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048,
                                              rope_theta=500000, mask_type="block_causal"),
    "1B": Llama3ModelArgs(dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn_dim_multiplier=1.5, multiple_of=256,
                          rope_theta=500000, rope_scaling_factor=32.0),
    "3B": Llama3ModelArgs(dim=3072, n_layers=28, n_heads=24, n_kv_heads=8, ffn_dim_multiplier=1.0, multiple_of=256,
                          rope_theta=500000, rope_scaling_factor=32.0),
    "8B": Llama3ModelArgs(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim_multiplier=1.3, multiple_of=1024,
                          rope_theta=500000),
    "70B": Llama3ModelArgs(dim=8192, n_layers=80, n_heads=64, n_kv_heads=8, ffn_dim_multiplier=1.3, multiple_of=4096,
                           rope_theta=500000),
    "405B": Llama3ModelArgs(dim=16384, n_layers=126, n_heads=128, n_kv_heads=8, ffn_dim_multiplier=1.2,
                            multiple_of=4096, rope_theta=500000),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in llama3_args:
        raise ValueError(f"unknown llama3 flavor '{flavor}', available: {sorted(llama3_args)}")
    return ModelSpec(
        name="llama3",
        flavor=flavor,
        model=copy.deepcopy(llama3_args[flavor]),
        parallelize_fn=parallelize_llama,
        pipelining_fn=pipeline_llm,
        build_loss_fn=build_cross_entropy_loss,
        state_dict_adapter=Llama3StateDictAdapter,
    )


__all__ = ["Llama3Model", "Llama3ModelArgs", "model_registry", "llama3_args", "parallelize_llama"]
