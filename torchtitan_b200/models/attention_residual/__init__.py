"""Dense Attention-Residual transformers: flavors and ``ModelSpec`` registry
(parity: reference ``experiments/attention_residual/__init__.py:106-769``; the
Llama-3-shaped flavors).  Pipeline parallelism for these models is not wired
(the residual state between stages is a list of block tensors)."""
from __future__ import annotations

import copy

from torchtitan_b200.components.loss import build_cross_entropy_loss
from torchtitan_b200.models.llama3.parallelize import parallelize_llama
from torchtitan_b200.parallel.pipeline import pipeline_llm
from torchtitan_b200.protocols import ModelSpec

from .model import AttnResModel, AttnResModelArgs

A = AttnResModelArgs
attn_res_args = {
    "debugmodel": A(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048, rope_theta=500000,
                    attn_res_blocks=3),
    "debugmodel_full": A(dim=256, n_layers=6, n_heads=16, n_kv_heads=8, vocab_size=2048, rope_theta=500000,
                         attn_res_blocks=6),
    "1B": A(dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn_dim_multiplier=1.5, multiple_of=256,
            rope_theta=500000, attn_res_blocks=8),
    "8B": A(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim_multiplier=1.3, multiple_of=1024,
            rope_theta=500000, attn_res_blocks=8),
}


def model_registry(flavor: str) -> ModelSpec:
    if flavor not in attn_res_args:
        raise ValueError(f"unknown attention_residual flavor '{flavor}', available: {sorted(attn_res_args)}")
    return ModelSpec(name="attention_residual", flavor=flavor, model=copy.deepcopy(attn_res_args[flavor]),
                     parallelize_fn=parallelize_llama, pipelining_fn=pipeline_llm, build_loss_fn=build_cross_entropy_loss)


__all__ = ["AttnResModel", "AttnResModelArgs", "model_registry", "attn_res_args"]
